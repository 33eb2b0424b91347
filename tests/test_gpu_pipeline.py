"""Host-buffer call pipeline (moe_b200_pipeline_*): calls on pinned host tensors give the
bit-identical outputs of the device-side forward on the same inputs, for ragged row
counts (including an empty call) and any pipeline depth."""

import numpy as np
import pytest

from gpu_util import to_dev

pytestmark = pytest.mark.gpu


def _device_forward(pkg, prob_args, weights, x, lg, dev):
    import torch
    prob = pkg.make_problem(x.shape[0], *prob_args[0], **prob_args[1])
    out = torch.empty_like(x)
    ws = torch.empty(max(pkg.workspace_size(prob), 256), dtype=torch.uint8, device=dev)
    pkg.forward(prob, dict(weights, input=x, router_probs=lg, output=out), ws)
    torch.cuda.synchronize(dev)
    return out.cpu()


@pytest.mark.parametrize("depth", [1, 3])
def test_pipeline_moe_matches_device_forward(pkg, orc, dev, depth):
    import torch
    H, I, E, k, Tmax = 256, 384, 8, 2, 300
    inp = orc.make_moe_inputs(T=Tmax, H=H, I=I, E=E, k=k, act="silu", gated=True,
                              dtype="float32", bias=True, seed=61)
    h = lambda n: torch.from_numpy(inp[n]).half()
    weights = dict(fc1_weights=h("fc1_w").to(dev), fc1_bias=h("fc1_b").to(dev),
                   fc2_weights=h("fc2_w").to(dev), fc2_bias=h("fc2_b").to(dev),
                   fc3_weights=h("fc3_w").to(dev), fc3_bias=h("fc3_b").to(dev))
    prob_args = ((H, I, E, pkg.FLOAT16), dict(has_fc3=True, **inp["attrs"]))
    prob = pkg.make_problem(Tmax, *prob_args[0], **prob_args[1])
    g = torch.Generator().manual_seed(7)
    rows = [300, 17, 0, 300, 128, 1]
    calls = []
    with pkg.Pipeline(prob, weights, depth=depth) as pl:
        for r in rows:
            hx = torch.randn(r, H, generator=g).half().pin_memory()
            hl = torch.randn(r, E, generator=g).half().pin_memory()
            ho = torch.full((r, H), float("nan"), dtype=torch.float16).pin_memory()
            pl.submit(hx, hl, ho)
            calls.append((hx, hl, ho))
        pl.synchronize()
        with pytest.raises(pkg.InvalidArgument):
            big = torch.zeros(Tmax + 1, H, dtype=torch.float16)
            pl.submit(big, torch.zeros(Tmax + 1, E, dtype=torch.float16), big)
    for hx, hl, ho in calls:
        if hx.shape[0] == 0:
            continue
        ref = _device_forward(pkg, prob_args, weights, hx.to(dev), hl.to(dev), dev)
        assert torch.equal(ho, ref)


def test_pipeline_qmoe_matches_device_forward(pkg, orc, dev):
    import torch
    T, H, I, E, k = 96, 256, 256, 8, 2
    q = orc.make_qmoe_inputs(T=T, H=H, I=I, E=E, k=k, bits=4, block_size=64,
                             scale_mu=-5.0, scale_sigma=0.3, seed=62)
    weights = dict(fc1_weights=to_dev(q["fc1_q"], dev), fc1_scales=to_dev(q["fc1_scales"], dev),
                   fc2_weights=to_dev(q["fc2_q"], dev), fc2_scales=to_dev(q["fc2_scales"], dev),
                   fc3_weights=to_dev(q["fc3_q"], dev), fc3_scales=to_dev(q["fc3_scales"], dev))
    prob_args = ((H, I, E, pkg.FLOAT16), dict(has_fc3=True, **q["attrs"]))
    prob = pkg.make_problem(T, *prob_args[0], **prob_args[1])
    hx = torch.from_numpy(q["x"]).pin_memory()
    hl = torch.from_numpy(q["router_probs"]).pin_memory()
    outs = [torch.empty(T, H, dtype=torch.float16).pin_memory() for _ in range(3)]
    with pkg.Pipeline(prob, weights, depth=2) as pl:
        for o in outs:
            pl.submit(hx, hl, o)
        pl.synchronize()
    ref = _device_forward(pkg, prob_args, weights, hx.to(dev), hl.to(dev), dev)
    for o in outs:
        assert torch.equal(o, ref)
    want = orc.qmoe(q["x"], q["router_probs"], q["fc1_q"], q["fc1_scales"], None, q["fc2_q"],
                    q["fc2_scales"], None, q["fc3_q"], q["fc3_scales"], None, **q["attrs"])
    np.testing.assert_allclose(outs[0].float().numpy(), want, rtol=2e-2, atol=2e-3)
