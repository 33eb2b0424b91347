"""GPU parity of the pre-MoE rows (residual add + RMS normalisation + router MatMul) and
of the composed block norm_router -> MoE layer against the oracle."""

import numpy as np
import pytest

from gpu_util import TOL, as_np, to_dev, torch_dtype

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype_name", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("H,E", [(256, 8), (4096, 8), (1000, 64), (2048, 130)])
@pytest.mark.parametrize("with_skip", [False, True])
def test_norm_router_matches_oracle(pkg, orc, dev, dtype_name, H, E, with_skip):
    import torch
    rng = np.random.default_rng(H + E)
    T = 333
    x = rng.standard_normal((T, H)).astype(np.float32)
    skip = rng.standard_normal((T, H)).astype(np.float32) if with_skip else None
    gamma = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    wr = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    dt = torch_dtype(dtype_name)
    dx, dw = to_dev(x, dev, dt), to_dev(wr, dev, dt)
    ds = None if skip is None else to_dev(skip, dev, dt)
    normed, logits, residual = pkg.norm_router(dx, to_dev(gamma, dev), 1e-6, dw, skip=ds)
    torch.cuda.synchronize()
    hx = as_np(dx).astype(np.float32)
    hs = None if ds is None else as_np(ds).astype(np.float32)
    odt = "bfloat16" if dtype_name == "bfloat16" else np.dtype(dtype_name)
    rn, rl, rr = orc.norm_router(hx, gamma, 1e-6, as_np(dw).astype(np.float32), skip=hs, dtype=odt)
    tol = dict(rtol=1e-5, atol=1e-6) if dtype_name == "float32" else TOL[dtype_name]
    np.testing.assert_allclose(as_np(normed), rn, **tol)
    np.testing.assert_allclose(as_np(logits), rl, **tol)
    if with_skip:
        np.testing.assert_allclose(as_np(residual), rr, **tol)


def test_norm_router_then_moe_block(pkg, orc, dev):
    """hidden -> (skip add, RMS norm, router) -> MoE layer, each step on the GPU, against the
    oracle composition.  The MoE consumes the GPU's own normalised rows and logits."""
    import torch
    T, H, I, E, k = 200, 512, 384, 8, 2
    inp = orc.make_moe_inputs(T=T, H=H, I=I, E=E, k=k, act="silu", gated=True,
                              dtype="float32", seed=17)
    rng = np.random.default_rng(18)
    skip = rng.standard_normal((T, H)).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    wr = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
    dt = torch.float16
    dx, ds, dw = to_dev(inp["x"], dev, dt), to_dev(skip, dev, dt), to_dev(wr, dev, dt)
    normed, logits, residual = pkg.norm_router(dx, to_dev(gamma, dev), 1e-5, dw, skip=ds)
    op = pkg.MoE(**inp["attrs"])
    w = {n: to_dev(inp[n], dev, dt) for n in ("fc1_w", "fc2_w", "fc3_w")}
    out = op([normed, logits, w["fc1_w"], None, w["fc2_w"], None, w["fc3_w"], None])
    op.release()
    torch.cuda.synchronize()
    # Oracle: routing and the experts on the GPU's normed rows and logits (the rounded
    # intermediate tensors are checked separately above).
    ref = orc.moe(as_np(normed), as_np(logits), as_np(w["fc1_w"]), None, as_np(w["fc2_w"]),
                  None, as_np(w["fc3_w"]), None, **inp["attrs"])
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])
    rn, rl, _ = orc.norm_router(as_np(dx).astype(np.float32), gamma, 1e-5,
                                as_np(dw).astype(np.float32),
                                skip=as_np(ds).astype(np.float32), dtype=np.float16)
    np.testing.assert_allclose(as_np(normed), rn, **TOL["float16"])
    np.testing.assert_allclose(as_np(logits), rl, **TOL["float16"])


def test_norm_router_rejects_bad_shapes(pkg, dev):
    import torch
    x = torch.zeros(4, 100, dtype=torch.float16, device=dev)
    with pytest.raises(pkg.InvalidArgument):
        pkg.norm_router(x, torch.ones(100, device=dev), 1e-6,
                        torch.zeros(8, 100, dtype=torch.float16, device=dev))
