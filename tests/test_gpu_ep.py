"""GPU tests of the expert-parallel path through the C ABI (dispatch, expert FFN on
received rows, combine), single process and, where two GPUs exist, two NCCL ranks."""

import os
import socket

import numpy as np
import pytest

from gpu_util import TOL, as_np, to_dev

pytestmark = pytest.mark.gpu


def _moe_case(orc, dev, T, H, I, E, k, seed, dtype):
    import torch
    inp = orc.make_moe_inputs(T=T, H=H, I=I, E=E, k=k, act="silu", gated=True, dtype="float32",
                              bias=True, normalize=1, seed=seed)
    dt = getattr(torch, dtype)
    d = {n: to_dev(inp[n], dev, dt) for n in ("x", "router_probs", "fc1_w", "fc1_b", "fc2_w",
                                                "fc2_b", "fc3_w", "fc3_b")}
    weights = dict(fc1_weights=d["fc1_w"], fc1_bias=d["fc1_b"], fc2_weights=d["fc2_w"],
                   fc2_bias=d["fc2_b"], fc3_weights=d["fc3_w"], fc3_bias=d["fc3_b"])
    return d, weights, inp["attrs"]


@pytest.mark.parametrize("dtype,transport", [("float16", "p2p"), ("bfloat16", "p2p"),
                                             ("float16", "collective"),
                                             ("float32", "collective")])
def test_ep_single_rank_matches_layer(pkg, orc, dev, dtype, transport):
    from onnxruntime_musa_b200 import ep
    d, weights, attrs = _moe_case(orc, dev, 300, 256, 384, 8, 2, 21, dtype)
    et = {"float16": pkg.FLOAT16, "bfloat16": pkg.BFLOAT16, "float32": pkg.FLOAT}[dtype]
    layer = ep.ExpertParallelMoE(pkg, num_experts=8, hidden_size=256, inter_size=384, dtype=et,
                                 has_fc3=True, local_weights=weights, transport=transport,
                                 **attrs)
    assert layer.transport == transport
    out = layer.forward(d["x"], d["router_probs"])
    op = pkg.MoE(**attrs)
    ref = op([d["x"], d["router_probs"], d["fc1_w"], d["fc1_b"], d["fc2_w"], d["fc2_b"],
              d["fc3_w"], d["fc3_b"]])
    op.release()
    np.testing.assert_allclose(as_np(out), as_np(ref), **TOL[dtype])


@pytest.mark.parametrize("T", [4, 400])  # decode kernels and dequantise + GEMM
def test_ep_single_rank_qmoe(pkg, orc, dev, T):
    from onnxruntime_musa_b200 import ep
    q = orc.make_qmoe_inputs(T=T, H=256, I=256, E=8, k=2, bits=4, block_size=128,
                             scale_mu=-5.0, scale_sigma=0.3, seed=T)
    g = lambda n: to_dev(q[n], dev)
    attrs = q["attrs"]
    weights = dict(fc1_weights=g("fc1_q"), fc1_scales=g("fc1_scales"), fc2_weights=g("fc2_q"),
                   fc2_scales=g("fc2_scales"), fc3_weights=g("fc3_q"), fc3_scales=g("fc3_scales"))
    layer = ep.ExpertParallelMoE(pkg, num_experts=8, hidden_size=256, inter_size=256,
                                 dtype=pkg.FLOAT16, has_fc3=True, local_weights=weights, **attrs)
    out = layer.forward(g("x"), g("router_probs"))
    ref = orc.qmoe(q["x"], q["router_probs"], q["fc1_q"], q["fc1_scales"], None, q["fc2_q"],
                   q["fc2_scales"], None, q["fc3_q"], q["fc3_scales"], None, **attrs)
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_ep_p2p_single_rank_ragged_calls(pkg, orc, dev):
    """Device-side exchange on one rank: successive calls with different row counts
    (including none) against the single-device layer; the output is bit-identical to the
    plain layer's (same kernels, same summation order)."""
    import torch
    from onnxruntime_musa_b200 import ep
    d, weights, attrs = _moe_case(orc, dev, 600, 256, 512, 16, 4, 23, "float16")
    layer = ep.ExpertParallelMoE(pkg, num_experts=16, hidden_size=256, inter_size=512,
                                 dtype=pkg.FLOAT16, has_fc3=True, local_weights=weights,
                                 transport="p2p", max_rows=600, **attrs)
    op = pkg.MoE(**attrs)
    for T in (600, 1, 0, 257, 600):
        x, lg = d["x"][:T].contiguous(), d["router_probs"][:T].contiguous()
        out = layer.forward(x, lg)
        ref = op([x, lg, d["fc1_w"], d["fc1_b"], d["fc2_w"], d["fc2_b"], d["fc3_w"], d["fc3_b"]])
        torch.cuda.synchronize()
        assert out.shape == (T, 256)
        np.testing.assert_allclose(as_np(out), as_np(ref), **TOL["float16"])
    op.release()
    with pytest.raises(ValueError):
        layer.forward(d["x"][:1].repeat(601, 1), d["router_probs"][:1].repeat(601, 1))
    layer.close()


def _nccl_worker(rank, world, port, q, transport="p2p", E=8):
    import torch
    import torch.distributed as dist
    import __graft_entry__ as ge
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        pkg, orc = ge.load_package(), ge.load_oracle()
        from onnxruntime_musa_b200 import ep
        d, weights, attrs = _moe_case(orc, dev, 512, 512, 256, E, 2, 33 + E, "float16")
        T_r = 256
        xs, ls = d["x"][rank * T_r:(rank + 1) * T_r], d["router_probs"][rank * T_r:(rank + 1) * T_r]
        layer = ep.ExpertParallelMoE(pkg, num_experts=E, hidden_size=512, inter_size=256,
                                     dtype=pkg.FLOAT16, has_fc3=True,
                                     local_weights=ep.shard_experts(weights, rank, world),
                                     transport=transport, **attrs)
        # Ragged per-rank calls: rank 1 sends fewer rows on the second call.
        out = layer.forward(xs.contiguous(), ls.contiguous())
        T2 = T_r if rank == 0 else 100
        out2 = layer.forward(xs[:T2].contiguous(), ls[:T2].contiguous())
        op = pkg.MoE(**attrs)
        ref = op([xs.contiguous(), ls.contiguous(), d["fc1_w"], d["fc1_b"], d["fc2_w"],
                  d["fc2_b"], d["fc3_w"], d["fc3_b"]])
        torch.cuda.synchronize()
        err = np.abs(as_np(out) - as_np(ref)) - (TOL["float16"]["atol"] +
                                                 TOL["float16"]["rtol"] * np.abs(as_np(ref)))
        err2 = np.abs(as_np(out2) - as_np(ref)[:T2]) - (
            TOL["float16"]["atol"] + TOL["float16"]["rtol"] * np.abs(as_np(ref)[:T2]))
        if hasattr(layer, "close"):
            layer.close()
        q.put((rank, float(max(err.max(), err2.max()))))
    except Exception as exc:
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport,E", [("p2p", 8), ("collective", 8), ("p2p", 2)],
                         ids=["p2p", "collective", "p2p_one_expert_per_rank"])
def test_ep_two_ranks(transport, E):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q, transport, E))
             for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        assert res[r] <= 0, f"rank {r} exceeds the fp16 tolerance by {res[r]}"


def test_ep_host_pipeline(pkg, orc, dev):
    """ep.HostPipeline: calls on pinned host tensors give the layer's own outputs."""
    import torch
    from onnxruntime_musa_b200 import ep
    d, weights, attrs = _moe_case(orc, dev, 256, 256, 384, 8, 2, 24, "float16")
    layer = ep.ExpertParallelMoE(pkg, num_experts=8, hidden_size=256, inter_size=384,
                                 dtype=pkg.FLOAT16, has_fc3=True, local_weights=weights,
                                 **attrs)
    pipe = ep.HostPipeline(layer, 256, torch.float16, dev, depth=2)
    g = torch.Generator().manual_seed(3)
    calls = []
    for T in (256, 100, 256, 7):
        hx = torch.randn(T, 256, generator=g).half().pin_memory()
        hl = torch.randn(T, 8, generator=g).half().pin_memory()
        ho = torch.empty(T, 256, dtype=torch.float16).pin_memory()
        pipe.submit(hx, hl, ho)
        calls.append((hx, hl, ho))
    pipe.synchronize()
    for hx, hl, ho in calls:
        ref = layer.forward(hx.to(dev), hl.to(dev)).cpu()
        assert torch.equal(ho, ref)
    layer.close()


def test_ep_connect_rejects_mismatched_regions(pkg, dev):
    """Two communicators of one 2-rank job whose regions differ (max_rows 64 against 128):
    connect refuses the peer's handle before it opens it (no peer memory is touched)."""
    import ctypes
    a = pkg.EpComm(0, 2, 64, 2, 256, 8, pkg.FLOAT16)
    b = pkg.EpComm(1, 2, 128, 2, 256, 8, pkg.FLOAT16)
    try:
        ha, hb = a.handle(), b.handle()
        n = ctypes.c_size_t()
        assert pkg.lib().moe_b200_ep_comm_handle_size(ctypes.byref(n)) == 0
        assert len(ha) == len(hb) == n.value > 64  # IPC handle + region description
        with pytest.raises(pkg.MoeB200Error, match="same arguments"):
            a.connect([ha, hb])
        with pytest.raises(pkg.MoeB200Error, match="same arguments"):
            b.connect([ha, hb])
        # a handle in the wrong rank slot is refused too
        c = pkg.EpComm(1, 2, 64, 2, 256, 8, pkg.FLOAT16)
        try:
            with pytest.raises(pkg.MoeB200Error, match="not a moe_b200_ep_comm handle"):
                a.connect([ha, ha])
        finally:
            c.close()
    finally:
        a.close()
        b.close()
