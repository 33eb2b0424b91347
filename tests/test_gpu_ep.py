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


@pytest.mark.parametrize("transport", ["p2p", "collective"])
@pytest.mark.parametrize("T,bits,bs", [(4, 4, 128), (400, 4, 128), (400, 8, 0), (37, 8, 0)],
                         ids=["T4_int4_bs128", "T400_int4_bs128", "T400_int8_row", "T37_int8_row"])
def test_ep_single_rank_qmoe(pkg, orc, dev, transport, T, bits, bs):
    """QMoE through both transports on one rank (p2p: codes converted inside the pair GEMM
    on the received rows; collective: the single-device QMoE steps) against the oracle."""
    from onnxruntime_musa_b200 import ep
    q = orc.make_qmoe_inputs(T=T, H=256, I=256, E=8, k=2, bits=bits, block_size=bs,
                             scale_mu=-5.0 if bits == 4 else -8.5, scale_sigma=0.3, seed=T + bits)
    g = lambda n: to_dev(q[n], dev)
    attrs = q["attrs"]
    weights = dict(fc1_weights=g("fc1_q"), fc1_scales=g("fc1_scales"), fc2_weights=g("fc2_q"),
                   fc2_scales=g("fc2_scales"), fc3_weights=g("fc3_q"), fc3_scales=g("fc3_scales"))
    layer = ep.ExpertParallelMoE(pkg, num_experts=8, hidden_size=256, inter_size=256,
                                 dtype=pkg.FLOAT16, has_fc3=True, local_weights=weights,
                                 transport=transport, **attrs)
    assert layer.transport == transport
    out = layer.forward(g("x"), g("router_probs"))
    ref = orc.qmoe(q["x"], q["router_probs"], q["fc1_q"], q["fc1_scales"], None, q["fc2_q"],
                   q["fc2_scales"], None, q["fc3_q"], q["fc3_scales"], None, **attrs)
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])
    if hasattr(layer, "close"):
        layer.close()


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


def test_ep_p2p_dedup_dispatch_is_bit_identical(pkg, orc, dev):
    """k >= 4: each token crosses to a rank once and the receiver gathers its expert rows
    locally (MOE_B200_EP_DEDUP); the expert rows, and so the outputs, are the same bits as
    with one copy per (token, expert)."""
    import torch
    from onnxruntime_musa_b200 import ep
    d, weights, attrs = _moe_case(orc, dev, 500, 256, 384, 16, 8, 29, "float16")
    outs = []
    for flag in ("1", "0"):
        os.environ["MOE_B200_EP_DEDUP"] = flag
        try:
            layer = ep.ExpertParallelMoE(pkg, num_experts=16, hidden_size=256, inter_size=384,
                                         dtype=pkg.FLOAT16, has_fc3=True, local_weights=weights,
                                         transport="p2p", **attrs)
            outs.append(layer.forward(d["x"], d["router_probs"]))
            outs.append(layer.forward(d["x"][:123].contiguous(), d["router_probs"][:123].contiguous()))
            torch.cuda.synchronize()
            layer.close()
        finally:
            del os.environ["MOE_B200_EP_DEDUP"]
    assert torch.equal(outs[0], outs[2]) and torch.equal(outs[1], outs[3])
    h = {n: as_np(v) for n, v in d.items()}
    ref = orc.moe(h["x"], h["router_probs"], h["fc1_w"], h["fc1_b"], h["fc2_w"], h["fc2_b"],
                  h["fc3_w"], h["fc3_b"], **attrs)
    np.testing.assert_allclose(as_np(outs[0]), ref, **TOL["float16"])


def _nccl_worker(rank, world, port, q, transport="p2p", E=8, kind="moe"):
    """One rank of a `world`-rank expert-parallel layer over NCCL (device-side p2p exchange
    or NCCL all-to-all).  Each rank routes its own tokens; two calls, the second ragged
    (rank 1 sends fewer rows).  Both outputs are checked against the oracle."""
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
        T_r = 256
        if kind in ("moe", "moe_k8"):
            d, weights, attrs = _moe_case(orc, dev, T_r * world, 512, 256, E,
                                          8 if kind == "moe_k8" else 2, 33 + E, "float16")
            h = {n: as_np(v) for n, v in d.items()}
            ref_fn = lambda x, lg: orc.moe(x, lg, h["fc1_w"], h["fc1_b"], h["fc2_w"],
                                           h["fc2_b"], h["fc3_w"], h["fc3_b"], **attrs)
        else:
            bits = 8 if kind.endswith("8") else 4
            qi = orc.make_qmoe_inputs(T=T_r * world, H=512, I=256, E=E, k=2, bits=bits,
                                      block_size=0 if bits == 8 else 128,
                                      scale_mu=-8.5 if bits == 8 else -5.0,
                                      scale_sigma=0.3, seed=44 + E)
            g = lambda n: to_dev(qi[n], dev)
            d = dict(x=g("x"), router_probs=g("router_probs"))
            weights = dict(fc1_weights=g("fc1_q"), fc1_scales=g("fc1_scales"),
                           fc2_weights=g("fc2_q"), fc2_scales=g("fc2_scales"),
                           fc3_weights=g("fc3_q"), fc3_scales=g("fc3_scales"))
            attrs = qi["attrs"]
            h = {n: as_np(v) for n, v in d.items()}
            ref_fn = lambda x, lg: orc.qmoe(x, lg, qi["fc1_q"], qi["fc1_scales"], None,
                                            qi["fc2_q"], qi["fc2_scales"], None, qi["fc3_q"],
                                            qi["fc3_scales"], None, **attrs)
        sl = slice(rank * T_r, (rank + 1) * T_r)
        xs, ls = d["x"][sl], d["router_probs"][sl]
        layer = ep.ExpertParallelMoE(pkg, num_experts=E, hidden_size=512, inter_size=256,
                                     dtype=pkg.FLOAT16, has_fc3=True,
                                     local_weights=ep.shard_experts(weights, rank, world),
                                     transport=transport, **attrs)
        assert layer.transport == transport
        out = layer.forward(xs.contiguous(), ls.contiguous())
        T2 = T_r if rank == 0 else 100
        out2 = layer.forward(xs[:T2].contiguous(), ls[:T2].contiguous())
        torch.cuda.synchronize()
        ref = ref_fn(h["x"][sl], h["router_probs"][sl])
        tol = lambda r: TOL["float16"]["atol"] + TOL["float16"]["rtol"] * np.abs(r)
        err = np.abs(as_np(out) - ref) - tol(ref)
        err2 = np.abs(as_np(out2) - ref[:T2]) - tol(ref[:T2])
        if hasattr(layer, "close"):
            layer.close()
        q.put((rank, float(max(err.max(), err2.max()))))
    except Exception as exc:
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,transport,E,kind", [
    (2, "p2p", 8, "moe"), (2, "collective", 8, "moe"), (2, "p2p", 2, "moe"),
    (2, "p2p", 16, "moe_k8"), (8, "p2p", 64, "moe_k8"),
    (2, "p2p", 8, "qmoe4"), (2, "p2p", 16, "qmoe8"), (2, "collective", 8, "qmoe4"),
    (4, "p2p", 8, "moe"), (4, "p2p", 16, "qmoe8"), (8, "p2p", 64, "moe"), (8, "p2p", 16, "qmoe8")],
    ids=lambda v: str(v))
def test_ep_multi_rank(world, transport, E, kind):
    """W NCCL ranks (one per GPU): outputs of every rank against the oracle."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q, transport, E, kind))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
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
