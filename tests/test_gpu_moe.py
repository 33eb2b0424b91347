"""GPU parity of the full MoE / QMoE layer through the C ABI against the oracle."""

import math
import os
import pathlib

import numpy as np
import pytest

from gpu_util import TOL, as_np, load_golden, moe_input_list, moe_inputs_on, to_dev, torch_dtype

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).parent / "golden"


def run_moe(pkg, d, attrs, out=None):
    op = pkg.MoE(**attrs)
    try:
        return op(moe_input_list(d), out=out)
    finally:
        op.release()


def oracle_out(orc, h, attrs):
    return orc.moe(h["x"], h["router_probs"], h["fc1_w"], h["fc1_b"], h["fc2_w"], h["fc2_b"],
                   h["fc3_w"], h["fc3_b"], **attrs)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("*.npz")), ids=lambda p: p.stem)
def test_golden_fixtures(pkg, orc, dev, path):
    import torch
    d, meta = load_golden(path)
    dt = torch_dtype(meta["dtype"])
    get = lambda n: to_dev(d[n], dev) if n in d.files else None
    if meta["op"] == "MoE":
        op = pkg.MoE(**meta["attrs"])
        out = op([get("x"), get("router_probs"), get("fc1_w"), get("fc1_b"), get("fc2_w"),
                  get("fc2_b"), get("fc3_w"), get("fc3_b")])
    else:
        op = pkg.QMoE(**meta["attrs"])
        out = op([get("x"), get("router_probs"), get("fc1_q"), get("fc1_scales"), None,
                  get("fc2_q"), get("fc2_scales"), None, get("fc3_q"), get("fc3_scales"), None])
    op.release()
    assert out.dtype == dt
    np.testing.assert_allclose(as_np(out), d["output"], **TOL[meta["dtype"]])
    mode = 2 if meta["attrs"].get("use_sparse_mixer") else meta["attrs"]["normalize_routing_weights"]
    idx, _ = pkg.route(get("router_probs"), meta["attrs"]["k"], mode)
    np.testing.assert_array_equal(idx.cpu().numpy(), d["expert_idx"])


def test_config1_fp32_silu_bias(pkg, orc, dev):
    """Benchmark config 1: fp32, T=256, H=512, I=1024, E=8, k=2, silu, fc1/fc2 bias."""
    inp = orc.make_moe_inputs(T=256, H=512, I=1024, E=8, k=2, act="silu", gated=False,
                              dtype="float32", bias=True, normalize=1, seed=20261201)
    d, h = moe_inputs_on(dev, inp, "float32")
    out = run_moe(pkg, d, inp["attrs"])
    np.testing.assert_allclose(as_np(out), oracle_out(orc, h, inp["attrs"]), **TOL["float32"])


CASES = [
    # (T, H, I, E, k, act, gated, bias, normalize, extra)
    (64, 256, 384, 8, 2, "silu", True, False, 1, {}),
    (200, 512, 256, 16, 4, "gelu", False, True, 0, {}),
    (129, 256, 512, 8, 2, "relu", True, True, 1, {}),
    (77, 128, 256, 4, 1, "identity", False, True, 0, {}),
    (300, 256, 1024, 64, 8, "silu", True, False, 1, {}),
    (1, 256, 256, 8, 2, "silu", True, False, 1, {}),
    (3, 136, 200, 8, 2, "silu", True, True, 1, {}),        # N, K not multiples of 64
]


@pytest.mark.parametrize("dtype_name", ["float16", "bfloat16"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"T{c[0]}H{c[1]}I{c[2]}E{c[3]}k{c[4]}{c[5]}")
def test_moe_half(pkg, orc, dev, dtype_name, case):
    T, H, I, E, k, act, gated, bias, norm, extra = case
    inp = orc.make_moe_inputs(T=T, H=H, I=I, E=E, k=k, act=act, gated=gated, dtype="float32",
                              bias=bias, normalize=norm, seed=T * 7 + E)
    d, h = moe_inputs_on(dev, inp, dtype_name)
    attrs = dict(inp["attrs"], **extra)
    out = run_moe(pkg, d, attrs)
    np.testing.assert_allclose(as_np(out), oracle_out(orc, h, attrs), **TOL[dtype_name])


@pytest.mark.parametrize("fusion", [0, 1, 2])
@pytest.mark.parametrize("dtype_name", ["float16", "float32"])
def test_swiglu_variants(pkg, orc, dev, fusion, dtype_name):
    import torch
    T, H, I, E, k = 96, 256, 192, 8, 2
    inp = orc.make_moe_inputs(T=T, H=H, I=I, E=E, k=k, act="swiglu", gated=True,
                              dtype="float32", bias=True, normalize=1, seed=fusion + 40)
    w1, w3, b1, b3 = inp["fc1_w"], inp["fc3_w"], inp["fc1_b"], inp["fc3_b"]
    if fusion == 1:
        W = np.empty((E, 2 * I, H), np.float32); W[:, 0::2] = w1; W[:, 1::2] = w3
        B = np.empty((E, 2 * I), np.float32); B[:, 0::2] = b1; B[:, 1::2] = b3
        inp.update(fc1_w=W, fc1_b=B, fc3_w=None, fc3_b=None)
    elif fusion == 2:
        inp.update(fc1_w=np.concatenate([w1, w3], 1), fc1_b=np.concatenate([b1, b3], 1),
                   fc3_w=None, fc3_b=None)
    d, h = moe_inputs_on(dev, inp, dtype_name)
    attrs = dict(activation_type="swiglu", k=k, normalize_routing_weights=1,
                 swiglu_fusion=fusion, activation_alpha=1.702, activation_beta=1.0,
                 swiglu_limit=0.5)
    out = run_moe(pkg, d, attrs)
    np.testing.assert_allclose(as_np(out), oracle_out(orc, h, attrs), **TOL[dtype_name])


def test_input_3d_and_empty(pkg, orc, dev):
    import torch
    inp = orc.make_moe_inputs(T=48, H=128, I=128, E=8, k=2, act="silu", gated=True,
                              dtype="float16", bias=False, seed=5)
    d, h = moe_inputs_on(dev, inp, "float16")
    d3 = dict(d, x=d["x"].view(4, 12, 128))
    out = run_moe(pkg, d3, inp["attrs"])
    assert out.shape == (4, 12, 128)
    np.testing.assert_allclose(as_np(out).reshape(48, 128), oracle_out(orc, h, inp["attrs"]),
                               **TOL["float16"])
    d0 = dict(d, x=d["x"][:0], router_probs=d["router_probs"][:0])
    out0 = run_moe(pkg, d0, inp["attrs"])
    assert out0.shape == (0, 128)


def test_shape_errors(pkg, orc, dev):
    import torch
    inp = orc.make_moe_inputs(T=8, H=64, I=64, E=4, k=2, act="silu", gated=False,
                              dtype="float16", seed=6)
    d, _ = moe_inputs_on(dev, inp, "float16")
    op = pkg.MoE(activation_type="silu", k=2)
    bad = moe_input_list(d)
    bad[2] = d["fc1_w"][:, :32].contiguous()
    with pytest.raises(pkg.InvalidArgument, match="fc1_experts_weights"):
        op(bad)
    bad = moe_input_list(d)
    bad[1] = d["router_probs"][:4].contiguous()
    with pytest.raises(pkg.InvalidArgument, match="router_probs"):
        op(bad)
    bad = moe_input_list(d)
    bad[4] = d["fc2_w"].float()
    with pytest.raises(pkg.InvalidArgument, match="fc2_experts_weights"):
        op(bad)
    op.release()
    op = pkg.MoE(activation_type="silu", k=5)
    with pytest.raises(pkg.InvalidArgument, match="k=5"):
        op(moe_input_list(d))
    op.release()


def test_tensor_core_path_matches_ffma_path(pkg, orc, dev):
    """The tcgen05 GEMMs and the FFMA GEMMs give the same layer output."""
    import torch
    inp = orc.make_moe_inputs(T=512, H=1024, I=768, E=8, k=2, act="silu", gated=True,
                              dtype="float32", seed=9)
    d, h = moe_inputs_on(dev, inp, "bfloat16")
    tc = run_moe(pkg, d, inp["attrs"])
    os.environ["MOE_B200_FORCE_SIMT"] = "1"
    try:
        simt = run_moe(pkg, d, inp["attrs"])
    finally:
        del os.environ["MOE_B200_FORCE_SIMT"]
    ref = oracle_out(orc, h, inp["attrs"])
    np.testing.assert_allclose(as_np(tc), ref, **TOL["bfloat16"])
    np.testing.assert_allclose(as_np(simt), ref, **TOL["bfloat16"])


def _torch_rows_reference(pkg, orc, d, rows, attrs):
    """fp32 PyTorch reference of the layer for a subset of rows (the layer is row-wise
    independent given each row's routing)."""
    import torch
    x = d["x"][rows].float()
    lg = d["router_probs"][rows].float().cpu().numpy()
    idx, w = orc.route(lg, attrs["k"], attrs["normalize_routing_weights"])
    out = torch.zeros_like(x)
    for i in range(len(rows)):
        for j in range(attrs["k"]):
            e = int(idx[i, j])
            g = x[i] @ d["fc1_w"][e].float().T
            u = x[i] @ d["fc3_w"][e].float().T
            a = torch.nn.functional.silu(g) * u
            out[i] += float(w[i, j]) * (a @ d["fc2_w"][e].float().T)
    return out.double().cpu().numpy()


def test_config2_mixtral_full_size(pkg, orc, dev):
    """Benchmark config 2 at full size: Mixtral-shaped fp16 layer, T=4096."""
    import torch
    g = torch.Generator(device=dev).manual_seed(20261202)
    T, H, I, E = 4096, 4096, 14336, 8
    d = dict(x=torch.randn(T, H, device=dev, generator=g).half(),
             router_probs=torch.randn(T, E, device=dev, generator=g).half(),
             fc1_w=(torch.randn(E, I, H, device=dev, generator=g) * 0.02).half(), fc1_b=None,
             fc2_w=(torch.randn(E, H, I, device=dev, generator=g) * 0.02).half(), fc2_b=None,
             fc3_w=(torch.randn(E, I, H, device=dev, generator=g) * 0.02).half(), fc3_b=None)
    attrs = dict(activation_type="silu", k=2, normalize_routing_weights=1)
    out1 = run_moe(pkg, d, attrs)
    out2 = run_moe(pkg, d, attrs)
    assert torch.equal(out1, out2), "layer output is not deterministic"
    rows = torch.tensor([0, 1, 777, 2048, 4095] + list(range(1000, 1027)), device=dev)
    ref = _torch_rows_reference(pkg, orc, d, rows, attrs)
    np.testing.assert_allclose(as_np(out1[rows]), ref, **TOL["float16"])


TC_CASES = [
    # (T, H, I, E, k, act, gated, bias, dtype)
    (300, 256, 384, 8, 2, "silu", True, False, "float16"),
    (1000, 512, 256, 16, 4, "gelu", False, True, "bfloat16"),
    (5, 128, 128, 64, 8, "silu", True, True, "float16"),       # most experts empty
    (700, 256, 520, 4, 1, "relu", True, False, "bfloat16"),    # N tail, one expert per row
    (2048, 1024, 768, 8, 2, "silu", True, False, "float16"),
]


@pytest.mark.parametrize("mode", ["1", "2"], ids=["single_cta", "cta_pair"])
@pytest.mark.parametrize("case", TC_CASES, ids=lambda c: f"T{c[0]}H{c[1]}I{c[2]}E{c[3]}k{c[4]}{c[5]}")
def test_tensor_core_kernels(pkg, orc, dev, mode, case):
    """Both tcgen05 kernels (one CTA per tile, and CTA pairs with cta_group::2)."""
    T, H, I, E, k, act, gated, bias, dtype_name = case
    inp = orc.make_moe_inputs(T=T, H=H, I=I, E=E, k=k, act=act, gated=gated, dtype="float32",
                              bias=bias, normalize=1, seed=T + E + int(mode))
    d, h = moe_inputs_on(dev, inp, dtype_name)
    os.environ["MOE_B200_TC_MODE"] = mode
    try:
        out = run_moe(pkg, d, inp["attrs"])
    finally:
        del os.environ["MOE_B200_TC_MODE"]
    np.testing.assert_allclose(as_np(out), oracle_out(orc, h, inp["attrs"]), **TOL[dtype_name])


def _qmoe_run(pkg, dev, q, attrs, fc3=True):
    get = lambda n: to_dev(q[n], dev) if q.get(n) is not None else None
    op = pkg.QMoE(**attrs)
    try:
        return op([get("x"), get("router_probs"), get("fc1_q"), get("fc1_scales"), get("fc1_b"),
                   get("fc2_q"), get("fc2_scales"), get("fc2_b"),
                   get("fc3_q") if fc3 else None, get("fc3_scales") if fc3 else None,
                   get("fc3_b") if fc3 else None])
    finally:
        op.release()


QMOE_DECODE_CASES = [
    # (T, H, I, E, k, bits, block_size)
    (1, 512, 384, 8, 2, 4, 128),
    (8, 512, 384, 8, 2, 4, 128),
    (32, 256, 512, 8, 2, 4, 32),
    (64, 512, 256, 8, 2, 8, 0),
    (17, 384, 640, 16, 2, 8, 64),
    (3, 256, 256, 64, 8, 4, 0),
]


@pytest.mark.parametrize("case", QMOE_DECODE_CASES, ids=lambda c: f"T{c[0]}H{c[1]}I{c[2]}E{c[3]}k{c[4]}b{c[5]}bs{c[6]}")
def test_qmoe_decode_path(pkg, orc, dev, case):
    """Weight-streaming decode kernels against the oracle and the dequantise+GEMM path."""
    T, H, I, E, k, bits, bs = case
    # Scales keep the outputs near unit scale, where the fp16 tolerances are meaningful.
    mu = -5.0 if bits == 4 else -8.5
    q = orc.make_qmoe_inputs(T=T, H=H, I=I, E=E, k=k, bits=bits, block_size=bs,
                             scale_mu=mu, scale_sigma=0.3, seed=T * 13 + bits)
    attrs = dict(q["attrs"], k=k)
    out = _qmoe_run(pkg, dev, q, attrs)
    ref = orc.qmoe(q["x"], q["router_probs"], q["fc1_q"], q["fc1_scales"], None, q["fc2_q"],
                   q["fc2_scales"], None, q["fc3_q"], q["fc3_scales"], None, **attrs)
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])
    os.environ["MOE_B200_QMOE_NO_DECODE"] = "1"
    try:
        out2 = _qmoe_run(pkg, dev, q, attrs)
    finally:
        del os.environ["MOE_B200_QMOE_NO_DECODE"]
    np.testing.assert_allclose(as_np(out2), ref, **TOL["float16"])


@pytest.mark.parametrize("case", [(1, 512, 384, 8, 2, 4, 128), (8, 512, 384, 8, 2, 4, 0),
                                  (64, 512, 256, 8, 2, 4, 256)],
                         ids=lambda c: f"T{c[0]}b{c[5]}bs{c[6]}")
def test_qmoe_decode_per_code_conversion(pkg, orc, dev, case):
    """int4 decode with the per-code conversion (MOE_B200_QDEC_RAW4=0) in the exact-code
    modes (one scale per row, or blocks of whole 128-wide chunks): the same outputs as
    the oracle and, within the tolerance, as the default biased-code kernel."""
    T, H, I, E, k, bits, bs = case
    q = orc.make_qmoe_inputs(T=T, H=H, I=I, E=E, k=k, bits=bits, block_size=bs,
                             scale_mu=-5.0, scale_sigma=0.3, seed=T * 7 + bs)
    attrs = dict(q["attrs"], k=k)
    ref = orc.qmoe(q["x"], q["router_probs"], q["fc1_q"], q["fc1_scales"], None, q["fc2_q"],
                   q["fc2_scales"], None, q["fc3_q"], q["fc3_scales"], None, **attrs)
    default = _qmoe_run(pkg, dev, q, attrs)
    os.environ["MOE_B200_QDEC_RAW4"] = "0"
    try:
        conv = _qmoe_run(pkg, dev, q, attrs)
    finally:
        del os.environ["MOE_B200_QDEC_RAW4"]
    assert np.isfinite(as_np(conv)).all()
    np.testing.assert_allclose(as_np(conv), ref, **TOL["float16"])
    np.testing.assert_allclose(as_np(conv), as_np(default), **TOL["float16"])


@pytest.mark.parametrize("shape", [(6, 4, 64), (300, 4, 0), (300, 8, 0), (300, 4, 64)],
                         ids=["decode_int4_bs64", "prefill_int4_rowscale", "prefill_int8_rowscale",
                              "prefill_int4_bs64"])
@pytest.mark.parametrize("variant", ["plain_gelu_bias", "swiglu_interleaved", "swiglu_halves"])
def test_qmoe_decode_variants(pkg, orc, dev, variant, shape):
    """Activation / fc1 layouts through the decode kernels (T=6) and the packed tensor-core
    GEMM (T=300), including per-row scales, whose scaling and biased-code correction run in
    the epilogue with the gate and linear halves' own scale addressing."""
    T, bits, bs = shape
    H, I, E, k = 256, 256, 8, 2
    rng = np.random.default_rng(77)
    # Scales keep the outputs near unit scale, where the fp16 tolerances are meaningful
    # (the dequantised fp16 weights carry ~5e-4 relative rounding; larger outputs put
    # near-zero elements past atol).
    q = orc.make_qmoe_inputs(T=T, H=H, I=I, E=E, k=k, bits=bits, block_size=bs,
                             scale_mu=-5.0 if bits == 4 else -8.5, scale_sigma=0.3, seed=78)
    attrs = dict(q["attrs"], k=k)
    fc3 = True
    if variant == "plain_gelu_bias":
        attrs["activation_type"] = "gelu"
        fc3 = False
        q["fc1_b"] = (rng.standard_normal((E, I)) * 0.05).astype(np.float16)
        q["fc2_b"] = (rng.standard_normal((E, H)) * 0.05).astype(np.float16)
    else:
        fusion = 1 if variant == "swiglu_interleaved" else 2
        attrs.update(activation_type="swiglu", swiglu_fusion=fusion, activation_alpha=1.702,
                     activation_beta=1.0, swiglu_limit=7.0)
        if fusion == 1:
            W = np.empty((E, 2 * I, q["fc1_q"].shape[2]), np.uint8)
            W[:, 0::2] = q["fc1_q"]; W[:, 1::2] = q["fc3_q"]
            S = np.empty((E, 2 * I) + q["fc1_scales"].shape[2:], np.float16)
            S[:, 0::2] = q["fc1_scales"]; S[:, 1::2] = q["fc3_scales"]
        else:
            W = np.concatenate([q["fc1_q"], q["fc3_q"]], 1)
            S = np.concatenate([q["fc1_scales"], q["fc3_scales"]], 1)
        q["fc1_q"], q["fc1_scales"] = W, S
        q["fc1_b"] = (rng.standard_normal((E, 2 * I)) * 0.05).astype(np.float16)
        fc3 = False
    out = _qmoe_run(pkg, dev, q, attrs, fc3=fc3)
    W1 = orc.dequantize(q["fc1_q"], q["fc1_scales"], bits, bs, H)
    W2 = orc.dequantize(q["fc2_q"], q["fc2_scales"], bits, bs, I)
    W3 = orc.dequantize(q["fc3_q"], q["fc3_scales"], bits, bs, H) if fc3 else None
    ref = orc.moe(q["x"], q["router_probs"], W1, q.get("fc1_b"), W2, q.get("fc2_b"), W3, None,
                  **{kk: v for kk, v in attrs.items() if kk not in ("expert_weight_bits", "block_size")})
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])


QMOE_PREFILL_CASES = [
    # (T, H, I, E, k, bits, block_size)
    (300, 512, 384, 8, 2, 4, 128),
    (400, 256, 640, 8, 2, 8, 0),
    (700, 384, 256, 16, 2, 4, 32),
    (260, 256, 256, 4, 4, 8, 64),
]


@pytest.mark.parametrize("case", QMOE_PREFILL_CASES, ids=lambda c: f"T{c[0]}H{c[1]}I{c[2]}E{c[3]}k{c[4]}b{c[5]}bs{c[6]}")
def test_qmoe_prefill_fused_dequant(pkg, orc, dev, case):
    """T*k beyond the decode sizes: packed weights dequantised in shared memory by the
    tensor-core kernel, against the oracle and the dequantise-to-HBM path."""
    T, H, I, E, k, bits, bs = case
    mu = -5.0 if bits == 4 else -8.5
    q = orc.make_qmoe_inputs(T=T, H=H, I=I, E=E, k=k, bits=bits, block_size=bs,
                             scale_mu=mu, scale_sigma=0.3, seed=T + bits)
    attrs = dict(q["attrs"], k=k)
    ref = orc.qmoe(q["x"], q["router_probs"], q["fc1_q"], q["fc1_scales"], None, q["fc2_q"],
                   q["fc2_scales"], None, q["fc3_q"], q["fc3_scales"], None, **attrs)
    out = _qmoe_run(pkg, dev, q, attrs)
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])
    os.environ["MOE_B200_QMOE_DEQUANT"] = "1"
    try:
        out2 = _qmoe_run(pkg, dev, q, attrs)
    finally:
        del os.environ["MOE_B200_QMOE_DEQUANT"]
    np.testing.assert_allclose(as_np(out2), ref, **TOL["float16"])
    np.testing.assert_allclose(as_np(out), as_np(out2), rtol=1e-2, atol=1e-3)


# Per-expert row counts around the 16-row granularity and the 128 / 256 tile sizes of the
# CTA-pair kernel: tails of 1..16 rows, exactly 128, one past 128 / 256, and an empty expert.
SWAP_COUNTS = [1, 15, 16, 17, 0, 127, 128, 129, 255, 256, 257, 391, 496]


@pytest.mark.parametrize("swap_max", ["0", "16", "128", "240"], ids=["off", "16", "128", "240"])
@pytest.mark.parametrize("variant", ["silu_bias_f16", "gelu_plain_bias_bf16",
                                     "swiglu_interleaved_f16", "swiglu_halves_bf16"])
def test_pair_kernel_swapped_tail_tiles(pkg, orc, dev, swap_max, variant):
    """CTA-pair kernel with the ragged last tile of each expert computed swapped (weights as
    M, rows as N) up to `swap_max` rows, against the oracle on exact per-expert counts."""
    counts = SWAP_COUNTS
    E, T, H, I, k = len(counts), sum(counts), 320, 200, 1
    act = {"silu_bias_f16": "silu", "gelu_plain_bias_bf16": "gelu"}.get(variant, "swiglu")
    gated = variant != "gelu_plain_bias_bf16"
    dtype_name = "bfloat16" if variant.endswith("bf16") else "float16"
    inp = orc.make_moe_inputs(T=T, H=H, I=I, E=E, k=k, act=act, gated=gated, dtype="float32",
                              bias=True, normalize=1, seed=int(swap_max) + len(variant))
    owner = np.repeat(np.arange(E), counts)
    np.random.default_rng(3).shuffle(owner)
    lg = inp["router_probs"] * 0.1
    lg[np.arange(T), owner] += 4.0
    inp["router_probs"] = lg
    attrs = dict(inp["attrs"])
    if act == "swiglu":
        fusion = 1 if "interleaved" in variant else 2
        w1, w3, b1, b3 = inp["fc1_w"], inp["fc3_w"], inp["fc1_b"], inp["fc3_b"]
        if fusion == 1:
            W = np.empty((E, 2 * I, H), np.float32); W[:, 0::2] = w1; W[:, 1::2] = w3
            B = np.empty((E, 2 * I), np.float32); B[:, 0::2] = b1; B[:, 1::2] = b3
            inp.update(fc1_w=W, fc1_b=B)
        else:
            inp.update(fc1_w=np.concatenate([w1, w3], 1), fc1_b=np.concatenate([b1, b3], 1))
        inp.update(fc3_w=None, fc3_b=None)
        attrs.update(swiglu_fusion=fusion, activation_alpha=1.702, activation_beta=1.0,
                     swiglu_limit=7.0)
    d, h = moe_inputs_on(dev, inp, dtype_name)
    idx, _ = pkg.route(d["router_probs"], k, 1)
    np.testing.assert_array_equal(np.bincount(idx.cpu().numpy().ravel(), minlength=E), counts)
    os.environ.update(MOE_B200_TC_MODE="2", MOE_B200_PAIR_SWAP_MAX=swap_max)
    try:
        out = run_moe(pkg, d, attrs)
    finally:
        del os.environ["MOE_B200_TC_MODE"], os.environ["MOE_B200_PAIR_SWAP_MAX"]
    np.testing.assert_allclose(as_np(out), oracle_out(orc, h, attrs), **TOL[dtype_name])


def test_stage_timing_entries(pkg, orc, dev):
    """forward_timed and forward_staged compute the same layer as forward and report
    non-negative stage times whose sum brackets the whole call."""
    import torch
    inp = orc.make_moe_inputs(T=512, H=256, I=384, E=8, k=2, act="silu", gated=True,
                              dtype="float32", seed=91)
    d, h = moe_inputs_on(dev, inp, "float16")
    ref = oracle_out(orc, h, inp["attrs"])
    out = torch.empty_like(d["x"])
    prob = pkg.make_problem(512, 256, 384, 8, pkg.FLOAT16, has_fc3=True, **inp["attrs"])
    tens = dict(input=d["x"], router_probs=d["router_probs"], fc1_weights=d["fc1_w"],
                fc2_weights=d["fc2_w"], fc3_weights=d["fc3_w"], output=out)
    ws = torch.empty(pkg.workspace_size(prob), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    ms = pkg.forward_timed(prob, tens, ws, stream)
    assert set(ms) == set(pkg.STAGES) and min(ms.values()) >= 0
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])
    out.zero_()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(pkg.STAGES) + 1)]
    for ev in evs:
        ev.record(stream)
    pkg.forward_staged(prob, tens, ws, evs, stream)
    torch.cuda.synchronize(dev)
    parts = [evs[i].elapsed_time(evs[i + 1]) for i in range(len(pkg.STAGES))]
    assert min(parts) >= 0
    assert abs(sum(parts) - evs[0].elapsed_time(evs[-1])) < 1e-3
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])
    with pytest.raises(pkg.InvalidArgument):
        pkg.forward_staged(prob, tens, ws, evs[:3], stream)
    # Only the fc1 boundaries recorded (None entries are skipped).
    i1 = pkg.STAGES.index("fc1")
    sparse = [None] * (len(pkg.STAGES) + 1)
    sparse[i1], sparse[i1 + 1] = evs[0], evs[1]
    out.zero_()
    pkg.forward_staged(prob, tens, ws, sparse, stream)
    torch.cuda.synchronize(dev)
    assert evs[0].elapsed_time(evs[1]) > 0
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])


@pytest.mark.parametrize("case", ["fp16_gated", "bf16_plain_bias", "fp32_simt"])
def test_moe_sparse_mixer(pkg, orc, dev, case):
    """use_sparse_mixer=1 through the whole layer (tensor-core and FFMA GEMM paths)."""
    dtype_name = {"fp16_gated": "float16", "bf16_plain_bias": "bfloat16",
                  "fp32_simt": "float32"}[case]
    gated = case == "fp16_gated"
    inp = orc.make_moe_inputs(T=300, H=256, I=384, E=8, k=2, act="silu" if gated else "gelu",
                              gated=gated, dtype="float32", bias=case != "fp16_gated",
                              normalize=1, seed=101)
    inp["router_probs"] *= 0.05  # close logits: the 2% band keeps several experts
    d, h = moe_inputs_on(dev, inp, dtype_name)
    attrs = dict(inp["attrs"], use_sparse_mixer=1)
    out = run_moe(pkg, d, attrs)
    np.testing.assert_allclose(as_np(out), oracle_out(orc, h, attrs), **TOL[dtype_name])


@pytest.mark.parametrize("T", [5, 300])  # decode kernels; dequantise + GEMM
def test_qmoe_sparse_mixer(pkg, orc, dev, T):
    q = orc.make_qmoe_inputs(T=T, H=256, I=256, E=8, k=2, bits=4, block_size=128,
                             scale_mu=-5.0, scale_sigma=0.3, seed=T + 5)
    q["router_probs"] = (q["router_probs"].astype(np.float32) * 0.05).astype(np.float16)
    attrs = dict(q["attrs"], use_sparse_mixer=1)
    out = _qmoe_run(pkg, dev, q, attrs)
    ref = orc.qmoe(q["x"], q["router_probs"], q["fc1_q"], q["fc1_scales"], None, q["fc2_q"],
                   q["fc2_scales"], None, q["fc3_q"], q["fc3_scales"], None, **attrs)
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])


@pytest.mark.parametrize("dtype_name", ["float16", "bfloat16"])
@pytest.mark.parametrize("case", [(700, 256, 320, 4, 2, "silu", True),
                                  (530, 192, 256, 8, 1, "gelu", False),
                                  (300, 128, 136, 3, 2, "swiglu", True)],
                         ids=["gated_k2", "plain_k1", "swiglu_halves"])
def test_gather_fused_into_pair_gemm(pkg, orc, dev, dtype_name, case):
    """MOE_B200_GATHER_FUSION=1: the CTA-pair kernel loads fc1's rows from the
    un-permuted input with TMA gather4 (normal and swapped tail tiles).  Identical values
    to the separate gather, and within tolerance of the oracle."""
    T, H, I, E, k, act, gated = case
    inp = orc.make_moe_inputs(T=T, H=H, I=I, E=E, k=k, act=act, gated=gated, dtype="float32",
                              bias=True, normalize=1, seed=T + E)
    attrs = dict(inp["attrs"])
    if act == "swiglu":
        inp.update(fc1_w=np.concatenate([inp["fc1_w"], inp["fc3_w"]], 1),
                   fc1_b=np.concatenate([inp["fc1_b"], inp["fc3_b"]], 1), fc3_w=None, fc3_b=None)
        attrs.update(swiglu_fusion=2, activation_alpha=1.702, activation_beta=1.0,
                     swiglu_limit=7.0)
    d, h = moe_inputs_on(dev, inp, dtype_name)
    env = {"MOE_B200_TC_MODE": "2", "MOE_B200_PAIR_SWAP_MAX": "240"}
    old = {n: os.environ.get(n) for n in list(env) + ["MOE_B200_GATHER_FUSION"]}
    try:
        os.environ.update(env)
        plain = run_moe(pkg, d, attrs)
        os.environ["MOE_B200_GATHER_FUSION"] = "1"
        fused = run_moe(pkg, d, attrs)
    finally:
        for n, v in old.items():
            if v is None:
                os.environ.pop(n, None)
            else:
                os.environ[n] = v
    np.testing.assert_array_equal(as_np(fused), as_np(plain))
    np.testing.assert_allclose(as_np(fused), oracle_out(orc, h, attrs), **TOL[dtype_name])


@pytest.mark.parametrize("case", [
    (300, 256, 384, 8, 2, "silu", True, False, "float16"),
    (1000, 512, 256, 16, 4, "gelu", False, True, "bfloat16"),
    (5, 128, 128, 64, 8, "silu", True, True, "float16"),        # swapped tail tiles only
    (700, 256, 520, 4, 1, "relu", True, False, "bfloat16"),     # k = 1
    (2048, 1024, 768, 64, 8, "silu", True, False, "float16"),   # C4-like, Zipf-free
    (3000, 520, 256, 8, 2, "silu", True, False, "float16"),     # H not a multiple of 32
], ids=lambda c: f"T{c[0]}H{c[1]}I{c[2]}E{c[3]}k{c[4]}{c[8]}")
def test_combine_fused_into_fc2_epilogue(pkg, orc, dev, case):
    """MOE_B200_FUSED_COMBINE=1: the fc2 epilogue combines each token's k rows (arrival
    count per 32-column segment, the completing row sums them in slot order).  Outputs
    are bit-identical to the separate combine kernel's, deterministic across calls, and
    within the tolerance of the oracle, for both tensor-core kernels."""
    import torch
    T, H, I, E, k, act, gated, bias, dtype_name = case
    inp = orc.make_moe_inputs(T=T, H=H, I=I, E=E, k=k, act=act, gated=gated, dtype="float32",
                              bias=bias, normalize=1, seed=T + E + 5)
    d, h = moe_inputs_on(dev, inp, dtype_name)
    ref = run_moe(pkg, d, inp["attrs"])
    for mode in ("1", "2"):
        os.environ["MOE_B200_FUSED_COMBINE"] = "1"
        os.environ["MOE_B200_TC_MODE"] = mode
        try:
            out1 = run_moe(pkg, d, inp["attrs"])
            out2 = run_moe(pkg, d, inp["attrs"])
            os.environ["MOE_B200_FUSED_COMBINE"] = "0"
            plain = run_moe(pkg, d, inp["attrs"])
        finally:
            del os.environ["MOE_B200_FUSED_COMBINE"]
            del os.environ["MOE_B200_TC_MODE"]
        assert torch.equal(out1, out2), "fused combine is not deterministic"
        assert torch.equal(out1, plain), f"mode {mode}: fused combine differs from the combine kernel"
    np.testing.assert_allclose(as_np(out1), oracle_out(orc, h, inp["attrs"]), **TOL[dtype_name])
    assert torch.equal(ref, plain)
