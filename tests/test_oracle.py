"""CPU tests of the oracle: hand-computed known answers, internal consistency,
the C restatement against the numpy one, and the committed golden fixtures."""

import ctypes
import math
import pathlib

import numpy as np
import pytest

GOLDEN = pathlib.Path(__file__).parent / "golden"


# ------------------------------------------------------------- known answers
def test_route_known_answer(orc):
    logits = np.array([[1.0, 3.0, 2.0, 3.0],     # tie 1 vs 3 -> lower index first
                       [0.0, 0.0, 0.0, 0.0],     # all equal -> 0, 1
                       [-1.0, -5.0, np.nan, -2.0]], dtype=np.float32)  # NaN reads as -inf
    idx, w = orc.route(logits, 2, 1)
    assert idx.tolist() == [[1, 3], [0, 1], [0, 3]]
    np.testing.assert_allclose(w[0], [0.5, 0.5])
    np.testing.assert_allclose(w[1], [0.5, 0.5])
    e = math.exp(-1.0)
    np.testing.assert_allclose(w[2], [1 / (1 + e), e / (1 + e)], rtol=1e-7)
    idx, w = orc.route(logits[:1], 1, 0)
    s = math.exp(1) + 2 * math.exp(3) + math.exp(2)
    assert idx.tolist() == [[1]]
    np.testing.assert_allclose(w, [[math.exp(3) / s]], rtol=1e-6)


def test_permutation_known_answer(orc):
    idx = np.array([[2, 0], [0, 2], [1, 2]], dtype=np.int32)
    offsets, pos, src = orc.permutation(idx, 4)
    assert offsets.tolist() == [0, 2, 3, 6, 6]
    # expert 0: (t0,j1)=1, (t1,j0)=2 ; expert 1: (t2,j0)=4 ; expert 2: (t0,j0)=0,(t1,j1)=3,(t2,j1)=5
    assert src.tolist() == [1, 2, 4, 0, 3, 5]
    assert pos.tolist() == [[3, 0], [1, 4], [2, 5]]


def test_dequant_known_answer(orc):
    codes = np.array([[[-8, 7, 0, -1, 3, -3, 5, 2]]], dtype=np.int16)
    p4 = orc.pack_int4(codes)
    assert p4.tolist() == [[[0xF0, 0x78, 0x5B, 0xAD]]]
    s = np.array([[2.0]])
    np.testing.assert_array_equal(orc.dequantize(p4, s, 4, 0, 8)[0, 0], codes[0, 0] * 2.0)
    sb = np.array([[[1.0, 0.5]]])
    np.testing.assert_array_equal(orc.dequantize(p4, sb, 4, 4, 8)[0, 0],
                                  codes[0, 0] * np.array([1, 1, 1, 1, .5, .5, .5, .5]))
    p8 = orc.pack_int8(np.array([[[-127, 127, 0]]]))
    assert p8.tolist() == [[[1, 255, 128]]]
    np.testing.assert_array_equal(orc.dequantize(p8, np.array([[0.25]]), 8, 0, 3)[0, 0],
                                  [-31.75, 31.75, 0.0])


def test_moe_known_answer(orc):
    # 2 tokens, H=2, I=2, E=2, k=1, identity activation, identity-like weights.
    x = np.array([[1.0, 2.0], [3.0, -1.0]])
    logits = np.array([[0.0, 1.0], [2.0, 0.0]])
    w1 = np.array([np.eye(2), 2 * np.eye(2)])            # expert 1 doubles
    w2 = np.array([np.eye(2), np.array([[0.0, 1.0], [1.0, 0.0]])])  # expert 1 swaps
    b2 = np.array([[0.0, 0.0], [1.0, 1.0]])
    out = orc.moe(x, logits, w1, None, w2, b2, activation_type="identity", k=1,
                  normalize_routing_weights=1)
    # token 0 -> expert 1 (weight 1): swap(2*x) + 1 = [5, 3]; token 1 -> expert 0: x
    np.testing.assert_allclose(out, [[5.0, 3.0], [3.0, -1.0]])
    out = orc.moe(x, logits, w1, None, w2, b2, activation_type="relu", k=1,
                  normalize_routing_weights=1)
    np.testing.assert_allclose(out, [[5.0, 3.0], [3.0, 0.0]])
    # Without normalisation the weight is the full-softmax probability.
    out = orc.moe(x, logits, w1, None, w2, b2, activation_type="identity", k=1,
                  normalize_routing_weights=0)
    p0 = math.exp(1) / (1 + math.exp(1))
    p1 = math.exp(2) / (1 + math.exp(2))
    np.testing.assert_allclose(out, [[5 * p0, 3 * p0], [3 * p1, -1 * p1]])


def test_gated_and_swiglu_forms_agree(orc):
    rng = np.random.default_rng(0)
    T, H, I, E = 5, 6, 4, 3
    x = rng.standard_normal((T, H))
    lg = rng.standard_normal((T, E))
    w1 = rng.standard_normal((E, I, H)) * 0.3
    w3 = rng.standard_normal((E, I, H)) * 0.3
    w2 = rng.standard_normal((E, H, I)) * 0.3
    b1 = rng.standard_normal((E, I)) * 0.1
    b3 = rng.standard_normal((E, I)) * 0.1
    silu_gate = orc.moe(x, lg, w1, b1, w2, None, w3, b3, activation_type="silu", k=2,
                        normalize_routing_weights=1)
    sw0 = orc.moe(x, lg, w1, b1, w2, None, w3, b3, activation_type="swiglu", k=2,
                  normalize_routing_weights=1)
    inter = np.empty((E, 2 * I, H)); inter[:, 0::2] = w1; inter[:, 1::2] = w3
    binter = np.empty((E, 2 * I)); binter[:, 0::2] = b1; binter[:, 1::2] = b3
    sw1 = orc.moe(x, lg, inter, binter, w2, None, activation_type="swiglu", swiglu_fusion=1,
                  k=2, normalize_routing_weights=1)
    sw2 = orc.moe(x, lg, np.concatenate([w1, w3], 1), np.concatenate([b1, b3], 1), w2, None,
                  activation_type="swiglu", swiglu_fusion=2, k=2, normalize_routing_weights=1)
    for o in (sw0, sw1, sw2):
        np.testing.assert_allclose(o, silu_gate, rtol=1e-12, atol=1e-12)


# ------------------------------------------------------------- C restatement
def _c_oracle():
    import __graft_entry__ as g
    so = g.ROOT / "oracle" / "_build" / "libmoe_oracle.so"
    if not so.exists():
        import subprocess
        subprocess.run(["make", "-s", "-C", str(g.ROOT / "oracle")], check=True)
    L = ctypes.CDLL(str(so))
    L.oracle_moe.restype = ctypes.c_int
    return L


def c_moe(L, x, logits, w1, b1, w2, b2, w3=None, b3=None, *, act="silu", k=2, normalize=1,
          fusion=0, bits=0, block_size=0, s1=None, s2=None, s3=None, alpha=1.0, beta=0.0,
          limit=math.inf):
    acts = {"relu": 0, "gelu": 1, "silu": 2, "identity": 3, "swiglu": 4}
    f32 = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.float32)
    x, logits = f32(x), f32(logits)
    T, H = x.shape
    E = logits.shape[1]
    if bits:
        I = w2.shape[2] * 8 // bits
        W = [np.ascontiguousarray(w) if w is not None else None for w in (w1, w2, w3)]
    else:
        I = w2.shape[2]
        W = [f32(w) for w in (w1, w2, w3)]
    out = np.zeros((T, H), dtype=np.float32)
    P = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)
    bs = [f32(b) for b in (b1, b2, b3)]
    ss = [f32(s) for s in (s1, s2, s3)]
    L.oracle_moe.argtypes = [ctypes.c_int64] * 4 + [ctypes.c_int] * 4 + [ctypes.c_float] * 3 + \
        [ctypes.c_int] * 2 + [ctypes.c_void_p] * 12
    rc = L.oracle_moe(T, H, I, E, k, normalize, acts[act], fusion, alpha, beta, limit, bits,
                      block_size, P(x), P(logits), P(W[0]), P(ss[0]), P(bs[0]), P(W[1]),
                      P(ss[1]), P(bs[1]), P(W[2]), P(ss[2]), P(bs[2]), P(out))
    assert rc == 0
    return out


@pytest.mark.parametrize("act,gated,bias", [("silu", False, True), ("silu", True, False),
                                            ("gelu", False, True), ("relu", True, True)])
def test_c_oracle_matches_numpy(orc, act, gated, bias):
    L = _c_oracle()
    inp = orc.make_moe_inputs(T=37, H=64, I=48, E=6, k=2, act=act, gated=gated,
                              dtype="float32", bias=bias, seed=3)
    ref = orc.moe(inp["x"], inp["router_probs"], inp["fc1_w"], inp["fc1_b"], inp["fc2_w"],
                  inp["fc2_b"], inp["fc3_w"], inp["fc3_b"], **inp["attrs"])
    out = c_moe(L, inp["x"], inp["router_probs"], inp["fc1_w"], inp["fc1_b"], inp["fc2_w"],
                inp["fc2_b"], inp["fc3_w"], inp["fc3_b"], act=act)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("bits,block", [(4, 16), (8, 0)])
def test_c_oracle_qmoe_matches_numpy(orc, bits, block):
    L = _c_oracle()
    q = orc.make_qmoe_inputs(T=9, H=64, I=32, E=4, k=2, bits=bits, block_size=block,
                             scale_mu=-4.0, scale_sigma=0.3)
    ref = orc.qmoe(q["x"], q["router_probs"], q["fc1_q"], q["fc1_scales"], None, q["fc2_q"],
                   q["fc2_scales"], None, q["fc3_q"], q["fc3_scales"], None, **q["attrs"])
    out = c_moe(L, q["x"], q["router_probs"], q["fc1_q"], None, q["fc2_q"], None, q["fc3_q"],
                None, bits=bits, block_size=block, s1=q["fc1_scales"], s2=q["fc2_scales"],
                s3=q["fc3_scales"])
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-5 * np.abs(ref).max())


# ------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("path", sorted(GOLDEN.glob("*.npz")), ids=lambda p: p.stem)
def test_golden_fixture(orc, path):
    import json
    d = np.load(path, allow_pickle=False)
    meta = json.loads(str(d["meta"]))
    get = lambda n: d[n] if n in d.files else None
    if meta["op"] == "MoE":
        out = orc.moe(d["x"], d["router_probs"], d["fc1_w"], get("fc1_b"), d["fc2_w"],
                      get("fc2_b"), get("fc3_w"), get("fc3_b"), **meta["attrs"])
    else:
        out = orc.qmoe(d["x"], d["router_probs"], d["fc1_q"], d["fc1_scales"], None,
                       d["fc2_q"], d["fc2_scales"], None, get("fc3_q"), get("fc3_scales"),
                       None, **meta["attrs"])
    idx, w = orc.route(d["router_probs"], meta["attrs"]["k"],
                       meta["attrs"]["normalize_routing_weights"],
                       meta["attrs"].get("use_sparse_mixer", 0))
    np.testing.assert_array_equal(idx, d["expert_idx"])
    np.testing.assert_allclose(w, d["route_w"], rtol=0, atol=0)
    np.testing.assert_allclose(out, d["output"], rtol=1e-12, atol=1e-12)


def test_sparse_mixer_known_answer(orc):
    """Sparse-mixer top-2 on hand-computed rows: experts within 2 * 0.01 relative distance
    of a pick's logit share its softmax; the second pick excludes the first."""
    s = np.array([[2.0, 1.99, 0.0, 1.0],
                  [-1.0, -1.01, -3.0, -1.015],
                  [1.0, 1.0, 1.0, 1.0]], dtype=np.float32)
    idx, w = orc.route(s, 2, 0, use_sparse_mixer=1)
    assert idx.tolist() == [[0, 1], [0, 1], [0, 1]]
    f = lambda d: math.exp(float(np.float32(d)))
    # row 0: pick e0 keeps e1 (0.01 / 2 = 0.005); pick e1 keeps only itself.
    np.testing.assert_allclose(w[0], [1 / (1 + f(1.99 - 2.0)), 1.0], rtol=1e-6)
    # row 1 (negative logits: the factor is |s_e|): pick e0 keeps e1 (0.0099) and e3
    # (0.0148); pick e1 keeps e3 (0.0049).
    np.testing.assert_allclose(
        w[1], [1 / (1 + f(-1.01 + 1.0) + f(-1.015 + 1.0)), 1 / (1 + f(-1.015 + 1.01))],
        rtol=1e-6)
    # row 2: all equal -> e0 over 4 kept, e1 over the 3 left.
    np.testing.assert_allclose(w[2], [0.25, 1 / 3], rtol=1e-6)
    with pytest.raises(ValueError):
        orc.route(s, 3, 0, use_sparse_mixer=1)


def test_norm_router_known_answer(orc):
    x = np.array([[3.0, 4.0, 0.0, 0.0]], dtype=np.float32)     # mean(x^2) = 25/4
    skip = np.array([[1.0, -4.0, 0.0, 2.0]], dtype=np.float32)  # h = [4, 0, 0, 2], mean 5
    gamma = np.array([1.0, 2.0, 1.0, 0.5], dtype=np.float32)
    wr = np.array([[1.0, 0.0, 0.0, 0.0], [0.0, 0.0, 0.0, 1.0]], dtype=np.float32)
    n, lg, res = orc.norm_router(x, gamma, 0.0, wr, dtype=np.float32)
    np.testing.assert_allclose(n, [[3 / 2.5, 8 / 2.5, 0, 0]], rtol=1e-6)
    np.testing.assert_allclose(lg, [[1.2, 0.0]], rtol=1e-6, atol=1e-7)
    assert res is None
    n, lg, res = orc.norm_router(x, gamma, 0.0, wr, skip=skip, dtype=np.float32)
    r = math.sqrt(5.0)
    np.testing.assert_allclose(res, [[4, 0, 0, 2]])
    np.testing.assert_allclose(n, [[4 / r, 0, 0, 1 / r]], rtol=1e-6)
    np.testing.assert_allclose(lg, [[4 / r, 1 / r]], rtol=1e-6)


def test_round_bf16_matches_torch(orc):
    import torch
    a = np.random.default_rng(0).standard_normal(20000).astype(np.float32) * 37
    a[:4] = [0.0, -0.0, 1e-40, 3.3895313892515355e38]
    assert np.array_equal(orc.round_bf16(a), torch.from_numpy(a).to(torch.bfloat16).float().numpy())
