"""Full-size parity of the benchmark configurations C2-C5 (exact shapes and value
distributions of the bench workloads) through the C ABI.

At these sizes the float64 oracle cannot run the whole layer in seconds, so each test
checks what is size-independent on every row and samples the rest:

* routing indices (``moe_b200_route``, the kernel the layer runs) bit-exact against the
  oracle's ``route`` on ALL rows, and the expert-ordered permutation bit-exact against
  ``permutation`` on all T*k routed rows;
* layer outputs on a sample of rows (all rows for the small token counts) against an
  fp32 PyTorch re-computation of the layer with the oracle's routing and, for QMoE, the
  oracle's ``dequantize`` of each touched expert;
* determinism: two calls give identical bits.

Tolerances are the parity bar of the path (fp16: rtol 2e-2, atol 2e-3) on outputs in
units of their row's RMS, plus a per-row relative L2 bound (see ``_assert_parity``).
"""

import numpy as np
import pytest

from gpu_util import TOL, as_np

pytestmark = pytest.mark.gpu


def _gen(dev, seed):
    import torch
    return torch.Generator(device=dev).manual_seed(seed)


def _check_routing(pkg, orc, logits, k, E):
    """Indices of the device router vs the oracle on every row; the permutation of the
    device indices vs the oracle's permutation.  Returns the oracle's (idx, w)."""
    lg = logits.float().cpu().numpy()
    ridx, rw = orc.route(lg, k, 1)
    idx, w = pkg.route(logits, k, 1)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-6, atol=1e-7)
    offsets, pos, src = pkg.permute(idx, E)
    ro, rp, rs = orc.permutation(ridx, E)
    np.testing.assert_array_equal(offsets.cpu().numpy(), ro)
    np.testing.assert_array_equal(pos.cpu().numpy(), rp)
    np.testing.assert_array_equal(src.cpu().numpy(), rs)
    return ridx, rw


def _rows_reference(x_rows, idx_rows, w_rows, expert_weights):
    """fp32 layer output of the given rows, out[r] = sum_j w[r,j] * FFN_e(x[r]) with
    FFN_e(x) = (silu(x W1^T) * x W3^T) W2^T and the oracle's routing.
    expert_weights(e) -> (W1, W3, W2) as fp32 CUDA tensors [N, K]."""
    import torch
    xr = x_rows.float()
    out = torch.zeros_like(xr)
    idx_t = torch.from_numpy(idx_rows).to(xr.device)
    w_t = torch.from_numpy(w_rows.astype(np.float32)).to(xr.device)
    for e in sorted(set(int(v) for v in np.unique(idx_rows))):
        r, j = torch.nonzero(idx_t == e, as_tuple=True)
        W1, W3, W2 = expert_weights(e)
        xe = xr[r]
        a = torch.nn.functional.silu(xe @ W1.T) * (xe @ W3.T)
        out.index_add_(0, r, w_t[r, j][:, None] * (a @ W2.T))
        del W1, W3, W2
    return out.double().cpu().numpy()


# Largest per-row relative L2 error allowed: 4x the floor of an fp16 layer.
ROW_REL_L2 = 1e-3


def _assert_parity(got, ref):
    """The parity bar (fp16: rtol 2e-2, atol 2e-3) on outputs expressed in units of
    their row's RMS, and a per-row relative L2 error bound.

    The bar's atol is an absolute error at unit output scale.  The benchmark configs
    give outputs of RMS ~1 (C2, C4), ~14 (C3) and ~1250 (C5), and an fp16 layer holds
    the fc1 activation and each expert's fc2 row in fp16.  Those roundings alone, applied
    to the exact fp32 layer (a float64 simulation at C5 shapes), leave errors of std
    2.4e-4 x RMS and maxima of 4e-3 x RMS where two experts' rows cancel, so at C3/C5
    an unscaled atol of 2e-3 is unreachable for any fp16 implementation of the op.
    Scaled by the row RMS the bar reads |got - ref| <= 2e-2 |ref| + 2e-3 RMS_row."""
    rms = np.sqrt(np.mean(ref ** 2, axis=1, keepdims=True))
    err = np.abs(got - ref)
    bound = TOL["float16"]["rtol"] * np.abs(ref) + TOL["float16"]["atol"] * np.maximum(rms, 1.0)
    bad = err > bound
    assert not bad.any(), (f"{int(bad.sum())} of {got.size} outputs beyond the bar; max err "
                           f"{err.max():.4g}, row RMS {rms.min():.4g}..{rms.max():.4g}")
    rel = np.sqrt(np.sum((got - ref) ** 2, axis=1)) / np.maximum(
        np.sqrt(np.sum(ref ** 2, axis=1)), 1e-30)
    assert rel.max() <= ROW_REL_L2, f"row relative L2 error {rel.max():.3g} > {ROW_REL_L2}"


def _sample_rows(idx, per_expert, extra=(), at_least=512):
    """Row sample covering every expert: the first `per_expert` tokens routed to each
    expert, fixed rows (first, last, ...), then evenly spaced rows up to `at_least`."""
    T = idx.shape[0]
    rows = set(int(r) for r in extra)
    for e in np.unique(idx):
        tok = np.nonzero((idx == e).any(axis=1))[0]
        rows.update(int(t) for t in tok[:per_expert])
    step = max(1, T // max(1, at_least))
    for r in range(0, T, step):
        if len(rows) >= min(T, at_least):
            break
        rows.add(r)
    return np.array(sorted(rows), dtype=np.int64)


def _run_moe(pkg, d, attrs):
    op = pkg.MoE(**attrs)
    try:
        return op([d["x"], d["router_probs"], d["fc1_w"], None, d["fc2_w"], None, d["fc3_w"],
                   None])
    finally:
        op.release()


def _run_qmoe(pkg, q, attrs):
    op = pkg.QMoE(**attrs)
    try:
        return op([q["x"], q["router_probs"], q["fc1_q"], q["fc1_s"], None, q["fc2_q"],
                   q["fc2_s"], None, q["fc3_q"], q["fc3_s"], None])
    finally:
        op.release()


# ------------------------------------------------------------------------------ C2
def test_c2_mixtral_fp16_full_size(pkg, orc, dev):
    """C2: T=4096, H=4096, I=14336, E=8, k=2, SwiGLU, fp16.  >= 512 sampled rows, at
    least 64 per expert."""
    import torch
    g = _gen(dev, 20261202)
    T, H, I, E, k = 4096, 4096, 14336, 8, 2
    d = dict(x=torch.randn(T, H, device=dev, generator=g).half(),
             router_probs=torch.randn(T, E, device=dev, generator=g).half(),
             fc1_w=(torch.randn(E, I, H, device=dev, generator=g) * 0.02).half(),
             fc2_w=(torch.randn(E, H, I, device=dev, generator=g) * 0.02).half(),
             fc3_w=(torch.randn(E, I, H, device=dev, generator=g) * 0.02).half())
    attrs = dict(activation_type="silu", k=k, normalize_routing_weights=1)
    idx, w = _check_routing(pkg, orc, d["router_probs"], k, E)
    out1 = _run_moe(pkg, d, attrs)
    out2 = _run_moe(pkg, d, attrs)
    assert torch.equal(out1, out2), "layer output is not deterministic"
    rows = _sample_rows(idx, 72, extra=(0, 1, 2047, 2048, T - 1))
    assert len(rows) >= 512
    ref = _rows_reference(d["x"][rows], idx[rows], w[rows],
                          lambda e: (d["fc1_w"][e].float(), d["fc3_w"][e].float(),
                                     d["fc2_w"][e].float()))
    _assert_parity(as_np(out1[torch.from_numpy(rows).to(dev)]), ref)


# ------------------------------------------------------------------------------ C4
def test_c4_fine_grained_zipf_full_size(pkg, orc, dev):
    """C4: T=16384, H=2048, I=768, E=64, k=8, SwiGLU, fp16, logits plus a per-expert
    Zipf(1.1) bias rescaled to [0, 3].  All 131072 routed rows: indices and permutation
    bit-exact; >= 512 sampled output rows over all experts."""
    import torch
    g = _gen(dev, 20261204)
    T, H, I, E, k = 16384, 2048, 768, 64, 8
    z = np.random.default_rng(20261204).zipf(1.1, E).astype(np.float64)
    bias_e = 3.0 * (z - z.min()) / max(z.max() - z.min(), 1e-12)
    logits = (torch.randn(T, E, device=dev, generator=g)
              + torch.from_numpy(bias_e).float().to(dev)[None, :]).half()
    d = dict(x=torch.randn(T, H, device=dev, generator=g).half(), router_probs=logits,
             fc1_w=(torch.randn(E, I, H, device=dev, generator=g) * 0.02).half(),
             fc2_w=(torch.randn(E, H, I, device=dev, generator=g) * 0.02).half(),
             fc3_w=(torch.randn(E, I, H, device=dev, generator=g) * 0.02).half())
    attrs = dict(activation_type="silu", k=k, normalize_routing_weights=1)
    idx, w = _check_routing(pkg, orc, logits, k, E)
    counts = np.bincount(idx.ravel(), minlength=E)
    assert counts.max() > 2 * counts.mean(), "the Zipf bias should unbalance the experts"
    out1 = _run_moe(pkg, d, attrs)
    out2 = _run_moe(pkg, d, attrs)
    assert torch.equal(out1, out2), "layer output is not deterministic"
    rows = _sample_rows(idx, 12, extra=(0, 1, T // 2, T - 1))
    assert len(rows) >= 512
    ref = _rows_reference(d["x"][rows], idx[rows], w[rows],
                          lambda e: (d["fc1_w"][e].float(), d["fc3_w"][e].float(),
                                     d["fc2_w"][e].float()))
    _assert_parity(as_np(out1[torch.from_numpy(rows).to(dev)]), ref)


# ----------------------------------------------------------------------- QMoE C3/C5
def _qmoe_weights(dev, g, E, H, I, bits, block, mu, sigma):
    """Packed codes drawn as bytes on the device (int4: every nibble uniform in [0, 15],
    i.e. codes uniform in [-8, 7]; int8: stored bytes uniform in [1, 255], i.e. codes
    uniform in [-127, 127]) and fp16 lognormal scales, [E, N, K*bits/8] and [E, N(, nb)]."""
    import torch

    def one(N, K):
        if bits == 4:
            q = torch.randint(0, 256, (E, N, K // 2), device=dev, generator=g, dtype=torch.uint8)
        else:
            q = torch.randint(1, 256, (E, N, K), device=dev, generator=g, dtype=torch.uint8)
        shape = (E, N, (K + block - 1) // block) if block else (E, N)
        s = torch.empty(shape, device=dev).log_normal_(mu, sigma, generator=g).half()
        return q, s

    q1, s1 = one(I, H)
    q3, s3 = one(I, H)
    q2, s2 = one(H, I)
    return dict(fc1_q=q1, fc1_s=s1, fc3_q=q3, fc3_s=s3, fc2_q=q2, fc2_s=s2)


def _dequant_expert(orc, q, e, bits, block, H, I):
    """The oracle's dequantisation of expert e's three matrices, as fp32 CUDA tensors."""
    import torch
    dev = q["fc1_q"].device

    def dq(name, K):
        w = orc.dequantize(q[name + "_q"][e:e + 1].cpu().numpy(),
                           q[name + "_s"][e:e + 1].cpu().numpy(), bits, block, K)[0]
        return torch.from_numpy(w.astype(np.float32)).to(dev)

    return dq("fc1", H), dq("fc3", H), dq("fc2", I)


class _QWeights:
    """One QMoE configuration's weights (shared by the token counts of a test) and the
    oracle's dequantisation of each expert, computed once on first use."""

    def __init__(self, orc, dev, *, H, I, E, bits, block, mu, sigma, seed):
        self.orc, self.dev = orc, dev
        self.H, self.I, self.E, self.bits, self.block = H, I, E, bits, block
        self.q = _qmoe_weights(dev, _gen(dev, seed), E, H, I, bits, block, mu, sigma)
        self.cache = {}

    def expert(self, e):
        if e not in self.cache:
            self.cache[e] = _dequant_expert(self.orc, self.q, e, self.bits, self.block,
                                            self.H, self.I)
        return self.cache[e]


def _qmoe_case(pkg, orc, dev, W, *, T, k, seed, sample):
    import torch
    g = _gen(dev, seed)
    q = dict(W.q)
    q["x"] = torch.randn(T, W.H, device=dev, generator=g).half()
    q["router_probs"] = torch.randn(T, W.E, device=dev, generator=g).half()
    attrs = dict(activation_type="silu", k=k, normalize_routing_weights=1,
                 expert_weight_bits=W.bits, block_size=W.block)
    idx, w = _check_routing(pkg, orc, q["router_probs"], k, W.E)
    out1 = _run_qmoe(pkg, q, attrs)
    out2 = _run_qmoe(pkg, q, attrs)
    assert torch.equal(out1, out2), "layer output is not deterministic"
    rows = np.arange(T) if sample is None else _sample_rows(idx, sample, extra=(0, T - 1))
    rows_t = torch.from_numpy(rows).to(dev)
    ref = _rows_reference(q["x"][rows_t], idx[rows], w[rows], W.expert)
    _assert_parity(as_np(out1[rows_t]), ref)
    return len(rows)


@pytest.fixture(scope="module")
def c3_weights(orc, dev):
    return _QWeights(orc, dev, H=4096, I=14336, E=8, bits=4, block=128, mu=-5.0, sigma=0.3,
                     seed=20261203)


@pytest.fixture(scope="module")
def c5_weights(orc, dev):
    return _QWeights(orc, dev, H=4096, I=6400, E=16, bits=8, block=0, mu=-6.0, sigma=0.25,
                     seed=20261205)


@pytest.mark.parametrize("T", [1, 8, 32, 64])
def test_c3_qmoe_int4_block128_full_size(pkg, orc, dev, c3_weights, T):
    """C3: Mixtral shape (H=4096, I=14336, E=8, k=2, SwiGLU), int4 codes uniform in
    [-8, 7] with fp16 block-128 scales lognormal(-5, 0.3); every output row checked."""
    _qmoe_case(pkg, orc, dev, c3_weights, T=T, k=2, seed=20261303 + T, sample=None)


@pytest.mark.parametrize("T", [1, 64, 1024, 16384, 65536])
def test_c5_qmoe_int8_per_row_full_size(pkg, orc, dev, c5_weights, T):
    """C5: H=4096, I=6400, E=16, k=2, SwiGLU, int8 codes uniform in [-127, 127] with one
    fp16 scale per output row, lognormal(-6, 0.25).  T=1/64 run the decode kernels,
    1024/16384 the code-converting tensor-core GEMM, 65536 (T*k > 16384) dequantises to
    HBM before the plain GEMMs.  Every row up to T=1024, else >= 512 sampled rows."""
    n = _qmoe_case(pkg, orc, dev, c5_weights, T=T, k=2, seed=20261305 + T,
                   sample=None if T <= 1024 else 40)
    assert n >= min(T, 512)
