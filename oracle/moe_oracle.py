"""CPU oracle for the com.microsoft MoE / QMoE hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this module, and only as the checker.  The product path (the CUDA library
under ``onnxruntime-musa_b200/``) never calls into it.

PARITY UNPINNED.  The arithmetic of this path is defined by the stock ONNX Runtime
1.26.0 CPU execution provider's ``com.microsoft::MoE`` and ``::QMoE`` kernels
(onnxruntime v1.26.0, commit 8c546c37b43caaca1fa25db430dab94b901cf277, the
submodule pinned at ``third_party/README.md:5-6`` of the reference).  That source is
an un-vendored submodule (``third_party/onnxruntime/`` is empty), the ``onnxruntime``
wheel is not installable offline, and the reference itself has no MoE kernel and no
MoE test, golden vector or fixture.  This file therefore restates the operator
contract from the published ``com.microsoft`` MoE/QMoE operator schema; it is pinned
only by the hand-computed known answers in ``tests/test_oracle.py``.

Conventions fixed here (and by the CUDA kernels, bit for bit where integer):

* Routing (``route``): the router input holds logits.  Each row is read as fp32.
  Top-k orders experts by value descending, ties to the LOWER expert index -- the
  rule of the reference's own TopK (``musa/ep/src/kernels/math/topk_impl.mu:46-65``,
  ``TopKPairBefore``).  Weights: with ``normalize_routing_weights`` the softmax is
  taken over the k selected logits; without it, over all E logits and the k
  selected probabilities are returned (softmax over the row, analog
  ``musa/ep/src/kernels/math/softmax_impl.mu:49-84``, fp32-or-wider accumulation).
  ``use_sparse_mixer=1`` (k = 2) is the sparse-mixer router published with Phi-3.5-MoE
  (``sparsemixer``, inference form, jitter_eps = 0.01), restated in
  ``route_sparse_mixer``; the ORT 1.26.0 source that would pin its details is absent.
* Permutation (``permutation``): rows routed to expert e are laid out contiguously,
  experts ascending; inside one expert, by token then by slot j.  ``offsets[e]`` is the
  exclusive prefix sum of the per-expert counts (analog: the reference's CumSum,
  ``musa/ep/src/kernels/math/cumsum_impl.mu:17``).
* Expert FFN: weights are ``[E, N, K]`` (each row one output channel, K contiguous).
  fc1 gives the gate pre-activation; with fc3 present the result is
  ``act(fc1(x)) * fc3(x)``; ``activation_type='swiglu'`` uses
  ``g * sigmoid(alpha * g) * (l + beta)`` with ``g = min(g, limit)``,
  ``l = clip(l, -limit, limit)`` where (g, l) come from fc1/fc3
  (``swiglu_fusion=0``), interleaved rows of fc1 (``1``) or its two halves (``2``).
  GELU is the erf form.  Biases are added before the activation / combine.
* Combine: ``out[t] = sum_j w[t, j] * y[t, j]`` in slot order.
* QMoE dequantisation (``dequantize``): symmetric codes stored unsigned with the
  implicit zero point 2^(bits-1); int4 packs element 2i in the low nibble and
  2i+1 in the high nibble of byte i along K; scales are ``[E, N]``
  (``block_size=0``) or ``[E, N, ceil(K / block_size)]``.

All arithmetic below is float64 (inputs are first read in their storage type).
"""

from __future__ import annotations

import math

import numpy as np

ACTIVATIONS = ("relu", "gelu", "silu", "identity", "swiglu")


# ----------------------------------------------------------------------------- routing

SPARSE_MIXER_JITTER_EPS = 0.01


def route_sparse_mixer(router_probs: np.ndarray, jitter_eps: float = SPARSE_MIXER_JITTER_EPS):
    """Sparse-mixer top-2 routing.  For each of two picks: m = the largest remaining
    logit and e* its expert (ties to the lower index; the second pick excludes the first);
    experts with ``(m - s_e) / max(|s_e|, m) > 2 * jitter_eps`` are dropped, and the pick's
    weight is ``1 / sum over kept e of exp(s_e - m)`` (its softmax probability over the
    kept experts).  The mask tests are evaluated in IEEE float32, as the kernel does."""
    s = np.asarray(router_probs).astype(np.float32)
    s = np.where(np.isnan(s), np.float32(-np.inf), s)
    T, E = s.shape
    if E < 2:
        raise ValueError("the sparse mixer needs at least two experts")
    idx = np.zeros((T, 2), dtype=np.int32)
    w = np.zeros((T, 2), dtype=np.float32)
    thr = np.float32(2.0) * np.float32(jitter_eps)
    avail = np.ones((T, E), dtype=bool)
    rows = np.arange(T)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        for r in range(2):
            cand = np.where(avail, s, np.float32(-np.inf))
            pick = np.argmax(cand, axis=1)          # first maximum: the lower index
            m = cand[rows, pick][:, None]
            ratio = (m - s) / np.maximum(np.abs(s), m)   # float32 throughout
            keep = avail & ~(ratio > thr)
            den = np.where(keep, np.exp(s.astype(np.float64) - m.astype(np.float64)), 0.0)
            idx[:, r] = pick
            w[:, r] = (1.0 / den.sum(axis=1)).astype(np.float32)
            avail[rows, pick] = False
    return idx, w


def route(router_probs: np.ndarray, k: int, normalize_routing_weights: int,
          use_sparse_mixer: int = 0):
    """Top-k routing of every row.  Returns (expert_idx int32 [T,k], weight f32 [T,k]).

    The tie rule (value descending, lower index first) follows
    ``musa/ep/src/kernels/math/topk_impl.mu:46-65``; the softmax follows
    ``musa/ep/src/kernels/math/softmax_impl.mu:49-84`` (max-subtracted exp, sum,
    divide), evaluated here in float64.
    """
    if use_sparse_mixer:
        if k != 2:
            raise ValueError("use_sparse_mixer routes top-2 (k must be 2)")
        return route_sparse_mixer(router_probs)
    logits = np.asarray(router_probs).astype(np.float32)
    logits = np.where(np.isnan(logits), np.float32(-np.inf), logits)  # NaN reads as -inf
    T, E = logits.shape
    if not (1 <= k <= E):
        raise ValueError(f"k={k} must be in [1, {E}]")
    # Stable argsort of the negated values keeps lower indices first among equal
    # values (-0.0 and 0.0 compare equal, as in the kernel's comparison).
    order = np.argsort(-logits, axis=1, kind="stable")
    idx = order[:, :k].astype(np.int32)
    sel = np.take_along_axis(logits, idx, axis=1).astype(np.float64)
    if normalize_routing_weights:
        m = sel[:, :1]
        e = np.exp(sel - m)
        w = e / e.sum(axis=1, keepdims=True)
    else:
        lg = logits.astype(np.float64)
        m = lg.max(axis=1, keepdims=True)
        denom = np.exp(lg - m).sum(axis=1, keepdims=True)
        w = np.exp(sel - m) / denom
    return idx, w.astype(np.float32)


def round_bf16(a) -> np.ndarray:
    """float32 values rounded to the nearest bfloat16 (ties to even), kept as float32."""
    u = np.ascontiguousarray(np.asarray(a, dtype=np.float32)).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    out = r.view(np.float32)
    return np.where(np.isnan(a), np.float32(np.nan), out)


def norm_router(x, gamma, epsilon, router_weight, skip=None, dtype=np.float16):
    """Pre-MoE rows: h = x (+ skip) summed in float32; residual = h in ``dtype``;
    normed = dtype(h * 1/sqrt(mean(h^2) + eps) * gamma) (the reference's RmsNormKernel,
    ``musa/ep/src/kernels/nn/rms_norm_impl.mu:10-45``: fp32 gamma, value * inv * gamma);
    logits = dtype(normed . router_weight[e]) over the ROUNDED normed values (the router
    MatMul consumes the stored tensor).  Norm and dot products in float64."""
    h = np.asarray(x).astype(np.float32)
    if skip is not None:
        h = h + np.asarray(skip).astype(np.float32)
    cast = ((lambda a: round_bf16(np.asarray(a, dtype=np.float32))) if dtype == "bfloat16"
            else (lambda a: a.astype(dtype)))
    residual = cast(h) if skip is not None else None
    hd = h.astype(np.float64)
    inv = 1.0 / np.sqrt((hd * hd).mean(axis=1, keepdims=True) + float(epsilon))
    normed = cast(hd * inv * np.asarray(gamma, dtype=np.float64)[None, :])
    logits = cast(normed.astype(np.float64) @ np.asarray(router_weight).astype(np.float64).T)
    return normed, logits, residual


def permutation(expert_idx: np.ndarray, num_experts: int):
    """Canonical dispatch order.  Returns (offsets int32 [E+1], pos int32 [T,k],
    src int32 [T*k]) where ``src[p]`` is the flat (t*k + j) routed row at permuted
    position p and ``pos[t, j]`` is its inverse."""
    T, k = expert_idx.shape
    flat = expert_idx.reshape(-1).astype(np.int64)
    if flat.size and (flat.min() < 0 or flat.max() >= num_experts):
        raise ValueError("expert index out of range")
    counts = np.bincount(flat, minlength=num_experts)
    offsets = np.zeros(num_experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    src = np.argsort(flat, kind="stable").astype(np.int32)
    pos = np.empty(T * k, dtype=np.int32)
    pos[src] = np.arange(T * k, dtype=np.int32)
    return offsets, pos.reshape(T, k), src


# ----------------------------------------------------------------------------- QMoE

def pack_int4(codes: np.ndarray) -> np.ndarray:
    """Signed int4 codes in [-8, 7], shape [..., K] (K even) -> uint8 [..., K/2]."""
    q = (codes.astype(np.int16) + 8).astype(np.uint8)
    return (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)


def pack_int8(codes: np.ndarray) -> np.ndarray:
    """Signed int8 codes in [-128, 127] -> uint8 with zero point 128."""
    return (codes.astype(np.int16) + 128).astype(np.uint8)


def dequantize(packed: np.ndarray, scales: np.ndarray, bits: int, block_size: int,
               K: int) -> np.ndarray:
    """uint8 weights [E, N, K*bits/8] + scales -> float64 [E, N, K]."""
    packed = np.asarray(packed, dtype=np.uint8)
    if bits == 4:
        lo = (packed & 0x0F).astype(np.int16)
        hi = (packed >> 4).astype(np.int16)
        q = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=np.int16)
        q[..., 0::2] = lo
        q[..., 1::2] = hi
        q = q[..., :K] - 8
    elif bits == 8:
        q = packed.astype(np.int16)[..., :K] - 128
    else:
        raise ValueError("expert_weight_bits must be 4 or 8")
    s = np.asarray(scales).astype(np.float64)
    if block_size == 0:
        if s.ndim != 2:
            raise ValueError("per-row scales must be [E, N]")
        return q.astype(np.float64) * s[..., None]
    nb = (K + block_size - 1) // block_size
    if s.shape[-1] != nb:
        raise ValueError(f"block scales must have {nb} blocks per row")
    s_full = np.repeat(s, block_size, axis=-1)[..., :K]
    return q.astype(np.float64) * s_full


# ----------------------------------------------------------------------------- FFN

def _act(name, x, alpha=1.0, beta=0.0, limit=math.inf, lin=None):
    if name == "relu":
        return np.maximum(x, 0.0)
    if name == "gelu":
        from scipy.special import erf  # scipy is part of the image
        return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))
    if name == "silu":
        return x / (1.0 + np.exp(-x))
    if name == "identity":
        return x
    if name == "swiglu":
        g = np.minimum(x, limit)
        l = np.clip(lin, -limit, limit)
        return g / (1.0 + np.exp(-alpha * g)) * (l + beta)
    raise ValueError(f"unknown activation_type {name!r}")


def expert_ffn(xe, W1, b1, W2, b2, W3=None, b3=None, *, activation_type="relu",
               swiglu_fusion=0, activation_alpha=1.0, activation_beta=0.0,
               swiglu_limit=math.inf):
    """float64 FFN of one expert on rows ``xe`` [M, H]; W* are that expert's [N, K]
    matrices and b* its bias vectors (or None)."""
    xe = np.asarray(xe).astype(np.float64)
    f64 = lambda a: None if a is None else np.asarray(a).astype(np.float64)
    W1, W2, W3, b1, b2, b3 = map(f64, (W1, W2, W3, b1, b2, b3))
    h = xe @ W1.T
    if b1 is not None:
        h = h + b1
    if activation_type == "swiglu":
        if W3 is not None and swiglu_fusion == 0:
            u = xe @ W3.T
            if b3 is not None:
                u = u + b3
            g = h
        elif swiglu_fusion == 1:
            g, u = h[:, 0::2], h[:, 1::2]
        elif swiglu_fusion == 2:
            half = h.shape[1] // 2
            g, u = h[:, :half], h[:, half:]
        else:
            raise ValueError("swiglu needs fc3 weights or swiglu_fusion 1/2")
        a = _act("swiglu", g, activation_alpha, activation_beta, swiglu_limit, u)
    else:
        a = _act(activation_type, h)
        if W3 is not None:
            u = xe @ W3.T
            if b3 is not None:
                u = u + b3
            a = a * u
    y = a @ W2.T
    if b2 is not None:
        y = y + b2
    return y


def moe(x, router_probs, fc1_w, fc1_b, fc2_w, fc2_b, fc3_w=None, fc3_b=None, *,
        activation_type="relu", k=1, normalize_routing_weights=0, swiglu_fusion=0,
        activation_alpha=1.0, activation_beta=0.0, swiglu_limit=math.inf,
        use_sparse_mixer=0, return_routing=False):
    """float64 reference of one MoE layer call.  ``x`` is [T,H] (or [B,S,H]);
    ``fc*_w`` are [E, N, K] (already dequantised for QMoE)."""
    x = np.asarray(x)
    shape = x.shape
    X = x.reshape(-1, shape[-1]).astype(np.float64)
    T, H = X.shape
    E = fc1_w.shape[0]
    idx, w = route(np.asarray(router_probs).reshape(T, E), k, normalize_routing_weights,
                   use_sparse_mixer)
    out = np.zeros((T, H), dtype=np.float64)
    sel = lambda a, e: None if a is None else np.asarray(a)[e]
    for e in range(E):
        tok, slot = np.nonzero(idx == e)
        if tok.size == 0:
            continue
        y = expert_ffn(X[tok], sel(fc1_w, e), sel(fc1_b, e), sel(fc2_w, e), sel(fc2_b, e),
                       sel(fc3_w, e), sel(fc3_b, e), activation_type=activation_type,
                       swiglu_fusion=swiglu_fusion, activation_alpha=activation_alpha,
                       activation_beta=activation_beta, swiglu_limit=swiglu_limit)
        out[tok] += w[tok, slot].astype(np.float64)[:, None] * y
    out = out.reshape(shape)
    if return_routing:
        return out, idx, w
    return out


def qmoe(x, router_probs, fc1_q, fc1_scales, fc1_b, fc2_q, fc2_scales, fc2_b,
         fc3_q=None, fc3_scales=None, fc3_b=None, *, expert_weight_bits=4,
         block_size=0, **attrs):
    """float64 reference of one QMoE layer call (dequantise, then ``moe``)."""
    H = np.asarray(x).shape[-1]
    W1 = dequantize(fc1_q, fc1_scales, expert_weight_bits, block_size, H)
    I2 = W1.shape[1]
    # fc2 consumes the activation width (= fc1 rows, halved for fused swiglu).
    fused = attrs.get("activation_type") == "swiglu" and attrs.get("swiglu_fusion", 0) in (1, 2)
    I = I2 // 2 if fused else I2
    W2 = dequantize(fc2_q, fc2_scales, expert_weight_bits, block_size, I)
    W3 = None if fc3_q is None else dequantize(fc3_q, fc3_scales, expert_weight_bits,
                                               block_size, H)
    return moe(x, router_probs, W1, fc1_b, W2, fc2_b, W3, fc3_b, **attrs)


# ----------------------------------------------------------------------------- inputs

CONFIGS = {
    # name: (T, H, I, E, k, activation, gated, dtype, bias)
    "c1_fp32_silu": dict(T=256, H=512, I=1024, E=8, k=2, act="silu", gated=False,
                         dtype="float32", bias=True, normalize=1),
    "c2_mixtral_fp16": dict(T=4096, H=4096, I=14336, E=8, k=2, act="silu", gated=True,
                            dtype="float16", bias=False, normalize=1),
    "c4_fine_fp16": dict(T=16384, H=2048, I=768, E=64, k=8, act="silu", gated=True,
                         dtype="float16", bias=False, normalize=1, zipf=True),
}


def make_moe_inputs(T, H, I, E, k, act="silu", gated=True, dtype="float16", bias=False,
                    normalize=1, zipf=False, seed=20261201):
    """Seeded synthetic inputs with the distributions of the benchmark configs:
    x, logits ~ N(0,1); weights ~ N(0, 0.02); biases ~ N(0, 0.01); an optional
    Zipf(1.1) per-expert logit bias rescaled to [0, 3] for load imbalance."""
    rng = np.random.default_rng(seed)
    dt = np.dtype(dtype) if dtype != "bfloat16" else np.float32
    x = rng.standard_normal((T, H), dtype=np.float32)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    if zipf:
        z = rng.zipf(1.1, E).astype(np.float64)
        span = z.max() - z.min()
        bias_e = 3.0 * (z - z.min()) / span if span > 0 else np.zeros(E)
        logits = (logits + bias_e[None, :]).astype(np.float32)
    w1 = (rng.standard_normal((E, I, H), dtype=np.float32) * 0.02)
    w2 = (rng.standard_normal((E, H, I), dtype=np.float32) * 0.02)
    w3 = (rng.standard_normal((E, I, H), dtype=np.float32) * 0.02) if gated else None
    b1 = (rng.standard_normal((E, I), dtype=np.float32) * 0.01) if bias else None
    b2 = (rng.standard_normal((E, H), dtype=np.float32) * 0.01) if bias else None
    b3 = (rng.standard_normal((E, I), dtype=np.float32) * 0.01) if (bias and gated) else None
    cast = (lambda a: None if a is None else a.astype(dt))
    return dict(x=cast(x), router_probs=cast(logits), fc1_w=cast(w1), fc1_b=cast(b1),
                fc2_w=cast(w2), fc2_b=cast(b2), fc3_w=cast(w3), fc3_b=cast(b3),
                attrs=dict(activation_type=act, k=k, normalize_routing_weights=normalize))


def make_qmoe_inputs(T, H, I, E, k, bits, block_size, scale_mu, scale_sigma,
                     seed=20261203):
    """Seeded QMoE inputs: codes uniform in [-8,7] (int4) or [-127,127] (int8),
    fp16 scales lognormal(mu, sigma), x and logits ~ N(0,1), SwiGLU via fc3."""
    rng = np.random.default_rng(seed)
    lo, hi = (-8, 7) if bits == 4 else (-127, 127)
    x = rng.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    logits = rng.standard_normal((T, E), dtype=np.float32).astype(np.float16)

    def weights(N, K):
        codes = rng.integers(lo, hi + 1, size=(E, N, K), dtype=np.int16)
        packed = pack_int4(codes) if bits == 4 else pack_int8(codes)
        if block_size:
            nb = (K + block_size - 1) // block_size
            sc = rng.lognormal(scale_mu, scale_sigma, size=(E, N, nb))
        else:
            sc = rng.lognormal(scale_mu, scale_sigma, size=(E, N))
        return packed, sc.astype(np.float16)

    q1, s1 = weights(I, H)
    q3, s3 = weights(I, H)
    q2, s2 = weights(H, I)
    return dict(x=x, router_probs=logits, fc1_q=q1, fc1_scales=s1, fc2_q=q2,
                fc2_scales=s2, fc3_q=q3, fc3_scales=s3,
                attrs=dict(activation_type="silu", k=k, normalize_routing_weights=1,
                           expert_weight_bits=bits, block_size=block_size))
