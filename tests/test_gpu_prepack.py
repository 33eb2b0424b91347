"""QMoE weight prepack: parity of prefill calls on prepacked weights against the oracle
and the per-call dequantisation path, the row threshold, and content-keyed sharing."""

import os

import numpy as np
import pytest

from gpu_util import TOL, as_np, to_dev

pytestmark = pytest.mark.gpu

# Routed rows (T * k) up to which QMoE calls take the decode kernels (packed codes).
DECODE_MAX_ROWS = 512

CASES = [
    # (T, H, I, E, k, bits, block_size)
    (1100, 512, 384, 8, 2, 8, 0),     # int8 per-row scales
    (1030, 384, 512, 8, 2, 4, 128),   # int4 blocks of 128
    (600, 256, 320, 16, 4, 4, 32),    # int4 blocks of 32, k = 4
]


def _inputs(orc, case, seed):
    T, H, I, E, k, bits, bs = case
    mu = -5.0 if bits == 4 else -8.5
    q = orc.make_qmoe_inputs(T=T, H=H, I=I, E=E, k=k, bits=bits, block_size=bs,
                             scale_mu=mu, scale_sigma=0.3, seed=seed)
    return q, dict(q["attrs"], k=k)


def _input_list(q, dev):
    get = lambda n: to_dev(q[n], dev) if q.get(n) is not None else None
    return [get("x"), get("router_probs"), get("fc1_q"), get("fc1_scales"), None,
            get("fc2_q"), get("fc2_scales"), None, get("fc3_q"), get("fc3_scales"), None]


def _oracle(orc, q, attrs):
    return orc.qmoe(q["x"], q["router_probs"], q["fc1_q"], q["fc1_scales"], None, q["fc2_q"],
                    q["fc2_scales"], None, q["fc3_q"], q["fc3_scales"], None, **attrs)


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"T{c[0]}E{c[3]}k{c[4]}b{c[5]}bs{c[6]}")
def test_kernel_prepack_parity(pkg, orc, dev, case):
    """A QMoE kernel object after pre-pack: prefill output within fp16 tolerance of the
    oracle and bit-identical to the per-call dequantise-to-HBM path (the same GEMMs on the
    same dequantised values)."""
    q, attrs = _inputs(orc, case, seed=sum(case))
    assert case[0] * case[4] > DECODE_MAX_ROWS
    ins = _input_list(q, dev)
    op = pkg.QMoE(**attrs)
    try:
        assert op.prepack(ins, share=False) is False
        out = op(ins)
    finally:
        op.release()
    np.testing.assert_allclose(as_np(out), _oracle(orc, q, attrs), **TOL["float16"])
    os.environ["MOE_B200_QMOE_DEQUANT"] = "1"
    try:
        op2 = pkg.QMoE(**attrs)
        try:
            ref = op2(ins)
        finally:
            op2.release()
    finally:
        del os.environ["MOE_B200_QMOE_DEQUANT"]
    np.testing.assert_array_equal(as_np(out).view(np.uint16), as_np(ref).view(np.uint16))


def test_below_threshold_and_other_weights(pkg, orc, dev):
    """Decode-sized calls, and calls under MOE_B200_PREPACK_MIN_ROWS when it is set, run
    the packed-code kernels exactly as without a prepack; a call whose weight inputs are
    other tensors ignores the prepack."""
    import torch
    case = (1100, 512, 384, 8, 2, 8, 0)
    q, attrs = _inputs(orc, case, seed=5)
    ins = _input_list(q, dev)
    plain = pkg.QMoE(**attrs)
    packed = pkg.QMoE(**attrs)
    try:
        packed.prepack(ins)
        for T in (1, 16, 256):  # T*k = 2, 32, 512: decode kernels
            small = [ins[0][:T].contiguous(), ins[1][:T].contiguous()] + ins[2:]
            a, b = plain(small), packed(small)
            np.testing.assert_array_equal(as_np(a).view(np.uint16), as_np(b).view(np.uint16))
        os.environ["MOE_B200_PREPACK_MIN_ROWS"] = "2048"
        try:  # T*k = 600 < 2048: the code-converting GEMM, as without a prepack
            small = [ins[0][:300].contiguous(), ins[1][:300].contiguous()] + ins[2:]
            a, b = plain(small), packed(small)
        finally:
            del os.environ["MOE_B200_PREPACK_MIN_ROWS"]
        np.testing.assert_array_equal(as_np(a).view(np.uint16), as_np(b).view(np.uint16))
        # Same shapes, other weights: the prepack must not be used.
        q2, _ = _inputs(orc, case, seed=6)
        ins2 = ins[:2] + _input_list(q2, dev)[2:]
        a, b = plain(ins2), packed(ins2)
        np.testing.assert_array_equal(as_np(a).view(np.uint16), as_np(b).view(np.uint16))
        ref2 = _oracle(orc, dict(q2, x=q["x"], router_probs=q["router_probs"]), attrs)
        np.testing.assert_allclose(as_np(b), ref2, **TOL["float16"])
    finally:
        plain.release()
        packed.release()
    torch.cuda.synchronize()


def test_explicit_api_and_threshold_override(pkg, orc, dev):
    """moe_b200_prepack_create + forward_prepacked with a caller workspace: the workspace
    shrinks by the dequantised copies, the output matches the kernel-object path, and
    MOE_B200_PREPACK_MIN_ROWS moves the switch-over."""
    import torch
    case = (700, 256, 384, 8, 2, 4, 64)
    q, attrs = _inputs(orc, case, seed=11)
    T, H, I, E, k, bits, bs = case
    t = {n: to_dev(q[m], dev) for n, m in [("input", "x"), ("router_probs", "router_probs"),
                                           ("fc1_weights", "fc1_q"), ("fc1_scales", "fc1_scales"),
                                           ("fc2_weights", "fc2_q"), ("fc2_scales", "fc2_scales"),
                                           ("fc3_weights", "fc3_q"), ("fc3_scales", "fc3_scales")]}
    out = torch.empty(T, H, dtype=torch.float16, device=dev)
    t["output"] = out
    prob = pkg.make_problem(T, H, I, E, pkg.FLOAT16, has_fc3=True, activation_type="silu", k=k,
                            normalize_routing_weights=1, expert_weight_bits=bits, block_size=bs)
    with pkg.Prepacked(prob, t) as pk:
        nbytes, refs = pk.info()
        assert refs == 1 and nbytes >= E * 3 * H * I * 2
        ref = _oracle(orc, q, attrs)
        # The code-converting path needs no dequantised copies either: same workspace.
        ws_pk = pkg.workspace_size(prob, pk)
        assert ws_pk == pkg.workspace_size(prob)
        ws = torch.empty(ws_pk, dtype=torch.uint8, device=dev)
        os.environ["MOE_B200_PREPACK_MIN_ROWS"] = "2048"
        try:  # T*k = 1400 < 2048: the prepack is not taken
            pkg.forward(prob, t, ws, prepacked=pk)
            torch.cuda.synchronize()
            conv = as_np(out).copy()
        finally:
            del os.environ["MOE_B200_PREPACK_MIN_ROWS"]
        np.testing.assert_allclose(conv, ref, **TOL["float16"])
        pkg.forward(prob, t, ws, prepacked=pk)
        torch.cuda.synchronize()
        np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])
        os.environ["MOE_B200_QMOE_DEQUANT"] = "1"
        try:
            ws2 = torch.empty(pkg.workspace_size(prob), dtype=torch.uint8, device=dev)
            assert ws2.numel() > ws_pk  # the per-call path holds the dequantised copies
            out2 = torch.empty_like(out)
            pkg.forward(prob, dict(t, output=out2), ws2)
            torch.cuda.synchronize()
        finally:
            del os.environ["MOE_B200_QMOE_DEQUANT"]
        np.testing.assert_array_equal(as_np(out).view(np.uint16), as_np(out2).view(np.uint16))
        # A prepack of other shapes is refused.
        prob_bad = pkg.make_problem(T, H, I, E, pkg.FLOAT16, has_fc3=True, activation_type="silu",
                                    k=k, normalize_routing_weights=1, expert_weight_bits=bits,
                                    block_size=bs * 2)
        with pytest.raises(pkg.InvalidArgument):
            pkg.forward(prob_bad, t, ws, prepacked=pk)


def test_sharing_by_content(pkg, orc, dev):
    """share=True: equal content at other addresses maps to one prepack (reference
    counted, freed with the last release); different content or share=False does not."""
    import torch
    case = (64, 256, 256, 4, 2, 8, 0)
    q, attrs = _inputs(orc, case, seed=21)
    T, H, I, E, k, bits, bs = case
    prob = pkg.make_problem(T, H, I, E, pkg.FLOAT16, has_fc3=True, activation_type="silu", k=k,
                            normalize_routing_weights=1, expert_weight_bits=bits, block_size=bs)

    def weights(qq):
        return {n: to_dev(qq[m], dev) for n, m in
                [("fc1_weights", "fc1_q"), ("fc1_scales", "fc1_scales"), ("fc2_weights", "fc2_q"),
                 ("fc2_scales", "fc2_scales"), ("fc3_weights", "fc3_q"),
                 ("fc3_scales", "fc3_scales")]}

    wa, wb = weights(q), weights(q)  # same content, separate allocations
    assert wa["fc1_weights"].data_ptr() != wb["fc1_weights"].data_ptr()
    a = pkg.Prepacked(prob, wa, share=True)
    b = pkg.Prepacked(prob, wb, share=True)
    assert a.handle.value == b.handle.value and a.info()[1] == 2
    c = pkg.Prepacked(prob, wb, share=False)
    assert c.handle.value != a.handle.value and c.info()[1] == 1
    wd = weights(q)
    wd["fc2_scales"][0, 0] += 1  # one changed scale: other content
    d = pkg.Prepacked(prob, wd, share=True)
    assert d.handle.value != a.handle.value
    b.release()
    assert a.info()[1] == 1
    a.release()
    e = pkg.Prepacked(prob, wa, share=True)  # registry entry gone: a new prepack
    assert e.info()[1] == 1
    for x in (c, d, e):
        x.release()
    torch.cuda.synchronize()


def test_pipeline_with_prepack_and_mixed_sizes(pkg, orc, dev):
    """Host-buffer pipeline over a QMoE layer: calls of prefill size (prepacked weights),
    of the code-converting GEMM's size and of decode size through one pipeline, each
    against the oracle."""
    import torch
    case = (1100, 256, 384, 8, 2, 8, 0)
    q, attrs = _inputs(orc, case, seed=31)
    T, H, I, E, k, bits, bs = case
    w = {n: to_dev(q[m], dev) for n, m in
         [("fc1_weights", "fc1_q"), ("fc1_scales", "fc1_scales"), ("fc2_weights", "fc2_q"),
          ("fc2_scales", "fc2_scales"), ("fc3_weights", "fc3_q"), ("fc3_scales", "fc3_scales")]}
    prob = pkg.make_problem(T, H, I, E, pkg.FLOAT16, has_fc3=True, activation_type="silu", k=k,
                            normalize_routing_weights=1, expert_weight_bits=bits, block_size=bs)
    hx = torch.from_numpy(q["x"]).pin_memory()
    hl = torch.from_numpy(q["router_probs"]).pin_memory()
    sizes = [T, 300, 3]
    outs = [torch.empty(n, H, dtype=torch.float16).pin_memory() for n in sizes]
    with pkg.Prepacked(prob, w) as pk, pkg.Pipeline(prob, w, depth=2) as pl:
        pl.set_prepacked(pk)
        assert pk.info()[1] == 2  # the pipeline holds a reference
        for n, o in zip(sizes, outs):
            pl.submit(hx[:n], hl[:n], o)
        pl.synchronize()
    for n, o in zip(sizes, outs):
        ref = _oracle(orc, dict(q, x=q["x"][:n], router_probs=q["router_probs"][:n]), attrs)
        np.testing.assert_allclose(o.numpy(), ref, **TOL["float16"])


def test_sharing_refuses_hash_collisions(pkg, orc, dev):
    """The sharing key is an order-independent sum over 8-byte words, so swapping two
    different words of the codes gives a colliding key for other weights; the registry
    compares the dequantised copies and gives the new weights a prepack of their own."""
    import torch
    case = (64, 256, 256, 4, 2, 8, 0)
    q, attrs = _inputs(orc, case, seed=23)
    T, H, I, E, k, bits, bs = case
    prob = pkg.make_problem(T, H, I, E, pkg.FLOAT16, has_fc3=True, activation_type="silu", k=k,
                            normalize_routing_weights=1, expert_weight_bits=bits, block_size=bs)

    def weights(qq):
        return {n: to_dev(np.ascontiguousarray(qq[m]), dev) for n, m in
                [("fc1_weights", "fc1_q"), ("fc1_scales", "fc1_scales"), ("fc2_weights", "fc2_q"),
                 ("fc2_scales", "fc2_scales"), ("fc3_weights", "fc3_q"),
                 ("fc3_scales", "fc3_scales")]}

    q2 = dict(q)
    codes = q["fc1_q"].copy()
    flat = codes.reshape(-1).view(np.uint64)
    j = int(np.nonzero(flat != flat[0])[0][0])
    flat[0], flat[j] = flat[j].copy(), flat[0].copy()  # same multiset of words, other weights
    q2["fc1_q"] = codes
    a = pkg.Prepacked(prob, weights(q), share=True)
    b = pkg.Prepacked(prob, weights(q2), share=True)
    assert b.handle.value != a.handle.value, "colliding weights shared a prepack"
    assert a.info()[1] == 1 and b.info()[1] == 1
    c = pkg.Prepacked(prob, weights(q2), share=True)  # equal to b: shared with b
    assert c.handle.value == b.handle.value and b.info()[1] == 2
    for x in (c, b, a):
        x.release()
    torch.cuda.synchronize()
