"""The oracle against independent implementations of the same published algorithms:
the Mixtral and Phi-3.5-MoE sparse MoE blocks of the installed ``transformers`` (CPU,
small random configurations, eval mode).  Mixtral: softmax -> top-k -> renormalised
weights, SwiGLU experts (gate and up halves of one [E, 2I, H] weight).  Phi-3.5-MoE: the
sparse-mixer top-2 router.  These cross-check the restatement of the operator contract;
they do not replace ONNX Runtime's own kernels, whose source is not available here."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")


def _init(block, seed):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in block.parameters():
            p.copy_(torch.randn(p.shape, generator=g, dtype=p.dtype) * 0.1)
    return block.eval()


def _weights(block, I):
    gu = block.experts.gate_up_proj.detach().double().numpy()   # [E, 2I, H]
    down = block.experts.down_proj.detach().double().numpy()    # [E, H, I]
    return gu, gu[:, :I], gu[:, I:], down


@pytest.mark.parametrize("T,H,I,E,k", [(37, 64, 48, 8, 2), (50, 32, 40, 16, 4)])
def test_mixtral_block(orc, T, H, I, E, k):
    from transformers import MixtralConfig
    from transformers.models.mixtral.modeling_mixtral import MixtralSparseMoeBlock
    cfg = MixtralConfig(hidden_size=H, intermediate_size=I, num_local_experts=E,
                        num_experts_per_tok=k, hidden_act="silu", router_jitter_noise=0.0)
    blk = _init(MixtralSparseMoeBlock(cfg).double(), seed=T + E)
    x = torch.randn(1, T, H, generator=torch.Generator().manual_seed(7), dtype=torch.float64)
    with torch.no_grad():
        ref = blk(x)[0].numpy()
        logits = (x[0] @ blk.gate.weight.T).numpy()
        _, hf_w, hf_idx = blk.gate(x[0])
    gu, w1, w3, w2 = _weights(blk, I)
    idx, w = orc.route(logits, k, 1)
    np.testing.assert_array_equal(idx, hf_idx.numpy())
    np.testing.assert_allclose(w, hf_w.numpy(), rtol=1e-6, atol=1e-7)
    # fc3 as the linear half, and the same weights as one fused [E, 2I, H] (halves).
    out3 = orc.moe(x[0].numpy(), logits, w1, None, w2, None, w3, None, activation_type="silu",
                   k=k, normalize_routing_weights=1)
    outf = orc.moe(x[0].numpy(), logits, gu, None, w2, None, activation_type="swiglu", k=k,
                   normalize_routing_weights=1, swiglu_fusion=2)
    np.testing.assert_allclose(out3, ref, rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(outf, ref, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("T,E,spread", [(200, 16, 1.0), (300, 8, 0.02), (200, 32, 0.005)])
def test_phimoe_sparse_mixer(orc, T, E, spread):
    """Router logits at several spreads, down to the scale of the 2 * 0.01 mask threshold
    (many experts near the cut): the same picks, the same weights."""
    from transformers import PhimoeConfig
    from transformers.models.phimoe.modeling_phimoe import PhimoeSparseMoeBlock
    H, I = 32, 24
    cfg = PhimoeConfig(hidden_size=H, intermediate_size=I, num_local_experts=E,
                       num_experts_per_tok=2, hidden_act="silu", router_jitter_noise=0.01,
                       input_jitter_noise=0.0)
    blk = _init(PhimoeSparseMoeBlock(cfg), seed=E)
    g = torch.Generator().manual_seed(T)
    x = torch.randn(1, T, H, generator=g)
    with torch.no_grad():
        # Router logits = 1 + spread * N(0, 1): large positive values with small gaps
        # exercise the relative mask (m - s) / max(|s|, m).
        blk.router.weight.copy_(torch.randn(E, H, generator=g) * spread / H ** 0.5)
        x[..., 0] = 1.0
        blk.router.weight[:, 0] += 1.0
        logits, hf_w, hf_idx = blk.router(x[0])
        ref = blk(x)[0].double().numpy()
    lg = logits.numpy()
    assert (np.sort(lg, axis=1)[:, -1] != np.sort(lg, axis=1)[:, -2]).all()  # no exact ties
    m = lg.max(axis=1, keepdims=True)
    kept = ((m - lg) / np.maximum(np.abs(lg), m) <= np.float32(0.02)).sum(axis=1)
    assert kept.max() > 1  # rows whose first pick shares its weight
    if spread >= 0.02:
        assert kept.min() < E  # and rows where the mask drops experts
    idx, w = orc.route(lg, 2, 1, use_sparse_mixer=1)
    np.testing.assert_array_equal(idx, hf_idx.numpy())
    np.testing.assert_allclose(w, hf_w.numpy(), rtol=2e-6, atol=1e-7)
    _, w1, w3, w2 = _weights(blk, I)
    out = orc.moe(x[0].double().numpy(), lg, w1, None, w2, None, w3, None,
                  activation_type="silu", k=2, use_sparse_mixer=1)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-6)
