"""Generates the small golden fixtures under tests/golden/ from the CPU oracle.

There are no upstream golden vectors for this path (the reference has no MoE code and
the ONNX Runtime CPU kernels that define it cannot be run here), so these fixtures
freeze the oracle's answers on seeded inputs: the CPU tests check the oracle still
reproduces them and the GPU tests compare the CUDA path with them.

    python tests/golden/make_golden.py
"""

import json
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from oracle import moe_oracle as orc  # noqa: E402


def save(name, arrays, meta):
    arrays = {k: v for k, v in arrays.items() if v is not None}
    np.savez_compressed(HERE / f"{name}.npz", meta=np.array(json.dumps(meta)), **arrays)


def moe_case(name, seed, T, H, I, E, k, act, gated, dtype, bias, normalize, ties=False,
             logit_scale=1.0, **extra):
    inp = orc.make_moe_inputs(T=T, H=H, I=I, E=E, k=k, act=act, gated=gated, dtype=dtype,
                              bias=bias, normalize=normalize, seed=seed)
    if logit_scale != 1.0:  # close logits: the sparse mixer's 2% band keeps several experts
        inp["router_probs"] = (inp["router_probs"].astype(np.float32) * logit_scale).astype(
            inp["router_probs"].dtype)
    if ties:  # quantise logits so that equal values (ties) are common
        inp["router_probs"] = (np.round(inp["router_probs"].astype(np.float32) * 2) / 2).astype(
            inp["router_probs"].dtype)
    attrs = dict(inp["attrs"], **extra)
    out = orc.moe(inp["x"], inp["router_probs"], inp["fc1_w"], inp["fc1_b"], inp["fc2_w"],
                  inp["fc2_b"], inp["fc3_w"], inp["fc3_b"], **attrs)
    idx, w = orc.route(inp["router_probs"], k, normalize, attrs.get("use_sparse_mixer", 0))
    save(name, dict(x=inp["x"], router_probs=inp["router_probs"], fc1_w=inp["fc1_w"],
                    fc1_b=inp["fc1_b"], fc2_w=inp["fc2_w"], fc2_b=inp["fc2_b"],
                    fc3_w=inp["fc3_w"], fc3_b=inp["fc3_b"], output=out, expert_idx=idx,
                    route_w=w), dict(op="MoE", dtype=dtype, attrs=attrs))


def qmoe_case(name, seed, T, H, I, E, k, bits, block, mu, sigma):
    q = orc.make_qmoe_inputs(T=T, H=H, I=I, E=E, k=k, bits=bits, block_size=block,
                             scale_mu=mu, scale_sigma=sigma, seed=seed)
    out = orc.qmoe(q["x"], q["router_probs"], q["fc1_q"], q["fc1_scales"], None, q["fc2_q"],
                   q["fc2_scales"], None, q["fc3_q"], q["fc3_scales"], None, **q["attrs"])
    idx, w = orc.route(q["router_probs"], k, 1)
    save(name, dict(x=q["x"], router_probs=q["router_probs"], fc1_q=q["fc1_q"],
                    fc1_scales=q["fc1_scales"], fc2_q=q["fc2_q"], fc2_scales=q["fc2_scales"],
                    fc3_q=q["fc3_q"], fc3_scales=q["fc3_scales"], output=out, expert_idx=idx,
                    route_w=w), dict(op="QMoE", dtype="float16", attrs=q["attrs"]))


if __name__ == "__main__":
    moe_case("moe_fp32_silu_bias", 11, T=24, H=64, I=96, E=8, k=2, act="silu", gated=False,
             dtype="float32", bias=True, normalize=1)
    moe_case("moe_fp16_swiglu_fc3", 12, T=40, H=128, I=64, E=8, k=2, act="silu", gated=True,
             dtype="float16", bias=False, normalize=1)
    moe_case("moe_fp16_ties_k4", 13, T=33, H=64, I=64, E=16, k=4, act="gelu", gated=False,
             dtype="float16", bias=True, normalize=0, ties=True)
    moe_case("moe_fp32_relu_k1", 14, T=17, H=32, I=48, E=4, k=1, act="relu", gated=False,
             dtype="float32", bias=True, normalize=0)
    moe_case("moe_fp16_sparse_mixer", 17, T=48, H=64, I=64, E=8, k=2, act="silu", gated=True,
             dtype="float16", bias=True, normalize=1, logit_scale=0.02, use_sparse_mixer=1)
    qmoe_case("qmoe_int4_block32", 15, T=12, H=128, I=64, E=4, k=2, bits=4, block=32,
              mu=-5.0, sigma=0.3)
    qmoe_case("qmoe_int8_rowscale", 16, T=10, H=64, I=128, E=4, k=2, bits=8, block=0,
              mu=-6.0, sigma=0.25)
    # Decode-sized QMoE (T*k <= 512, H and I multiples of 128): the weight-streaming
    # kernels, int4 with 128-wide blocks (biased codes) and int8 with per-row scales.
    qmoe_case("qmoe_int4_block128_decode", 18, T=3, H=256, I=128, E=8, k=2, bits=4, block=128,
              mu=-5.0, sigma=0.3)
    qmoe_case("qmoe_int8_rowscale_decode", 19, T=5, H=128, I=256, E=4, k=2, bits=8, block=0,
              mu=-6.0, sigma=0.25)
    print("fixtures:", sorted(p.name for p in HERE.glob("*.npz")))
