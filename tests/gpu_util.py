"""Helpers shared by the GPU parity tests."""

import json

import numpy as np

# Output tolerances of the parity bar: fp32 rtol 1e-4 (atol chosen here: 1e-6);
# fp16 / bf16 rtol 2e-2, atol 2e-3.
TOL = {"float32": dict(rtol=1e-4, atol=1e-6), "float16": dict(rtol=2e-2, atol=2e-3),
       "bfloat16": dict(rtol=2e-2, atol=2e-3)}


def torch_dtype(name):
    import torch
    return {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[name]


def to_dev(a, dev, dtype=None):
    """numpy -> CUDA tensor (optionally cast); None stays None."""
    import torch
    if a is None:
        return None
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t.to(dtype) if dtype is not None else t


def as_np(t):
    """CUDA tensor -> float64 numpy of the values the device holds (bf16 exact)."""
    return None if t is None else t.detach().float().cpu().numpy().astype(np.float64)


def moe_inputs_on(dev, inp, dtype_name):
    """Casts an oracle input dict to device tensors of `dtype_name`; returns (device
    tensors, the exact values they hold as float64 numpy for the oracle)."""
    dt = torch_dtype(dtype_name)
    keys = ["x", "router_probs", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "fc3_w", "fc3_b"]
    d = {k: to_dev(inp[k], dev, dt) for k in keys}
    h = {k: as_np(v) for k, v in d.items()}
    return d, h


def moe_input_list(d):
    return [d["x"], d["router_probs"], d["fc1_w"], d["fc1_b"], d["fc2_w"], d["fc2_b"],
            d["fc3_w"], d["fc3_b"]]


def load_golden(path):
    d = np.load(path, allow_pickle=False)
    meta = json.loads(str(d["meta"]))
    return d, meta
