"""GPU test of moe_b200_route_noalloc, the router entry point that allocates nothing.

Some callers cannot allocate device memory where they route (memory planned up front,
or owned by an arena that only hands a kernel its inputs and outputs); this entry
point keeps its scratch in a static device array instead.  The test calls it through
the C ABI and checks it against moe_b200_route (the allocating entry point) on two
calls in a row, so the second call runs on the array the first one left behind.
This file is collected last on purpose.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(pkg, logits, k, normalize):
    import torch
    T, E = logits.shape
    idx = torch.full((T, k), -1, dtype=torch.int32, device=logits.device)
    w = torch.full((T, k), -1.0, dtype=torch.float32, device=logits.device)
    stream = torch.cuda.current_stream().cuda_stream
    rc = pkg.lib().moe_b200_route_noalloc(logits.data_ptr(), pkg.elem_type_of(logits), T, E,
                                          k, normalize, idx.data_ptr(), w.data_ptr(), stream)
    pkg.check(rc)
    torch.cuda.synchronize()
    return idx, w


@pytest.mark.parametrize("T,E,k,normalize,dtype", [
    (4096, 8, 2, 1, "float16"),
    (3000, 64, 8, 0, "bfloat16"),
    (65536, 256, 8, 1, "float32"),   # the largest size the static scratch holds
])
def test_noalloc_route_matches_route(pkg, dev, T, E, k, normalize, dtype):
    import torch
    dt = getattr(torch, dtype)
    for call in range(2):
        g = torch.Generator(device=dev).manual_seed(1000 * call + E)
        logits = torch.randn(T, E, device=dev, generator=g).to(dt)
        if call == 1:
            logits = (logits * 2).round() / 2  # frequent ties on the second call
        ref_idx, ref_w = pkg.route(logits, k, normalize)
        idx, w = _noalloc(pkg, logits, k, normalize)
        assert torch.equal(idx, ref_idx), f"call {call}: expert indices differ"
        np.testing.assert_allclose(w.cpu().numpy(), ref_w.cpu().numpy(), rtol=0, atol=0)


def test_noalloc_route_rejects_oversize(pkg, dev):
    import torch
    logits = torch.zeros(65537, 256, device=dev, dtype=torch.float16)
    with pytest.raises(pkg.InvalidArgument, match="static scratch"):
        _noalloc(pkg, logits, 2, 1)
