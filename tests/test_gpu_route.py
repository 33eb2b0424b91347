"""GPU parity of routing and the dispatch plan: bit-exact against the oracle."""

import numpy as np
import pytest

from gpu_util import as_np, to_dev, torch_dtype

pytestmark = pytest.mark.gpu


def _logits(T, E, seed, ties, dtype_name):
    rng = np.random.default_rng(seed)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    if ties:  # few distinct values -> frequent exact ties
        lg = np.round(lg * 2) / 2
    return lg


@pytest.mark.parametrize("dtype_name", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("E,k", [(8, 1), (8, 2), (16, 2), (64, 8), (128, 4), (256, 8), (5, 5)])
@pytest.mark.parametrize("ties", [False, True])
@pytest.mark.parametrize("normalize", [0, 1])
def test_route_bit_exact(pkg, orc, dev, dtype_name, E, k, ties, normalize):
    T = 1000
    lg = to_dev(_logits(T, E, E * 31 + k, ties, dtype_name), dev, torch_dtype(dtype_name))
    idx, w = pkg.route(lg, k, normalize)
    ridx, rw = orc.route(as_np(lg).astype(np.float32), k, normalize)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


def test_route_nan_and_inf(pkg, orc, dev):
    import torch
    lg = np.array([[np.nan, 1.0, -np.inf, 1.0], [-np.inf, -np.inf, -np.inf, 0.5],
                   [np.inf, 0.0, 1.0, 2.0]], dtype=np.float32)
    idx, _ = pkg.route(to_dev(lg, dev), 2, 1)
    ridx, _ = orc.route(lg, 2, 1)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)


@pytest.mark.parametrize("T,E,k,skew", [(1, 8, 2, False), (255, 8, 2, False),
                                         (257, 8, 2, False), (4096, 64, 8, True),
                                         (3000, 256, 8, False), (5000, 16, 1, True)])
def test_permute_bit_exact(pkg, orc, dev, T, E, k, skew):
    rng = np.random.default_rng(T + E)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    if skew:
        lg[:, : E // 4] += 4.0  # most rows to a few experts; others empty
    idx, _ = pkg.route(to_dev(lg, dev), k, 1)
    offsets, pos, src = pkg.permute(idx, E)
    ro, rp, rs = orc.permutation(idx.cpu().numpy(), E)
    np.testing.assert_array_equal(offsets.cpu().numpy(), ro)
    np.testing.assert_array_equal(pos.cpu().numpy(), rp)
    np.testing.assert_array_equal(src.cpu().numpy(), rs)


def test_permute_all_to_one_expert(pkg, orc, dev):
    import torch
    idx = torch.full((777, 1), 3, dtype=torch.int32, device=dev)
    offsets, pos, src = pkg.permute(idx, 8)
    assert offsets.cpu().tolist() == [0, 0, 0, 0, 777, 777, 777, 777, 777]
    assert src.cpu().tolist() == list(range(777))


def test_permute_rejects_out_of_range(pkg, dev):
    import torch
    idx = torch.tensor([[0, 9]], dtype=torch.int32, device=dev)
    with pytest.raises(pkg.InvalidArgument, match="out of range"):
        pkg.permute(idx, 8)


def test_route_deterministic(pkg, dev):
    import torch
    lg = torch.randn(20000, 64, device=dev, dtype=torch.float16)
    a = pkg.route(lg, 8, 1)
    b = pkg.route(lg, 8, 1)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("dtype_name", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("E", [2, 8, 64, 256])
@pytest.mark.parametrize("ties", [False, True])
def test_route_sparse_mixer(pkg, orc, dev, dtype_name, E, ties):
    """Routing mode 2 (sparse-mixer top-2): indices bit-exact, weights to fp32 rounding."""
    T = 1000
    lg = _logits(T, E, E * 7 + 3, ties, dtype_name)
    lg[::7] *= 0.01  # logits close together: many experts inside the 2% band
    d = to_dev(lg, dev, torch_dtype(dtype_name))
    idx, w = pkg.route(d, 2, 2)
    ridx, rw = orc.route(as_np(d).astype(np.float32), 2, 0, use_sparse_mixer=1)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    with pytest.raises(pkg.InvalidArgument):
        pkg.route(d, 3, 2)
