"""Failure handling on the GPU without a fault: the tensor-core kernels' bounded waits.

With the test hook MOE_B200_TEST_STALL=1 the GEMM producers issue no loads, so the MMA
and epilogue warps wait on barriers that never complete.  Every wait is bounded (2 s of
%globaltimer): the kernel records an error code, frees its tensor memory and returns, the
call reports EP_FAIL, and the context stays usable for the next call.
"""

import os
import time

import numpy as np
import pytest

from gpu_util import TOL, as_np, moe_input_list, moe_inputs_on

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["1", "2"], ids=["single_cta", "cta_pair"])
def test_bounded_wait_expires_cleanly(pkg, orc, dev, mode):
    import torch
    inp = orc.make_moe_inputs(T=300, H=256, I=256, E=4, k=2, act="silu", gated=True,
                              dtype="float32", seed=91)
    d, h = moe_inputs_on(dev, inp, "float16")
    op = pkg.MoE(**inp["attrs"])
    os.environ.update(MOE_B200_TEST_STALL="1", MOE_B200_TRACE_SYNC="1", MOE_B200_TC_MODE=mode)
    try:
        t0 = time.time()
        with pytest.raises(pkg.EPFail, match="device error code"):
            op(moe_input_list(d))
        assert time.time() - t0 < 60
    finally:
        for v in ("MOE_B200_TEST_STALL", "MOE_B200_TRACE_SYNC", "MOE_B200_TC_MODE"):
            os.environ.pop(v, None)
    out = op(moe_input_list(d))  # the context is still usable
    torch.cuda.synchronize()
    op.release()
    ref = orc.moe(h["x"], h["router_probs"], h["fc1_w"], h["fc1_b"], h["fc2_w"], h["fc2_b"],
                  h["fc3_w"], h["fc3_b"], **inp["attrs"])
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])


def test_ep_exchange_wait_expires_cleanly(pkg, orc, dev):
    """Device-side expert-parallel exchange: with the test hook the rows / return flags are
    never raised (a peer that does not take part looks the same to the waiter).  The
    waits give up after 2 s each, the call reports device error 6 (peer timeout), and the
    next call on the same communicator is correct."""
    import torch
    from onnxruntime_musa_b200 import ep
    inp = orc.make_moe_inputs(T=200, H=256, I=256, E=4, k=2, act="silu", gated=True,
                              dtype="float32", seed=92)
    d, h = moe_inputs_on(dev, inp, "float16")
    weights = dict(fc1_weights=d["fc1_w"], fc2_weights=d["fc2_w"], fc3_weights=d["fc3_w"])
    layer = ep.ExpertParallelMoE(pkg, num_experts=4, hidden_size=256, inter_size=256,
                                 dtype=pkg.FLOAT16, has_fc3=True, local_weights=weights,
                                 transport="p2p", **inp["attrs"])
    layer.forward(d["x"], d["router_probs"])  # connect
    os.environ.update(MOE_B200_TEST_STALL="1", MOE_B200_TRACE_SYNC="1")
    try:
        t0 = time.time()
        with pytest.raises(pkg.EPFail, match="device error code 6"):
            layer.forward(d["x"], d["router_probs"])
        assert time.time() - t0 < 60
    finally:
        for v in ("MOE_B200_TEST_STALL", "MOE_B200_TRACE_SYNC"):
            os.environ.pop(v, None)
    out = layer.forward(d["x"], d["router_probs"])
    torch.cuda.synchronize()
    layer.close()
    ref = orc.moe(h["x"], h["router_probs"], h["fc1_w"], None, h["fc2_w"], None, h["fc3_w"],
                  None, **inp["attrs"])
    np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])
