"""GPU tests of the CUDA runtime layer of the C ABI, the pieces the plugin's factory,
allocator, stream and data transfer retarget from the MUSA runtime
(musa/ep/src/ep_factory.cc:389-455, ep_allocator.h:86-321, ep_stream.cc:30-185,
ep_data_transfer.cc:108-161)."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H2H, H2D, D2H, D2D = 0, 1, 2, 3


def _vp():
    return ctypes.c_void_p()


def _busy(torch, stream_handle, buf, n_iter=40):
    """Queues long work on the raw stream that ends by writing `buf` (so a consumer that
    is not ordered after it would read stale values)."""
    s = torch.cuda.ExternalStream(stream_handle)
    with torch.cuda.stream(s):
        a = torch.randn(4096, 4096, device=buf.device)
        for _ in range(n_iter):
            a = torch.tanh(a @ a * 1e-3)
        buf.copy_(torch.arange(buf.numel(), device=buf.device, dtype=buf.dtype) + a[0, 0] * 0)


def test_device_discovery(pkg, dev):
    import torch
    devs = pkg.get_ep_devices()
    assert len(devs) == torch.cuda.device_count() >= 1
    d = devs[0]
    assert d["vendor_id"] == 0x10DE and d["vendor"] == "NVIDIA"
    assert d["compute_capability"] == (10, 0), d
    props = torch.cuda.get_device_properties(0)
    assert d["sm_count"] == props.multi_processor_count
    assert d["total_memory"] == props.total_memory
    assert d["name"] == props.name and d["ep_name"] == pkg.get_ep_name()
    p = pkg.DeviceProps()
    with pytest.raises(pkg.MoeB200Error):
        pkg.check(pkg.lib().moe_b200_device_props_get(len(devs) + 7, ctypes.byref(p)))
    pkg.check(pkg.lib().moe_b200_set_device(0))


def test_alloc_and_pinned_alloc(pkg, dev):
    L = pkg.lib()
    p, h = _vp(), _vp()
    pkg.check(L.moe_b200_alloc(0, ctypes.byref(p)))
    assert p.value is None  # zero bytes: NULL, like the allocator's Alloc(0)
    n = 3 << 20
    pkg.check(L.moe_b200_alloc(n, ctypes.byref(p)))
    pkg.check(L.moe_b200_alloc_pinned(n, ctypes.byref(h)))
    try:
        assert p.value % 256 == 0 and h.value
        src = np.random.default_rng(0).integers(0, 255, n, dtype=np.uint8)
        ctypes.memmove(h.value, src.ctypes.data, n)
        back = np.zeros(n, dtype=np.uint8)
        pkg.check(L.moe_b200_copy(p, h, n, H2D, None))
        pkg.check(L.moe_b200_copy(back.ctypes.data, p, n, D2H, None))
        np.testing.assert_array_equal(back, src)
    finally:
        pkg.check(L.moe_b200_free(p))
        pkg.check(L.moe_b200_free_pinned(h))
    pkg.check(L.moe_b200_free(None))
    pkg.check(L.moe_b200_free_pinned(None))
    with pytest.raises(pkg.MoeB200Error):  # far beyond the device's memory
        pkg.check(L.moe_b200_alloc(1 << 50, ctypes.byref(p)))


def test_notification_orders_two_streams(pkg, dev):
    """Producer stream A writes a buffer after long work; consumer stream B waits on the
    notification activated on A, then copies the buffer: B must see A's values."""
    import torch
    L = pkg.lib()
    sa, sb, ev = _vp(), _vp(), _vp()
    pkg.check(L.moe_b200_stream_create(ctypes.byref(sa)))
    pkg.check(L.moe_b200_stream_create(ctypes.byref(sb)))
    pkg.check(L.moe_b200_notification_create(ctypes.byref(ev)))
    try:
        buf = torch.zeros(1 << 20, device=dev)
        dst = torch.full_like(buf, -1.0)
        torch.cuda.synchronize()
        _busy(torch, sa.value, buf)
        pkg.check(L.moe_b200_notification_activate(ev, sa))
        pkg.check(L.moe_b200_notification_wait(ev, sb))
        pkg.check(L.moe_b200_copy(dst.data_ptr(), buf.data_ptr(), buf.numel() * 4, D2D, sb))
        pkg.check(L.moe_b200_stream_synchronize(sb))
        assert torch.equal(dst, torch.arange(buf.numel(), device=dev, dtype=buf.dtype))
        pkg.check(L.moe_b200_notification_synchronize(ev))
    finally:
        pkg.check(L.moe_b200_notification_destroy(ev))
        pkg.check(L.moe_b200_stream_destroy(sa))
        pkg.check(L.moe_b200_stream_destroy(sb))


def test_copy_kinds_and_d2h_ordering(pkg, dev):
    import torch
    L = pkg.lib()
    s = _vp()
    pkg.check(L.moe_b200_stream_create(ctypes.byref(s)))
    try:
        n = 1 << 20
        buf = torch.zeros(n, device=dev)
        host = np.zeros(n, dtype=np.float32)
        want = np.arange(n, dtype=np.float32)
        # D2H on the producer's stream waits for that stream's work
        _busy(torch, s.value, buf)
        pkg.check(L.moe_b200_copy(host.ctypes.data, buf.data_ptr(), n * 4, D2H, s))
        np.testing.assert_array_equal(host, want)
        # D2H without a stream waits for the whole device (the producer is a
        # non-blocking stream the legacy stream does not order against)
        buf.zero_()
        torch.cuda.synchronize()
        host[:] = 0
        _busy(torch, s.value, buf)
        pkg.check(L.moe_b200_copy(host.ctypes.data, buf.data_ptr(), n * 4, D2H, None))
        np.testing.assert_array_equal(host, want)
        # H2D then D2D on one stream, host to host, and the no-op cases
        h2 = np.random.default_rng(1).standard_normal(n).astype(np.float32)
        other = torch.empty_like(buf)
        pkg.check(L.moe_b200_copy(buf.data_ptr(), h2.ctypes.data, n * 4, H2D, s))
        pkg.check(L.moe_b200_copy(other.data_ptr(), buf.data_ptr(), n * 4, D2D, s))
        pkg.check(L.moe_b200_stream_synchronize(s))
        np.testing.assert_array_equal(other.cpu().numpy(), h2)
        h3 = np.zeros_like(h2)
        pkg.check(L.moe_b200_copy(h3.ctypes.data, h2.ctypes.data, n * 4, H2H, s))
        np.testing.assert_array_equal(h3, h2)
        pkg.check(L.moe_b200_copy(h3.ctypes.data, h3.ctypes.data, n * 4, H2H, None))
        pkg.check(L.moe_b200_copy(None, None, 0, D2H, None))
        with pytest.raises(pkg.InvalidArgument):
            pkg.check(L.moe_b200_copy(h3.ctypes.data, None, 4, D2H, None))
        with pytest.raises(pkg.InvalidArgument):
            pkg.check(L.moe_b200_copy(h3.ctypes.data, h2.ctypes.data, 4, 9, None))
    finally:
        pkg.check(L.moe_b200_stream_destroy(s))


def test_kernel_compute_on_user_stream(pkg, orc, dev):
    """A layer call on a stream from moe_b200_stream_create (the user_compute_stream
    case) is ordered after a notification from another stream that produced its input."""
    import torch
    from gpu_util import TOL, as_np, to_dev
    L = pkg.lib()
    inp = orc.make_moe_inputs(T=96, H=256, I=256, E=8, k=2, act="silu", gated=True,
                              dtype="float16", seed=3)
    sp, sc, ev = _vp(), _vp(), _vp()
    pkg.check(L.moe_b200_stream_create(ctypes.byref(sp)))
    pkg.check(L.moe_b200_stream_create(ctypes.byref(sc)))
    pkg.check(L.moe_b200_notification_create(ctypes.byref(ev)))
    op = pkg.MoE(**inp["attrs"])
    try:
        x_host = to_dev(inp["x"], torch.device("cpu")).pin_memory()
        x = torch.zeros(x_host.shape, dtype=x_host.dtype, device=dev)
        t = lambda a: None if a is None else to_dev(a, dev)
        ins = [x, t(inp["router_probs"]), t(inp["fc1_w"]), None, t(inp["fc2_w"]), None,
               t(inp["fc3_w"]), None]
        out = torch.empty_like(x)
        torch.cuda.synchronize()
        pkg.check(L.moe_b200_copy(x.data_ptr(), x_host.data_ptr(), x.numel() * 2, H2D, sp))
        pkg.check(L.moe_b200_notification_activate(ev, sp))
        pkg.check(L.moe_b200_notification_wait(ev, sc))
        op(ins, out=out, stream=sc.value)
        pkg.check(L.moe_b200_stream_synchronize(sc))
        ref = orc.moe(inp["x"], inp["router_probs"], inp["fc1_w"], None, inp["fc2_w"], None,
                      inp["fc3_w"], None, **inp["attrs"])
        np.testing.assert_allclose(as_np(out), ref, **TOL["float16"])
    finally:
        op.release()
        pkg.check(L.moe_b200_notification_destroy(ev))
        pkg.check(L.moe_b200_stream_destroy(sp))
        pkg.check(L.moe_b200_stream_destroy(sc))


_TRACE_SCRIPT = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import __graft_entry__ as ge
pkg, orc = ge.load_package(), ge.load_oracle()
inp = orc.make_moe_inputs(T=40, H=128, I=128, E=4, k=2, act="silu", gated=True,
                          dtype="float16", seed=2)
t = lambda a: None if a is None else torch.from_numpy(a).cuda()
op = pkg.MoE(**inp["attrs"])
for _ in range(2):
    op([t(inp["x"]), t(inp["router_probs"]), t(inp["fc1_w"]), None, t(inp["fc2_w"]), None,
        t(inp["fc3_w"]), None])
torch.cuda.synchronize()
op.release()
"""


def test_kernel_trace_lines(dev):
    """MOE_B200_TRACE_KERNELS prints CREATE / BEGIN / END / RELEASE lines per kernel
    object (the reference's MUSA_EP_TRACE_KERNELS), END carrying the status; with
    MOE_B200_TRACE_SYNC each compute is synchronised before END."""
    import os
    import pathlib
    import subprocess
    import sys
    root = str(pathlib.Path(__file__).resolve().parents[1])
    env = dict(os.environ, MOE_B200_TRACE_KERNELS="1", MOE_B200_TRACE_SYNC="1")
    r = subprocess.run([sys.executable, "-c", _TRACE_SCRIPT, root], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stderr.splitlines() if ln.startswith("MOE_B200_KERNEL_")]
    kinds = [ln.split()[0] for ln in lines]
    assert kinds == ["MOE_B200_KERNEL_CREATE", "MOE_B200_KERNEL_BEGIN", "MOE_B200_KERNEL_END",
                     "MOE_B200_KERNEL_BEGIN", "MOE_B200_KERNEL_END",
                     "MOE_B200_KERNEL_RELEASE"], lines
    impl = {ln.split()[2] for ln in lines}
    assert len(impl) == 1, lines
    assert all(ln.endswith("status=0") for ln in lines if "KERNEL_END" in ln), lines
    assert all(" MoE " in ln for ln in lines), lines
