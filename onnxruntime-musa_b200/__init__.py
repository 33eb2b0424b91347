"""B200 MoE / QMoE execution-provider package (host side over the C ABI).

Mirrors the reference plugin's Python surface
(``musa/ep/python/onnxruntime_musa/__init__.py:18-92``: ``get_library_path``,
``get_ep_name``, ``get_ep_names``, ``make_provider_options``) and exposes the
``com.microsoft`` ``MoE`` / ``QMoE`` kernels of ``lib/libmoe_b200.so`` as kernel
objects with the reference kernel framework's create / compute / release life cycle
(``musa/ep/src/kernels/shared_inc/kernel_base.h:33-97``).

The directory name is not a Python identifier; import it as
``onnxruntime_musa_b200`` through :func:`load_package` (done by ``tests/conftest.py``,
``bench.py`` and ``__graft_entry__.py``).  Device memory in the helpers below is
PyTorch's; the compute runs in the CUDA library only -- there is no CPU path, and a
missing library raises.
"""

from __future__ import annotations

import ctypes
import math
import os
import pathlib
from typing import Any, Mapping, Sequence

_DIR = pathlib.Path(__file__).resolve().parent
_LIB_PATH = _DIR / "lib" / "libmoe_b200.so"

EP_NAME = "B200MoEExecutionProvider"

# Status codes (OrtErrorCode values) and element types (ONNX TensorProto codes).
OK, FAIL, INVALID_ARGUMENT, NOT_IMPLEMENTED, EP_FAIL = 0, 1, 2, 9, 11
FLOAT, UINT8, INT32, FLOAT16, BFLOAT16 = 1, 2, 6, 10, 16
ACTIVATIONS = {"relu": 0, "gelu": 1, "silu": 2, "identity": 3, "swiglu": 4}


class MoeB200Error(RuntimeError):
    """A non-OK status from the library; ``code`` is the OrtErrorCode value."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{_CODE_NAMES.get(code, code)}] {message}")
        self.code = code


class InvalidArgument(MoeB200Error, ValueError):
    pass


class NotImplementedByEP(MoeB200Error, NotImplementedError):
    pass


class EPFail(MoeB200Error):
    pass


_CODE_NAMES = {FAIL: "FAIL", INVALID_ARGUMENT: "INVALID_ARGUMENT",
               NOT_IMPLEMENTED: "NOT_IMPLEMENTED", EP_FAIL: "EP_FAIL"}
_CODE_CLASS = {INVALID_ARGUMENT: InvalidArgument, NOT_IMPLEMENTED: NotImplementedByEP,
               EP_FAIL: EPFail}


# ----------------------------------------------------------------------- C structs

class Attrs(ctypes.Structure):
    _fields_ = [("activation_type", ctypes.c_int32), ("k", ctypes.c_int32),
                ("normalize_routing_weights", ctypes.c_int32),
                ("use_sparse_mixer", ctypes.c_int32), ("swiglu_fusion", ctypes.c_int32),
                ("swiglu_limit", ctypes.c_float), ("activation_alpha", ctypes.c_float),
                ("activation_beta", ctypes.c_float), ("expert_weight_bits", ctypes.c_int32),
                ("block_size", ctypes.c_int32)]


class Problem(ctypes.Structure):
    _fields_ = [("num_rows", ctypes.c_int64), ("hidden_size", ctypes.c_int64),
                ("inter_size", ctypes.c_int64), ("num_experts", ctypes.c_int64),
                ("dtype", ctypes.c_int32), ("has_fc3", ctypes.c_int32), ("attrs", Attrs)]


class Tensors(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "input", "router_probs", "fc1_weights", "fc1_scales", "fc1_bias", "fc2_weights",
        "fc2_scales", "fc2_bias", "fc3_weights", "fc3_scales", "fc3_bias", "output")]


class TensorRef(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("elem_type", ctypes.c_int32),
                ("rank", ctypes.c_int32), ("dims", ctypes.c_int64 * 4)]


class ProviderOptions(ctypes.Structure):
    _fields_ = [("device_id", ctypes.c_int32), ("has_user_compute_stream", ctypes.c_int32),
                ("user_compute_stream", ctypes.c_void_p),
                ("use_ep_level_unified_stream", ctypes.c_int32),
                ("do_copy_in_default_stream", ctypes.c_int32),
                ("enable_prepack_weight_sharing", ctypes.c_int32),
                ("ep_world_size", ctypes.c_int32), ("ep_rank", ctypes.c_int32)]


class DeviceProps(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("vendor_id", ctypes.c_uint32),
                ("device_id", ctypes.c_int32), ("sm_count", ctypes.c_int32),
                ("cc_major", ctypes.c_int32), ("cc_minor", ctypes.c_int32),
                ("total_memory", ctypes.c_uint64), ("pci_bus_id", ctypes.c_int32)]


# Every symbol the public header declares, with its ctypes signature.
_VP, _I32, _I64, _SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
_PI32 = ctypes.POINTER(ctypes.c_int32)
_PF = ctypes.POINTER(ctypes.c_float)
SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "moe_b200_abi_version": (ctypes.c_int, []),
    "moe_b200_last_error": (ctypes.c_char_p, []),
    "moe_b200_kernel_create": (ctypes.c_int, [ctypes.c_char_p, _I32,
                                              ctypes.POINTER(ctypes.c_char_p),
                                              ctypes.POINTER(ctypes.c_char_p),
                                              ctypes.POINTER(_VP)]),
    "moe_b200_kernel_compute": (ctypes.c_int, [_VP, _I32, ctypes.POINTER(TensorRef),
                                               ctypes.POINTER(TensorRef), _VP]),
    "moe_b200_kernel_release": (ctypes.c_int, [_VP]),
    "moe_b200_workspace_size": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(_SZ)]),
    "moe_b200_forward": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Tensors), _VP,
                                        _SZ, _VP]),
    "moe_b200_forward_timed": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Tensors),
                                              _VP, _SZ, _VP, _PF, _I32]),
    "moe_b200_forward_staged": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Tensors),
                                               _VP, _SZ, _VP, ctypes.POINTER(_VP), _I32]),
    "moe_b200_ep_comm_create": (ctypes.c_int, [_I32, _I32, _I64, _I32, _I64, _I64, _I32,
                                               ctypes.POINTER(_VP)]),
    "moe_b200_ep_comm_handle_size": (ctypes.c_int, [ctypes.POINTER(_SZ)]),
    "moe_b200_ep_comm_get_handle": (ctypes.c_int, [_VP, _VP]),
    "moe_b200_ep_comm_connect": (ctypes.c_int, [_VP, _VP]),
    "moe_b200_ep_comm_destroy": (ctypes.c_int, [_VP]),
    "moe_b200_ep_workspace_size": (ctypes.c_int, [_VP, ctypes.POINTER(Problem),
                                                  ctypes.POINTER(_SZ)]),
    "moe_b200_ep_forward": (ctypes.c_int, [_VP, ctypes.POINTER(Problem), ctypes.POINTER(Tensors),
                                           _VP, _SZ, _VP]),
    "moe_b200_ep_forward_staged": (ctypes.c_int, [_VP, ctypes.POINTER(Problem),
                                                  ctypes.POINTER(Tensors), _VP, _SZ, _VP,
                                                  ctypes.POINTER(_VP), _I32]),
    "moe_b200_norm_router": (ctypes.c_int, [_I32, _I64, _I64, _I64, _VP, _VP, _VP,
                                            ctypes.c_float, _VP, _VP, _VP, _VP, _VP]),
    "moe_b200_pipeline_create": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Tensors),
                                                _I32, ctypes.POINTER(_VP)]),
    "moe_b200_pipeline_submit": (ctypes.c_int, [_VP, _VP, _VP, _VP, _I64]),
    "moe_b200_pipeline_set_prepacked": (ctypes.c_int, [_VP, _VP]),
    "moe_b200_pipeline_synchronize": (ctypes.c_int, [_VP]),
    "moe_b200_pipeline_destroy": (ctypes.c_int, [_VP]),
    "moe_b200_ep_dispatch": (ctypes.c_int, [ctypes.POINTER(Problem), _VP, _VP, _VP, _VP, _VP,
                                            _VP, _VP, _SZ, _VP]),
    "moe_b200_expert_ffn": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Tensors), _VP,
                                           _VP, _SZ, _VP]),
    "moe_b200_ep_combine": (ctypes.c_int, [_I32, _I64, _I64, _I32, _VP, _VP, _VP, _VP, _VP]),
    "moe_b200_route": (ctypes.c_int, [_VP, _I32, _I64, _I64, _I32, _I32, _VP, _VP, _VP]),
    "moe_b200_route_noalloc": (ctypes.c_int, [_VP, _I32, _I64, _I64, _I32, _I32, _VP, _VP, _VP]),
    "moe_b200_permute_workspace_size": (_SZ, [_I64, _I32, _I64]),
    "moe_b200_permute": (ctypes.c_int, [_VP, _I64, _I32, _I64, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "moe_b200_prepack_create": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Tensors),
                                               _I32, _VP, ctypes.POINTER(_VP)]),
    "moe_b200_prepack_info": (ctypes.c_int, [_VP, ctypes.POINTER(_SZ), _PI32]),
    "moe_b200_prepack_release": (ctypes.c_int, [_VP]),
    "moe_b200_workspace_size_prepacked": (ctypes.c_int, [ctypes.POINTER(Problem), _VP,
                                                         ctypes.POINTER(_SZ)]),
    "moe_b200_forward_prepacked": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Tensors),
                                                  _VP, _VP, _SZ, _VP, ctypes.POINTER(_VP), _I32]),
    "moe_b200_kernel_prepack": (ctypes.c_int, [_VP, _I32, ctypes.POINTER(TensorRef), _I32, _VP,
                                               _PI32]),
    "moe_b200_device_count": (ctypes.c_int, [_PI32]),
    "moe_b200_device_props_get": (ctypes.c_int, [_I32, ctypes.POINTER(DeviceProps)]),
    "moe_b200_set_device": (ctypes.c_int, [_I32]),
    "moe_b200_provider_options_parse": (ctypes.c_int, [_I32, ctypes.POINTER(ctypes.c_char_p),
                                                       ctypes.POINTER(ctypes.c_char_p),
                                                       ctypes.POINTER(ProviderOptions)]),
    "moe_b200_alloc": (ctypes.c_int, [_SZ, ctypes.POINTER(_VP)]),
    "moe_b200_free": (ctypes.c_int, [_VP]),
    "moe_b200_alloc_pinned": (ctypes.c_int, [_SZ, ctypes.POINTER(_VP)]),
    "moe_b200_free_pinned": (ctypes.c_int, [_VP]),
    "moe_b200_stream_create": (ctypes.c_int, [ctypes.POINTER(_VP)]),
    "moe_b200_stream_destroy": (ctypes.c_int, [_VP]),
    "moe_b200_stream_synchronize": (ctypes.c_int, [_VP]),
    "moe_b200_notification_create": (ctypes.c_int, [ctypes.POINTER(_VP)]),
    "moe_b200_notification_activate": (ctypes.c_int, [_VP, _VP]),
    "moe_b200_notification_wait": (ctypes.c_int, [_VP, _VP]),
    "moe_b200_notification_synchronize": (ctypes.c_int, [_VP]),
    "moe_b200_notification_destroy": (ctypes.c_int, [_VP]),
    "moe_b200_copy": (ctypes.c_int, [_VP, _VP, _SZ, _I32, _VP]),
}

_lib: ctypes.CDLL | None = None


def get_library_path() -> str:
    """Path of the plugin's shared library (raises if it has not been built);
    ``MOE_B200_LIBRARY`` names another build of it."""
    alt = os.environ.get("MOE_B200_LIBRARY")
    if alt:
        if not pathlib.Path(alt).is_file():
            raise RuntimeError(f"MOE_B200_LIBRARY={alt} is not a file")
        return alt
    if not _LIB_PATH.is_file():
        raise RuntimeError(f"{_LIB_PATH} is missing: run __graft_entry__.build() "
                           "(the MoE path has no CPU fallback)")
    return str(_LIB_PATH)


def get_ep_name() -> str:
    return EP_NAME


def get_ep_names() -> list[str]:
    return [EP_NAME]


def lib() -> ctypes.CDLL:
    """The loaded C ABI library with typed entry points."""
    global _lib
    if _lib is None:
        L = ctypes.CDLL(get_library_path())
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        if L.moe_b200_abi_version() != 1:
            raise RuntimeError("libmoe_b200 ABI version mismatch")
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != OK:
        msg = lib().moe_b200_last_error().decode(errors="replace")
        raise _CODE_CLASS.get(status, MoeB200Error)(status, msg)


# ------------------------------------------------------------------ provider options

def _as_bool_option(value: bool) -> str:
    if not isinstance(value, bool):
        raise TypeError("provider boolean options must be bool values")
    return "1" if value else "0"


def make_provider_options(*, device_id: int = 0, user_compute_stream: Any = None,
                          use_ep_level_unified_stream: bool | None = None,
                          do_copy_in_default_stream: bool = True,
                          ep_world_size: int | None = None, ep_rank: int | None = None
                          ) -> dict[str, str]:
    """Provider options as key/value strings (the reference's option surface plus the
    expert-parallel keys ``ep_world_size`` / ``ep_rank``)."""
    if device_id < 0:
        raise ValueError("device_id must be non-negative")
    opts = {"device_id": str(device_id),
            "do_copy_in_default_stream": _as_bool_option(do_copy_in_default_stream)}
    if user_compute_stream is not None:
        addr = user_compute_stream if isinstance(user_compute_stream, int) else int(
            getattr(user_compute_stream, "value", user_compute_stream) or 0)
        if addr <= 0:
            raise ValueError("user_compute_stream must be a non-null cudaStream_t address")
        opts.update(has_user_compute_stream="1", user_compute_stream=str(addr),
                    use_ep_level_unified_stream="1")
    elif use_ep_level_unified_stream is not None:
        opts["use_ep_level_unified_stream"] = _as_bool_option(use_ep_level_unified_stream)
    if ep_world_size is not None:
        if ep_world_size < 1 or ep_rank is None or not (0 <= ep_rank < ep_world_size):
            raise ValueError("ep_world_size >= 1 and 0 <= ep_rank < ep_world_size required")
        opts.update(ep_world_size=str(ep_world_size), ep_rank=str(ep_rank))
    return opts


def parse_provider_options(options: Mapping[str, str]) -> dict[str, Any]:
    """The session's provider options as the library parses them
    (``moe_b200_provider_options_parse``): defaults filled in, validated, the user stream
    implying the unified stream.  Raises InvalidArgument on a malformed option."""
    keys = [str(k).encode() for k in options]
    vals = [str(v).encode() for v in options.values()]
    n = len(keys)
    ak = (ctypes.c_char_p * max(n, 1))(*keys)
    av = (ctypes.c_char_p * max(n, 1))(*vals)
    o = ProviderOptions()
    check(lib().moe_b200_provider_options_parse(n, ak, av, ctypes.byref(o)))
    return {name: getattr(o, name) for name, _ in ProviderOptions._fields_}


# --------------------------------------------------------------------- devices

def get_ep_devices() -> list[dict[str, Any]]:
    """Devices the EP would advertise (CUDA devices; vendor 0x10DE)."""
    n = ctypes.c_int32(0)
    check(lib().moe_b200_device_count(ctypes.byref(n)))
    out = []
    for d in range(n.value):
        p = DeviceProps()
        check(lib().moe_b200_device_props_get(d, ctypes.byref(p)))
        out.append(dict(name=p.name.decode(), vendor="NVIDIA", vendor_id=p.vendor_id,
                        device_id=p.device_id, sm_count=p.sm_count,
                        compute_capability=(p.cc_major, p.cc_minor),
                        total_memory=p.total_memory, ep_name=EP_NAME))
    return out


# ------------------------------------------------------------------- tensors

def _torch():
    import torch
    return torch


def elem_type_of(t) -> int:
    torch = _torch()
    m = {torch.float32: FLOAT, torch.float16: FLOAT16, torch.bfloat16: BFLOAT16,
         torch.uint8: UINT8, torch.int32: INT32}
    if t.dtype not in m:
        raise TypeError(f"unsupported tensor dtype {t.dtype}")
    return m[t.dtype]


def tensor_ref(t) -> TensorRef:
    r = TensorRef()
    if t is None:
        r.data = None
        return r
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("tensors passed to the EP must be contiguous CUDA tensors")
    if t.dim() > 4:
        raise ValueError("rank > 4")
    r.data = t.data_ptr()
    r.elem_type = elem_type_of(t)
    r.rank = t.dim()
    for i, d in enumerate(t.shape):
        r.dims[i] = d
    return r


def _stream_handle(stream) -> int | None:
    torch = _torch()
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


# ------------------------------------------------------------------- kernels

def _attr_str(v) -> str:
    if isinstance(v, bool):
        return "1" if v else "0"
    if isinstance(v, float):
        return "inf" if math.isinf(v) and v > 0 else repr(v)
    return str(v)


class MoE:
    """``com.microsoft::MoE`` (opset 1) kernel object.

    ``compute(inputs)`` takes the schema's inputs in order -- input, router_probs,
    fc1_experts_weights, fc1_experts_bias, fc2_experts_weights, fc2_experts_bias,
    fc3_experts_weights, fc3_experts_bias (None for absent optional inputs) -- as
    contiguous CUDA tensors and returns the output tensor.
    """

    op_type = "MoE"

    def __init__(self, **attrs):
        names = [n.encode() for n in attrs]
        values = [_attr_str(v).encode() for v in attrs.values()]
        arr_n = (ctypes.c_char_p * max(len(names), 1))(*names)
        arr_v = (ctypes.c_char_p * max(len(values), 1))(*values)
        h = ctypes.c_void_p()
        check(lib().moe_b200_kernel_create(self.op_type.encode(), len(names), arr_n, arr_v,
                                           ctypes.byref(h)))
        self._h = h
        self.attrs = dict(attrs)

    def compute(self, inputs: Sequence[Any], out=None, stream=None):
        torch = _torch()
        x = inputs[0]
        if out is None:
            out = torch.empty_like(x)
        refs = (TensorRef * len(inputs))(*[tensor_ref(t) for t in inputs])
        oref = tensor_ref(out)
        check(lib().moe_b200_kernel_compute(self._h, len(inputs), refs, ctypes.byref(oref),
                                            _stream_handle(stream)))
        return out

    __call__ = compute

    def prepack(self, inputs: Sequence[Any], share: bool = False, stream=None) -> bool:
        """Pre-pack the node's constant weights (QMoE: dequantised copies used by
        prefill-sized calls; ``share`` is the session option
        ``ep.musa.enable_prepack_weight_sharing``).  Returns ORT's ``is_packed`` (always
        False: decode-sized calls still read the packed initializers)."""
        refs = (TensorRef * len(inputs))(*[tensor_ref(t) for t in inputs])
        packed = ctypes.c_int32(0)
        check(lib().moe_b200_kernel_prepack(self._h, len(inputs), refs, int(bool(share)),
                                            _stream_handle(stream), ctypes.byref(packed)))
        return bool(packed.value)

    def release(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            check(lib().moe_b200_kernel_release(self._h))
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class QMoE(MoE):
    """``com.microsoft::QMoE`` kernel object.  Inputs: input, router_probs,
    fc1_experts_weights, fc1_scales, fc1_experts_bias, fc2_experts_weights, fc2_scales,
    fc2_experts_bias, fc3_experts_weights, fc3_scales, fc3_experts_bias."""

    op_type = "QMoE"


# ------------------------------------------------------------ explicit workspace

def make_problem(num_rows, hidden_size, inter_size, num_experts, dtype, has_fc3=False,
                 activation_type="relu", k=1, normalize_routing_weights=0,
                 use_sparse_mixer=0, swiglu_fusion=0, swiglu_limit=math.inf,
                 activation_alpha=1.0, activation_beta=0.0, expert_weight_bits=0,
                 block_size=0) -> Problem:
    a = Attrs(ACTIVATIONS[activation_type] if isinstance(activation_type, str)
              else activation_type, k, normalize_routing_weights, use_sparse_mixer,
              swiglu_fusion, swiglu_limit, activation_alpha, activation_beta,
              expert_weight_bits, block_size)
    return Problem(num_rows, hidden_size, inter_size, num_experts, dtype, int(has_fc3), a)


def workspace_size(problem: Problem, prepacked: "Prepacked | None" = None) -> int:
    n = ctypes.c_size_t(0)
    if prepacked is None:
        check(lib().moe_b200_workspace_size(ctypes.byref(problem), ctypes.byref(n)))
    else:
        check(lib().moe_b200_workspace_size_prepacked(ctypes.byref(problem), prepacked.handle,
                                                      ctypes.byref(n)))
    return n.value


def forward(problem: Problem, tensors: Mapping[str, Any], workspace, stream=None,
            prepacked: "Prepacked | None" = None, events=None) -> None:
    """One layer call with a caller-owned workspace (a CUDA uint8 tensor); with
    ``prepacked``, prefill-sized QMoE calls run on the prepacked weights; ``events``
    (8 CUDA events) records the stage boundaries as :func:`forward_staged` does."""
    t = _tensors_struct(tensors)
    if prepacked is None and events is None:
        check(lib().moe_b200_forward(ctypes.byref(problem), ctypes.byref(t),
                                     workspace.data_ptr(), workspace.numel(),
                                     _stream_handle(stream)))
        return
    ev = None
    if events is not None:
        ev = (ctypes.c_void_p * len(events))(*[None if e is None else e.cuda_event
                                               for e in events])
    check(lib().moe_b200_forward_prepacked(
        ctypes.byref(problem), ctypes.byref(t),
        None if prepacked is None else prepacked.handle, workspace.data_ptr(),
        workspace.numel(), _stream_handle(stream), ev, 0 if events is None else len(events)))


class Prepacked:
    """Dequantised copies of a QMoE node's expert weights (``moe_b200_prepack_create``).
    ``weights`` maps fc1/fc2/fc3 ``*_weights`` and ``*_scales`` to CUDA tensors;
    ``share=True`` reuses an existing prepack of identical content."""

    def __init__(self, problem: Problem, weights: Mapping[str, Any], share: bool = False,
                 stream=None):
        t = _tensors_struct(weights)
        h = ctypes.c_void_p()
        check(lib().moe_b200_prepack_create(ctypes.byref(problem), ctypes.byref(t),
                                            int(bool(share)), _stream_handle(stream),
                                            ctypes.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    def info(self) -> tuple[int, int]:
        """(device bytes, reference count)."""
        n, r = ctypes.c_size_t(0), ctypes.c_int32(0)
        check(lib().moe_b200_prepack_info(self._h, ctypes.byref(n), ctypes.byref(r)))
        return n.value, r.value

    def release(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            check(lib().moe_b200_prepack_release(self._h))
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.release()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


def _tensors_struct(tensors: Mapping[str, Any]) -> Tensors:
    t = Tensors()
    for name, _ in Tensors._fields_:
        v = tensors.get(name)
        setattr(t, name, None if v is None else (v if isinstance(v, int) else v.data_ptr()))
    return t


def ep_dispatch(problem: Problem, router_probs, x, stream=None):
    """Expert-parallel step 1: route all rows over all experts and gather the routed rows
    in expert order.  Returns (send_rows [T*k, H], expert_offsets [E+1], permuted_pos
    [T, k], route_weight [T, k])."""
    torch = _torch()
    T, H = x.shape
    k, E = problem.attrs.k, problem.num_experts
    dev = x.device
    send = torch.empty((T * k, H), dtype=x.dtype, device=dev)
    offs = torch.empty(E + 1, dtype=torch.int32, device=dev)
    pos = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), dtype=torch.float32, device=dev)
    ws = torch.empty(workspace_size(problem), dtype=torch.uint8, device=dev)
    check(lib().moe_b200_ep_dispatch(ctypes.byref(problem), router_probs.data_ptr(), x.data_ptr(),
                                     send.data_ptr(), offs.data_ptr(), pos.data_ptr(),
                                     w.data_ptr(), ws.data_ptr(), ws.numel(),
                                     _stream_handle(stream)))
    return send, offs, pos, w


def expert_ffn(problem: Problem, tensors: Mapping[str, Any], row_expert, stream=None) -> None:
    """Expert-parallel step 2: the expert FFN of rows whose (local) expert is given
    (``problem`` with k=1 and the local experts; ``tensors['output']`` receives one
    row per input row)."""
    torch = _torch()
    dev = tensors["input"].device
    ws = torch.empty(workspace_size(problem), dtype=torch.uint8, device=dev)
    t = _tensors_struct(tensors)
    check(lib().moe_b200_expert_ffn(ctypes.byref(problem), ctypes.byref(t),
                                    row_expert.data_ptr() if row_expert.numel() else None,
                                    ws.data_ptr(), ws.numel(), _stream_handle(stream)))


def ep_combine(expert_rows, permuted_pos, route_weight, out, stream=None):
    """Expert-parallel step 3: out[t] = sum_j w[t,j] * expert_rows[permuted_pos[t,j]]."""
    T, k = permuted_pos.shape
    check(lib().moe_b200_ep_combine(elem_type_of(out), T, out.shape[-1], k,
                                    expert_rows.data_ptr() if expert_rows.numel() else None,
                                    permuted_pos.data_ptr() if T else None,
                                    route_weight.data_ptr() if T else None,
                                    out.data_ptr() if T else None, _stream_handle(stream)))
    return out


STAGES = ("route", "plan", "gather", "dequant", "fc1", "fc2", "combine")


def forward_timed(problem: Problem, tensors: Mapping[str, Any], workspace, stream=None
                  ) -> dict[str, float]:
    """``forward`` plus the CUDA-event time (ms) of each stage on ``stream``."""
    t = Tensors()
    for name, _ in Tensors._fields_:
        v = tensors.get(name)
        setattr(t, name, None if v is None else (v if isinstance(v, int) else v.data_ptr()))
    ms = (ctypes.c_float * len(STAGES))()
    check(lib().moe_b200_forward_timed(ctypes.byref(problem), ctypes.byref(t),
                                       workspace.data_ptr(), workspace.numel(),
                                       _stream_handle(stream), ms, len(STAGES)))
    return dict(zip(STAGES, list(ms)))


def forward_staged(problem: Problem, tensors: Mapping[str, Any], workspace, events,
                   stream=None) -> None:
    """``forward`` that records ``events`` (len(STAGES) + 1 ``torch.cuda.Event`` objects
    with timing, each recorded at least once before, or None to skip a boundary) at the
    stage boundaries, without synchronising; ``events[i].elapsed_time(events[i + 1])`` is
    stage i."""
    t = Tensors()
    for name, _ in Tensors._fields_:
        v = tensors.get(name)
        setattr(t, name, None if v is None else (v if isinstance(v, int) else v.data_ptr()))
    handles = (_VP * len(events))(*[None if ev is None else ev.cuda_event for ev in events])
    check(lib().moe_b200_forward_staged(ctypes.byref(problem), ctypes.byref(t),
                                        workspace.data_ptr(), workspace.numel(),
                                        _stream_handle(stream), handles, len(events)))


# Phases of one device-side expert-parallel call (moe_b200_ep_forward_staged).
EP_PHASES = ("route_plan", "counts", "send_rows", "wait_rows", "fc1", "fc2_return",
             "wait_return", "combine")


class EpComm:
    """This rank's region of the device-side expert-parallel exchange
    (``moe_b200_ep_comm_*``).  ``handle()`` is exported to the other ranks, whose handles
    (rank order) are passed to ``connect``."""

    def __init__(self, rank: int, world: int, max_rows: int, k_max: int, hidden_size: int,
                 num_experts: int, dtype: int):
        h = _VP()
        check(lib().moe_b200_ep_comm_create(rank, world, max_rows, k_max, hidden_size,
                                            num_experts, dtype, ctypes.byref(h)))
        self._h = h
        self.max_rows, self.k_max = max_rows, k_max

    def handle(self) -> bytes:
        n = _SZ()
        check(lib().moe_b200_ep_comm_handle_size(ctypes.byref(n)))
        buf = ctypes.create_string_buffer(n.value)
        check(lib().moe_b200_ep_comm_get_handle(self._h, buf))
        return buf.raw

    def connect(self, handles: Sequence[bytes]) -> None:
        blob = b"".join(handles)
        check(lib().moe_b200_ep_comm_connect(self._h, ctypes.c_char_p(blob)))

    def workspace_size(self, problem: Problem) -> int:
        n = _SZ()
        check(lib().moe_b200_ep_workspace_size(self._h, ctypes.byref(problem), ctypes.byref(n)))
        return n.value

    def forward(self, problem: Problem, tensors: Mapping[str, Any], workspace, stream=None):
        t = Tensors()
        for name, _ in Tensors._fields_:
            v = tensors.get(name)
            setattr(t, name, None if v is None else (v if isinstance(v, int) else v.data_ptr()))
        check(lib().moe_b200_ep_forward(self._h, ctypes.byref(problem), ctypes.byref(t),
                                        workspace.data_ptr(), workspace.numel(),
                                        _stream_handle(stream)))

    def forward_staged(self, problem: Problem, tensors: Mapping[str, Any], workspace, events,
                       stream=None):
        """``forward`` recording ``events`` (EP_PHASES + 1 timing events, each recorded
        once before) at the phase boundaries, without synchronising."""
        t = Tensors()
        for name, _ in Tensors._fields_:
            v = tensors.get(name)
            setattr(t, name, None if v is None else (v if isinstance(v, int) else v.data_ptr()))
        handles = (_VP * len(events))(*[None if ev is None else ev.cuda_event for ev in events])
        check(lib().moe_b200_ep_forward_staged(self._h, ctypes.byref(problem), ctypes.byref(t),
                                               workspace.data_ptr(), workspace.numel(),
                                               _stream_handle(stream), handles, len(events)))

    def close(self) -> None:
        if self._h:
            check(lib().moe_b200_ep_comm_destroy(self._h))
            self._h = _VP()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Pipeline:
    """Calls of one layer on host tensors (``moe_b200_pipeline_*``): inputs and outputs in
    pinned host memory, weights on the device.  ``submit`` enqueues a call and returns;
    the H2D copy of the next call and the D2H copy of the previous one overlap the
    compute of this one.  Host tensors must stay alive until :meth:`synchronize`."""

    def __init__(self, problem: Problem, weights: Mapping[str, Any], depth: int = 2):
        t = Tensors()
        for name, _ in Tensors._fields_:
            v = weights.get(name)
            setattr(t, name, None if v is None else (v if isinstance(v, int) else v.data_ptr()))
        self._weights = dict(weights)  # keeps the device tensors alive
        self._max_rows = problem.num_rows
        h = _VP()
        check(lib().moe_b200_pipeline_create(ctypes.byref(problem), ctypes.byref(t), depth,
                                             ctypes.byref(h)))
        self._h = h

    def submit(self, host_input, host_router_probs, host_output) -> None:
        rows = host_input.shape[0] if host_input.dim() == 2 else host_input.numel() // \
            host_input.shape[-1]
        check(lib().moe_b200_pipeline_submit(self._h, host_input.data_ptr(),
                                             host_router_probs.data_ptr(),
                                             host_output.data_ptr(), rows))

    def set_prepacked(self, prepacked: "Prepacked | None") -> None:
        """Later calls may take the prepacked QMoE weights (the pipeline holds a reference)."""
        check(lib().moe_b200_pipeline_set_prepacked(
            self._h, None if prepacked is None else prepacked.handle))

    def synchronize(self) -> None:
        check(lib().moe_b200_pipeline_synchronize(self._h))

    def close(self) -> None:
        if self._h:
            check(lib().moe_b200_pipeline_destroy(self._h))
            self._h = _VP()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ stages

def norm_router(x, gamma, epsilon: float, router_weight, skip=None, stream=None):
    """Pre-MoE rows on the GPU: (normed [T,H], router_logits [T,E], residual [T,H] or None).
    ``residual`` = x + skip when ``skip`` is given; ``gamma`` is fp32 [H]."""
    torch = _torch()
    T, H = x.shape
    E = router_weight.shape[0]
    normed = torch.empty_like(x)
    logits = torch.empty((T, E), dtype=x.dtype, device=x.device)
    residual = torch.empty_like(x) if skip is not None else None
    ptr = lambda t: None if t is None else t.data_ptr()
    check(lib().moe_b200_norm_router(elem_type_of(x), T, H, E, x.data_ptr(), ptr(skip),
                                     gamma.data_ptr(), float(epsilon), router_weight.data_ptr(),
                                     ptr(residual), normed.data_ptr(), logits.data_ptr(),
                                     _stream_handle(stream)))
    return normed, logits, residual


def route(router_probs, k: int, normalize_routing_weights: int, stream=None):
    """Top-k routing on the GPU: (expert_idx int32 [T,k], route_weight f32 [T,k])."""
    torch = _torch()
    T, E = router_probs.shape
    idx = torch.empty((T, k), dtype=torch.int32, device=router_probs.device)
    w = torch.empty((T, k), dtype=torch.float32, device=router_probs.device)
    check(lib().moe_b200_route(router_probs.data_ptr(), elem_type_of(router_probs), T, E, k,
                               int(normalize_routing_weights), idx.data_ptr(), w.data_ptr(),
                               _stream_handle(stream)))
    return idx, w


def permute(expert_idx, num_experts: int, stream=None):
    """Dispatch plan: (offsets [E+1], permuted_pos [T,k], permuted_src [T*k])."""
    torch = _torch()
    T, k = expert_idx.shape
    dev = expert_idx.device
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    pos = torch.empty((T, k), dtype=torch.int32, device=dev)
    src = torch.empty(T * k, dtype=torch.int32, device=dev)
    nbytes = lib().moe_b200_permute_workspace_size(T, k, num_experts)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    check(lib().moe_b200_permute(expert_idx.data_ptr(), T, k, num_experts, offsets.data_ptr(),
                                 pos.data_ptr(), src.data_ptr(), ws.data_ptr(), nbytes,
                                 _stream_handle(stream)))
    return offsets, pos, src
