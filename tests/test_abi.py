"""CPU tests of the C ABI boundary: the library loads, exports exactly the symbols the
public header declares, and its host-side logic (attribute parsing, validation,
workspace planning, provider options) behaves like the reference plugin's."""

import math
import pathlib
import re
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "moe_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(moe_b200_\w+)\(", text, re.M))


def test_header_symbols_exported(pkg):
    L = pkg.lib()
    decl = declared_symbols()
    assert len(decl) >= 25
    for name in decl:
        assert hasattr(L, name), name
    assert decl == set(pkg.SIGNATURES), "ctypes signatures out of sync with the header"
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.get_library_path()],
                         capture_output=True, text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert exported == decl, f"unexpected exports: {exported ^ decl}"


def test_abi_version(pkg):
    assert pkg.lib().moe_b200_abi_version() == 1


def test_kernel_create_attributes(pkg):
    op = pkg.MoE(activation_type="silu", k=2, normalize_routing_weights=1)
    op.release()
    op = pkg.QMoE(activation_type="swiglu", k=2, expert_weight_bits=8, block_size=0,
                  swiglu_fusion=1, swiglu_limit=7.0, activation_alpha=1.702, activation_beta=1.0)
    op.release()
    with pytest.raises(pkg.InvalidArgument, match="activation_type"):
        pkg.MoE(activation_type="tanh")
    with pytest.raises(pkg.InvalidArgument, match="unknown attribute"):
        pkg.MoE(activation_type="relu", foo=1)
    with pytest.raises(pkg.InvalidArgument, match="k=0"):
        pkg.MoE(k=0)
    with pytest.raises(pkg.InvalidArgument, match="not an integer"):
        pkg.MoE(k="two")
    with pytest.raises(pkg.InvalidArgument, match="expert_weight_bits"):
        pkg.QMoE(expert_weight_bits=3)
    with pytest.raises(pkg.InvalidArgument, match="QMoE attribute"):
        pkg.MoE(expert_weight_bits=4)


def test_workspace_planning(pkg):
    p = pkg.make_problem(4096, 4096, 14336, 8, pkg.FLOAT16, has_fc3=True,
                         activation_type="silu", k=2, normalize_routing_weights=1)
    ws = pkg.workspace_size(p)
    R = 4096 * 2
    # gathered input + activation dominate: R*H*2 + R*I*2
    assert R * 4096 * 2 + R * 14336 * 2 <= ws < R * 4096 * 2 + R * 14336 * 2 + (1 << 22)
    q = pkg.make_problem(64, 4096, 14336, 8, pkg.FLOAT16, has_fc3=True, activation_type="silu",
                         k=2, expert_weight_bits=4, block_size=128)
    assert pkg.workspace_size(q) > 0


@pytest.mark.parametrize("kw,exc,msg", [
    (dict(k=9), "InvalidArgument", "k=9"),
    (dict(use_sparse_mixer=1, k=3), "InvalidArgument", "must be 2"),
    (dict(use_sparse_mixer=2), "InvalidArgument", "use_sparse_mixer=2"),
    (dict(activation_type="swiglu"), "InvalidArgument", "needs fc3"),
    (dict(activation_type="swiglu", swiglu_fusion=3), "InvalidArgument", "swiglu_fusion"),
    (dict(expert_weight_bits=4, block_size=24), "InvalidArgument", "block_size"),
])
def test_problem_validation(pkg, kw, exc, msg):
    base = dict(k=2, activation_type="silu")
    base.update(kw)
    p = pkg.make_problem(16, 64, 64, 8, pkg.FLOAT16, **base)
    with pytest.raises(getattr(pkg, exc), match=msg):
        pkg.workspace_size(p)


def test_sparse_mixer_problem_accepted(pkg):
    p = pkg.make_problem(16, 64, 64, 8, pkg.FLOAT16, k=2, activation_type="silu",
                         use_sparse_mixer=1)
    assert pkg.workspace_size(p) > 0


def test_no_device_is_zero_devices(pkg):
    import torch
    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    assert pkg.get_ep_devices() == []


def test_provider_options(pkg):
    assert pkg.make_provider_options() == {"device_id": "0", "do_copy_in_default_stream": "1"}
    o = pkg.make_provider_options(device_id=3, user_compute_stream=12345)
    assert o["has_user_compute_stream"] == "1" and o["user_compute_stream"] == "12345"
    assert o["use_ep_level_unified_stream"] == "1"
    o = pkg.make_provider_options(use_ep_level_unified_stream=False, ep_world_size=4, ep_rank=1)
    assert o["use_ep_level_unified_stream"] == "0" and o["ep_world_size"] == "4"
    with pytest.raises(ValueError):
        pkg.make_provider_options(device_id=-1)
    with pytest.raises(ValueError):
        pkg.make_provider_options(user_compute_stream=0)
    with pytest.raises(TypeError):
        pkg.make_provider_options(do_copy_in_default_stream=1)
    with pytest.raises(ValueError):
        pkg.make_provider_options(ep_world_size=2, ep_rank=2)
    assert pkg.get_ep_names() == [pkg.get_ep_name()] == ["B200MoEExecutionProvider"]


def test_new_entries_validate_before_touching_the_device(pkg):
    """Argument checks of the pipeline, device-side EP, pre-MoE rows and routing-mode
    entries run on the host before any CUDA call (so they are testable without a GPU)."""
    import ctypes
    L = pkg.lib()
    h = ctypes.c_void_p()
    # EP communicator: world beyond 8 ranks, rank outside the world, fp32, uneven experts.
    assert L.moe_b200_ep_comm_create(0, 9, 16, 2, 64, 16, pkg.FLOAT16, ctypes.byref(h)) == pkg.INVALID_ARGUMENT
    assert L.moe_b200_ep_comm_create(2, 2, 16, 2, 64, 16, pkg.FLOAT16, ctypes.byref(h)) == pkg.INVALID_ARGUMENT
    assert L.moe_b200_ep_comm_create(0, 2, 16, 2, 64, 16, pkg.FLOAT, ctypes.byref(h)) == pkg.NOT_IMPLEMENTED
    assert L.moe_b200_ep_comm_create(0, 3, 16, 2, 64, 16, pkg.FLOAT16, ctypes.byref(h)) == pkg.INVALID_ARGUMENT
    assert L.moe_b200_ep_comm_create(0, 2, 16, 2, 60, 16, pkg.FLOAT16, ctypes.byref(h)) == pkg.INVALID_ARGUMENT
    # Pipeline: depth outside [1, 8], no problem.
    p = pkg.make_problem(16, 64, 64, 8, pkg.FLOAT16, k=2, activation_type="silu")
    t = pkg.Tensors()
    assert L.moe_b200_pipeline_create(ctypes.byref(p), ctypes.byref(t), 0, ctypes.byref(h)) == pkg.INVALID_ARGUMENT
    assert L.moe_b200_pipeline_create(None, ctypes.byref(t), 2, ctypes.byref(h)) == pkg.INVALID_ARGUMENT
    # Pre-MoE rows: hidden size not a multiple of 8; nothing to do for zero rows.
    assert L.moe_b200_norm_router(pkg.FLOAT16, 4, 100, 8, None, None, None, ctypes.c_float(1e-6),
                                  None, None, None, None, None) == pkg.INVALID_ARGUMENT
    assert L.moe_b200_norm_router(pkg.FLOAT16, 0, 128, 8, None, None, None, ctypes.c_float(1e-6),
                                  None, None, None, None, None) == pkg.OK
    assert L.moe_b200_norm_router(99, 4, 128, 8, None, None, None, ctypes.c_float(1e-6),
                                  None, None, None, None, None) == pkg.NOT_IMPLEMENTED
    # Routing modes: 2 (sparse mixer) needs k = 2; 3 is not a mode.
    assert L.moe_b200_route(None, pkg.FLOAT16, 4, 8, 3, 2, None, None, None) == pkg.INVALID_ARGUMENT
    assert L.moe_b200_route(None, pkg.FLOAT16, 4, 8, 2, 3, None, None, None) == pkg.INVALID_ARGUMENT
    assert L.moe_b200_route_noalloc(None, pkg.FLOAT16, 4, 8, 3, 2, None, None, None) == pkg.INVALID_ARGUMENT
    # Stage events: fewer than stages + 1.
    evs = (ctypes.c_void_p * 3)()
    assert L.moe_b200_forward_staged(ctypes.byref(p), ctypes.byref(t), None, 0, None, evs, 3) == pkg.INVALID_ARGUMENT


def test_prepack_entries_validate_before_touching_the_device(pkg):
    """QMoE weight prepack: argument checks on the host (no CUDA call)."""
    import ctypes
    L = pkg.lib()
    h = ctypes.c_void_p()
    t = pkg.Tensors()
    # MoE (bits 0) has nothing to prepack; QMoE with NULL codes or scales is refused.
    p = pkg.make_problem(0, 128, 128, 8, pkg.FLOAT16, k=2, activation_type="silu")
    assert L.moe_b200_prepack_create(ctypes.byref(p), ctypes.byref(t), 0, None,
                                     ctypes.byref(h)) == pkg.INVALID_ARGUMENT
    q = pkg.make_problem(0, 128, 128, 8, pkg.FLOAT16, has_fc3=True, k=2, activation_type="silu",
                         expert_weight_bits=4, block_size=128)
    assert L.moe_b200_prepack_create(ctypes.byref(q), ctypes.byref(t), 1, None,
                                     ctypes.byref(h)) == pkg.INVALID_ARGUMENT
    # Shape checks are the layer call's: a block size that is not a power of two.
    bad = pkg.make_problem(0, 128, 128, 8, pkg.FLOAT16, k=2, activation_type="silu",
                           expert_weight_bits=8, block_size=48)
    assert L.moe_b200_prepack_create(ctypes.byref(bad), ctypes.byref(t), 0, None,
                                     ctypes.byref(h)) == pkg.INVALID_ARGUMENT
    assert L.moe_b200_prepack_create(None, ctypes.byref(t), 0, None, ctypes.byref(h)) == pkg.INVALID_ARGUMENT
    assert L.moe_b200_prepack_info(None, None, None) == pkg.INVALID_ARGUMENT
    assert L.moe_b200_prepack_release(None) == pkg.OK
    # Without a prepack the prepacked workspace size is the plain one.
    n1, n2 = ctypes.c_size_t(0), ctypes.c_size_t(0)
    q.num_rows = 4096
    assert L.moe_b200_workspace_size(ctypes.byref(q), ctypes.byref(n1)) == pkg.OK
    assert L.moe_b200_workspace_size_prepacked(ctypes.byref(q), None, ctypes.byref(n2)) == pkg.OK
    assert n1.value == n2.value > 0
    # Stage events of the prepacked forward: fewer than stages + 1.
    evs = (ctypes.c_void_p * 3)()
    assert L.moe_b200_forward_prepacked(ctypes.byref(q), ctypes.byref(t), None, None, 0, None,
                                        evs, 3) == pkg.INVALID_ARGUMENT
    # Kernel pre-pack of an MoE node: nothing to pack, is_packed = 0.
    op = pkg.MoE(k=2, activation_type="silu")
    try:
        refs = (pkg.TensorRef * 8)()
        packed = ctypes.c_int32(7)
        assert L.moe_b200_kernel_prepack(op._h, 8, refs, 0, None, ctypes.byref(packed)) == pkg.OK
        assert packed.value == 0
    finally:
        op.release()
    op = pkg.QMoE(k=2, activation_type="silu", expert_weight_bits=4, block_size=128)
    try:
        refs = (pkg.TensorRef * 11)()
        assert L.moe_b200_kernel_prepack(op._h, 11, refs, 0, None, None) == pkg.INVALID_ARGUMENT
    finally:
        op.release()


C_CONSUMER = r"""
#include <stdio.h>
#include <string.h>
#include "moe_b200.h"

int main(void) {
  if (moe_b200_abi_version() != MOE_B200_ABI_VERSION) return 10;
  moe_b200_problem p;
  memset(&p, 0, sizeof(p));
  p.num_rows = 16; p.hidden_size = 64; p.inter_size = 64; p.num_experts = 8;
  p.dtype = MOE_B200_FLOAT16; p.attrs.k = 2; p.attrs.activation_type = MOE_B200_ACT_SILU;
  p.attrs.swiglu_limit = 1e30f; p.attrs.activation_alpha = 1.0f;
  size_t ws = 0;
  if (moe_b200_workspace_size(&p, &ws) != MOE_B200_OK || ws == 0) return 11;
  p.attrs.k = 9;  /* more experts per token than experts */
  if (moe_b200_workspace_size(&p, &ws) != MOE_B200_INVALID_ARGUMENT) return 12;
  if (strlen(moe_b200_last_error()) == 0) return 13;
  moe_b200_prepacked* pk = NULL;
  moe_b200_tensors t;
  memset(&t, 0, sizeof(t));
  p.attrs.k = 2;
  if (moe_b200_prepack_create(&p, &t, 0, NULL, &pk) != MOE_B200_INVALID_ARGUMENT) return 14;
  printf("ok %zu\n", ws);
  return 0;
}
"""


def test_header_is_plain_c_and_links(pkg, tmp_path):
    """A C99 program includes the header, links the library and calls host-only entries
    (the binding a cgo / FFI consumer would make)."""
    import shutil
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "consumer.c"
    src.write_text(C_CONSUMER)
    lib = pathlib.Path(pkg.get_library_path())
    exe = tmp_path / "consumer"
    inc = pathlib.Path(__file__).resolve().parents[1] / "include"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-pedantic", f"-I{inc}", str(src),
                    "-o", str(exe), str(lib), f"-Wl,-rpath,{lib.parent}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert r.stdout.startswith("ok ")


def _ref(pkg, dims, et, addr=0x10000):
    r = pkg.TensorRef()
    r.data = addr if dims is not None else None
    r.elem_type = et
    if dims is not None:
        r.rank = len(dims)
        for i, d in enumerate(dims):
            r.dims[i] = d
    return r


def _compute(pkg, op, specs, out_dims, out_et):
    """kernel_compute with placeholder device pointers: only the host-side checks run."""
    import ctypes
    refs = (pkg.TensorRef * len(specs))(*[_ref(pkg, d, e) for d, e in specs])
    o = _ref(pkg, out_dims, out_et)
    return pkg.lib().moe_b200_kernel_compute(op._h, len(specs), refs, ctypes.byref(o), None)


def test_kernel_compute_rejects_bad_inputs_on_the_host(pkg):
    """Shape, type and arity checks of the kernel object, in the order the schema gives its
    inputs, return before any CUDA call."""
    F16, U8, I32 = pkg.FLOAT16, pkg.UINT8, pkg.INT32
    T, H, I, E = 16, 64, 32, 8
    moe = pkg.MoE(k=2, activation_type="silu")
    try:
        good = [((T, H), F16), ((T, E), F16), ((E, I, H), F16), (None, F16), ((E, H, I), F16),
                (None, F16), ((E, I, H), F16), (None, F16)]

        def bad(i, spec, out=(T, H), out_et=F16, n=None):
            specs = list(good)
            if i is not None:
                specs[i] = spec
            return _compute(pkg, moe, specs[:n] if n else specs, out, out_et)

        IA, NI = pkg.INVALID_ARGUMENT, pkg.NOT_IMPLEMENTED
        assert bad(None, None, n=4) == IA                       # fewer than 5 inputs
        assert bad(0, ((T, H), I32)) == NI                      # input element type
        assert bad(0, ((H,), F16)) == IA                        # input rank
        assert bad(1, ((T + 1, E), F16)) == IA                  # router rows
        assert bad(1, ((T, E), pkg.BFLOAT16)) == IA             # router type
        assert bad(2, ((E, I, H + 8), F16)) == IA               # fc1 K
        assert bad(2, ((E + 1, I, H), F16)) == IA               # fc1 experts
        assert bad(4, ((E, H + 8, I), F16)) == IA               # fc2 rows
        assert bad(6, ((E, I + 8, H), F16)) == IA               # fc3 rows
        assert bad(3, ((E, I + 1), F16)) == IA                  # fc1 bias
        assert bad(5, ((E, H), pkg.FLOAT)) == IA                # fc2 bias type
        assert bad(None, None, out=(T, H + 8)) == IA            # output shape
        assert bad(None, None, out_et=pkg.FLOAT) == IA          # output type
        assert "output" in pkg.lib().moe_b200_last_error().decode()
    finally:
        moe.release()

    q = pkg.QMoE(k=2, activation_type="silu", expert_weight_bits=4, block_size=32)
    try:
        goodq = [((T, H), F16), ((T, E), F16), ((E, I, H // 2), U8), ((E, I, H // 32), F16),
                 (None, F16), ((E, H, I // 2), U8), ((E, H, I // 32), F16), (None, F16),
                 ((E, I, H // 2), U8), ((E, I, H // 32), F16), (None, F16)]

        def badq(i, spec, n=None):
            specs = list(goodq)
            if i is not None:
                specs[i] = spec
            return _compute(pkg, q, specs[:n] if n else specs, (T, H), F16)

        IA, NI = pkg.INVALID_ARGUMENT, pkg.NOT_IMPLEMENTED
        assert badq(None, None, n=6) == IA                      # fewer than 7 inputs
        assert badq(2, ((E, I, H), U8)) == IA                   # codes not packed 2 per byte
        assert badq(2, ((E, I, H // 2), F16)) == IA             # codes not uint8
        assert badq(3, ((E, I, H // 32 + 1), F16)) == IA        # block count of fc1 scales
        assert badq(3, ((E, I), F16)) == IA                     # per-row scales, block_size 32
        assert badq(6, (None, F16)) == IA                       # fc2 scales missing
        assert badq(9, (None, F16)) == IA                       # fc3 scales missing
        specs = goodq + [((E, I), U8)]                          # fc1 zero points (asymmetric)
        assert _compute(pkg, q, specs, (T, H), F16) == NI
    finally:
        q.release()


def test_provider_options_parse(pkg):
    """The C++ option parser: defaults, the user-stream rules and the validation
    messages of the reference's ParseMusaProviderOptionsFromSession."""
    d = pkg.parse_provider_options({})
    assert d == dict(device_id=0, has_user_compute_stream=0, user_compute_stream=None,
                     use_ep_level_unified_stream=0, do_copy_in_default_stream=1,
                     enable_prepack_weight_sharing=0, ep_world_size=1, ep_rank=0)
    d = pkg.parse_provider_options(pkg.make_provider_options(device_id=3,
                                                             user_compute_stream=0x7f00))
    assert d["device_id"] == 3 and d["user_compute_stream"] == 0x7f00
    assert d["has_user_compute_stream"] == 1 and d["use_ep_level_unified_stream"] == 1
    d = pkg.parse_provider_options({"user_compute_stream": "0x10", "other.key": "x",
                                    "ep.musa.enable_prepack_weight_sharing": "1",
                                    "ep_world_size": "4", "ep_rank": "3",
                                    "do_copy_in_default_stream": "0"})
    assert d["user_compute_stream"] == 16 and d["has_user_compute_stream"] == 1
    assert d["enable_prepack_weight_sharing"] == 1 and d["do_copy_in_default_stream"] == 0
    assert (d["ep_world_size"], d["ep_rank"]) == (4, 3)
    assert pkg.parse_provider_options({"user_compute_stream": "nullptr"})[
        "user_compute_stream"] is None
    bad = [({"device_id": "-1"}, "non-negative"), ({"device_id": "1x"}, "expected integer"),
           ({"device_id": ""}, "expected integer"), ({"device_id": "99999999999"}, "integer"),
           ({"do_copy_in_default_stream": "2"}, "expected 0 or 1"),
           ({"has_user_compute_stream": "1"}, "is null"),
           ({"user_compute_stream": "abc"}, "uintptr_t"),
           ({"ep_world_size": "2", "ep_rank": "2"}, "ep_rank")]
    for opts, msg in bad:
        with pytest.raises(pkg.InvalidArgument, match=msg):
            pkg.parse_provider_options(opts)
