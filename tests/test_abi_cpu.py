"""The C-ABI boundary without a GPU: libforge_b200.so loads, exports every
function include/*.h declares, keeps the v1 structs byte-compatible with the
reference header (self/forge/forge_tier_v1.h:74-97) and the bf16 descriptor
layout (self/cuda/runtime_bf16_emit.hexa:164-170), answers the dispatch
argument checks with the reference's return codes before touching the GPU,
and rounds host bf16 arrays exactly like the oracle. No compute call is made:
compute needs a B200 and fails loudly without one."""
import ctypes as C
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")


def header_functions():
    names = set()
    for fn in sorted(os.listdir(INCLUDE)):
        if not fn.endswith(".h"):
            continue
        txt = open(os.path.join(INCLUDE, fn)).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        txt = re.sub(r"//[^\n]*", "", txt)
        txt = "\n".join(l for l in txt.splitlines() if not l.lstrip().startswith("#"))
        txt = re.sub(r"typedef\s+struct\s+\w*\s*\{.*?\}\s*\w+\s*;", "", txt, flags=re.S)
        for m in re.finditer(r"\b((?:forge|hexa)_\w+)\s*\(", txt):
            names.add(m.group(1))
    return names


def test_headers_declare_the_boundary():
    names = header_functions()
    for must in ("forge_api_version_v1", "forge_tier_dispatch_v1", "forge_register_specialized_v1",
                 "forge_tier_dispatch_v2", "hexa_farr_bf16_alloc", "hexa_farr_bf16_free", "hexa_farr_bf16_from_f64",
                 "hexa_farr_bf16_to_f64", "hexa_farr_bf16_to_device", "hexa_farr_bf16_to_host",
                 "hexa_farr_q4_alloc", "hexa_kv_alloc", "forge_b200_decode_step", "forge_flash_decode_noalloc"):
        assert must in names, must
    assert len(names) > 60


def test_library_exports_every_header_function(forge):
    L = forge.lib()
    missing = [n for n in sorted(header_functions()) if not hasattr(L, n)]
    assert not missing, missing


def test_library_hides_internal_symbols(forge):
    L = forge.lib()
    for internal in ("forge_fail", "forge_gemv_launch", "forge_b200_width", "forge_prefill_dispatch"):
        assert not hasattr(L, internal), internal


def test_versions(forge):
    L = forge.lib()
    assert L.forge_api_version_v1() == 0x00010000
    assert L.forge_api_version_v2() == 0x00020000


def test_v1_struct_layouts(forge):
    assert C.sizeof(forge.ForgeShapeInfo) == 32
    assert C.sizeof(forge.ForgeArgs) == 72
    assert forge.ForgeArgs.count.offset == 64
    assert C.sizeof(forge.HexaFarrBf16) == 32
    assert (forge.HexaFarrBf16.len.offset, forge.HexaFarrBf16.loc.offset, forge.HexaFarrBf16.owns.offset) == (16, 24, 28)


def _dispatch(forge, fam, prec, det=0, shape=(2, 2, 3, 0), ins=(), outs=(), v2=False):
    L = forge.lib()
    s = forge.ForgeShapeInfo(*shape)
    a = forge.forge_args(*ins)
    b = forge.forge_args(*outs)
    f = L.forge_tier_dispatch_v2 if v2 else L.forge_tier_dispatch_v1
    return f(fam, C.byref(s), 0, prec, det, C.byref(a), C.byref(b))


def test_v1_dispatch_return_codes(forge):
    F = forge
    # reference order (forge_tier_v1_emit.hexa:275-375): pedantic needs FP64
    assert _dispatch(F, F.FORGE_KERNEL_MATMUL, F.FORGE_PREC_PURE_BF16, det=1) == F.FORGE_PRECISION_UNSUPPORTED
    assert _dispatch(F, F.FORGE_KERNEL_MATMUL, 9) == F.FORGE_PRECISION_UNSUPPORTED
    assert _dispatch(F, 0, F.FORGE_PREC_PURE_BF16) == F.FORGE_INVALID_ARGS
    assert _dispatch(F, 99, F.FORGE_PREC_FP64) == F.FORGE_INVALID_ARGS
    # no FP64 or LayerCast path in this library: unsupported, never a CPU fallback
    for fam in range(1, 9):
        assert _dispatch(F, fam, F.FORGE_PREC_FP64, ins=(1, 2), outs=(3,)) == F.FORGE_KERNEL_UNSUPPORTED
        assert _dispatch(F, fam, F.FORGE_PREC_LAYERCAST_BF16_FP32) == F.FORGE_KERNEL_UNSUPPORTED
    # bf16 families not built: unsupported
    for fam in (F.FORGE_KERNEL_FWD_BWD_LINEAR, F.FORGE_KERNEL_ATTN_DT_FWD, F.FORGE_KERNEL_ATTN_DT_BWD):
        assert _dispatch(F, fam, F.FORGE_PREC_PURE_BF16, ins=(1, 2), outs=(3,)) == F.FORGE_KERNEL_UNSUPPORTED
    # bad slot counts, null slots and bad shapes are rejected before any device work
    assert _dispatch(F, F.FORGE_KERNEL_MATMUL, F.FORGE_PREC_PURE_BF16, ins=(0,), outs=(0,)) == F.FORGE_INVALID_ARGS
    assert _dispatch(F, F.FORGE_KERNEL_MATMUL, F.FORGE_PREC_PURE_BF16, ins=(0, 0), outs=(0,)) == F.FORGE_INVALID_ARGS
    assert _dispatch(F, F.FORGE_KERNEL_MATMUL, F.FORGE_PREC_PURE_BF16, shape=(0, 2, 3, 0), ins=(1, 1),
                     outs=(1,)) == F.FORGE_INVALID_ARGS
    assert _dispatch(F, F.FORGE_KERNEL_FFN_FUSED, F.FORGE_PREC_PURE_BF16, ins=(0, 0), outs=(0,)) == F.FORGE_INVALID_ARGS
    L = F.lib()
    assert L.forge_tier_dispatch_v1(1, None, 0, 2, 0, None, None) == F.FORGE_INVALID_ARGS


def test_v2_dispatch_return_codes(forge):
    F = forge
    assert _dispatch(F, 15, F.FORGE_PREC_PURE_BF16, v2=True) == F.FORGE_INVALID_ARGS
    assert _dispatch(F, 24, F.FORGE_PREC_PURE_BF16, v2=True) == F.FORGE_INVALID_ARGS
    assert _dispatch(F, F.FORGE_KERNEL_GEMV_W4A16_G128, F.FORGE_PREC_PURE_BF16, v2=True) == F.FORGE_PRECISION_UNSUPPORTED
    assert _dispatch(F, F.FORGE_KERNEL_GEMV_BF16, F.FORGE_PREC_W4A16_G128_BF16, v2=True) == F.FORGE_PRECISION_UNSUPPORTED
    assert _dispatch(F, F.FORGE_KERNEL_GEMV_W4A16_G128, F.FORGE_PREC_W4A16_G128_BF16, det=1,
                     v2=True) == F.FORGE_PRECISION_UNSUPPORTED
    assert _dispatch(F, F.FORGE_KERNEL_GEMV_W4A16_G128, F.FORGE_PREC_W4A16_G128_BF16, ins=(0, 0), outs=(0,),
                     v2=True) == F.FORGE_INVALID_ARGS
    assert _dispatch(F, F.FORGE_KERNEL_DECODE_STEP, F.FORGE_PREC_PURE_BF16, ins=(0, 0), outs=(0,),
                     v2=True) == F.FORGE_INVALID_ARGS
    # v1 families pass through v2 unchanged
    assert _dispatch(F, F.FORGE_KERNEL_MATMUL, F.FORGE_PREC_FP64, ins=(1, 2), outs=(3,),
                     v2=True) == F.FORGE_KERNEL_UNSUPPORTED


def test_register_specialized(forge):
    F = forge
    L = F.lib()
    s = F.ForgeShapeInfo(1, 2, 3, 0)
    fn = C.cast(L.forge_api_version_v1, C.c_void_p)
    assert L.forge_register_specialized_v1(1, C.byref(s), 0, 0, fn) == F.FORGE_OK
    assert L.forge_register_specialized_v1(1, None, 0, 0, fn) == F.FORGE_INVALID_ARGS
    assert L.forge_register_specialized_v1(1, C.byref(s), 0, 0, None) == F.FORGE_INVALID_ARGS


def test_bf16_farr_host_round_trip(forge, oracle):
    L = forge.lib()
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(1000) * 10, [0.0, -0.0, 1e-40, 65504.0, 3.3e38]])
    f = L.hexa_farr_bf16_alloc(len(x))
    assert f and f.contents.len == len(x) and f.contents.loc == 0 and f.contents.owns == 1
    hb = np.ctypeslib.as_array(C.cast(f.contents.h_buf, C.POINTER(C.c_uint16)), shape=(len(x),))
    assert np.all(hb == 0)
    assert L.hexa_farr_bf16_from_f64(x.ctypes.data, f, len(x)) == 0
    # RNE through fp32, the reference's _hx_f32_to_bf16_rne (runtime_bf16_emit.hexa:264-277)
    assert np.array_equal(hb, oracle.f32_to_bf16(x.astype(np.float32)))
    back = np.empty(len(x))
    assert L.hexa_farr_bf16_to_f64(f, back.ctypes.data, len(x)) == 0
    assert np.array_equal(back, oracle.bf16_to_f32(hb).astype(np.float64))
    assert L.hexa_farr_bf16_from_f64(x.ctypes.data, f, len(x) + 1) != 0   # n above len
    L.hexa_farr_bf16_free(f)
    L.hexa_farr_bf16_free(None)


def test_descriptor_argument_checks(forge):
    L = forge.lib()
    assert not L.hexa_farr_w_alloc(0, 15, 64)       # rows % 16
    assert not L.hexa_farr_q4_alloc(16, 128, 64)     # group 64 unsupported
    assert not L.hexa_kv_alloc(1, 1, 1, 16, 96)      # head_dim 96 unsupported
    assert not L.hexa_farr_bf16_alloc(-1)


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="checks the no-GPU failure path")
def test_compute_fails_loudly_without_gpu(forge):
    L = forge.lib()
    f = L.hexa_farr_bf16_alloc(16)
    assert L.hexa_farr_bf16_to_device(f) != 0
    assert L.forge_b200_last_error()
    L.hexa_farr_bf16_free(f)
    h = C.c_void_p()
    d = forge.ForgeModelDesc(n_layer=1, d_model=64, n_head=2, n_kv_head=2, head_dim=64, ffn=64, vocab=64,
                             rms_eps=1e-5, rope_theta=1e4, max_batch=1, max_ctx=16, tp_size=1)
    assert L.forge_b200_create(C.byref(d), 0, C.byref(h)) != 0


def test_python_binding_types_every_header_function(forge):
    """Every C entry has explicit ctypes argument types in the binding (an
    untyped call would pass 64-bit pointers as 32-bit ints)."""
    L = forge.lib()
    untyped = [n for n in sorted(header_functions()) if getattr(L, n).argtypes is None]
    assert not untyped, untyped
