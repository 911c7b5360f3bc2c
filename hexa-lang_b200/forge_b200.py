"""ctypes binding of libforge_b200.so — the host-side mirror of forge's decode
interface for Python callers (tests, bench). The library itself is C/CUDA;
this module only marshals arguments. It refuses to run without the built
shared library: there is no Python or CPU fallback of any kernel.

Reference interface mirrored: the flame decode loop over nn_decoder_fwd +
nn_decoder_predict (stdlib/flame/decoder_lib.hexa:93-208, 485-500) becomes
ForgeModel.generate/step; forge's per-op GEMV entry
(_hx_cuda_farr_packed_gemv_offset_gpu, self/cuda/runtime_cuda_emit.hexa:1858)
becomes gemv_w4a16/gemv_bf16 on device pointers.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("FORGE_B200_LIB") or os.path.join(HERE, "libforge_b200.so")

FORGE_WEIGHT_BF16 = 0
FORGE_WEIGHT_Q4_G128 = 1
FORGE_PERM_NONE, FORGE_PERM_QKV, FORGE_PERM_GATEUP = 0, 1, 2


class ForgeModelDesc(C.Structure):
    _fields_ = [
        ("n_layer", C.c_int32), ("d_model", C.c_int32), ("n_head", C.c_int32),
        ("n_kv_head", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
        ("vocab", C.c_int32), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
        ("weight_kind", C.c_int32), ("tied_head", C.c_int32), ("max_batch", C.c_int32),
        ("max_ctx", C.c_int32), ("tp_rank", C.c_int32), ("tp_size", C.c_int32),
        ("act_mode", C.c_int32), ("reserved", C.c_int32 * 5),
    ]


class ForgeLayerWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "g1", "g2")]


class ForgeStTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int32), ("ndim", C.c_int32), ("shape", C.c_int64 * 8),
                ("offset", C.c_int64), ("nbytes", C.c_int64), ("data", C.c_void_p)]


# safetensors dtype codes (include/forge_safetensors.h) and their names
ST_DTYPES = ["BOOL", "U8", "I8", "I16", "U16", "F16", "BF16", "I32", "U32", "F32", "F64", "I64", "U64",
             "F8_E4M3", "F8_E5M2"]
FORGE_ST_NOT_FOUND = -6


class ForgePagedKvStats(C.Structure):
    _fields_ = [("num_pages", C.c_int32), ("page_tokens", C.c_int32), ("head_dim", C.c_int32),
                ("used_pages", C.c_int32), ("free_pages", C.c_int32), ("seq_count", C.c_int32),
                ("stat_alloc", C.c_int64), ("stat_release", C.c_int64), ("stat_reuse", C.c_int64)]


class ForgeClmBlock(C.Structure):
    _fields_ = [("cout", C.c_int64), ("rest", C.c_int64), ("offset", C.c_int64)]


# continuous batching (include/forge_serve.h): request phases and records
FORGE_CB_QUEUED, FORGE_CB_PREFILL, FORGE_CB_DECODE, FORGE_CB_PREEMPTED, FORGE_CB_SWAPPED, FORGE_CB_DONE = range(6)
SERVE_REQUEST_FIELDS = ("req_id", "prompt_len", "max_gen", "priority", "deadline", "phase", "tokens_generated",
                        "kv_slots_used", "enqueue_time", "start_time", "finish_time", "was_preempted",
                        "preempt_count")
SERVE_STATS_FIELDS = ("queue_size", "running_count", "swapped_count", "completed_count", "kv_used", "kv_free",
                      "step", "total_tokens", "total_preemptions")
SERVE_THROUGHPUT_FIELDS = ("tokens_per_step", "avg_latency", "avg_wait_time", "max_latency", "max_wait_time",
                           "total_tokens", "total_preemptions", "total_swaps_out", "total_swaps_in",
                           "total_requests_done")


class ForgeServeRequest(C.Structure):
    _fields_ = [(n, C.c_int64) for n in SERVE_REQUEST_FIELDS]


class ForgeServeStats(C.Structure):
    _fields_ = [(n, C.c_int64) for n in SERVE_STATS_FIELDS]


class ForgeServeThroughput(C.Structure):
    _fields_ = [(n, C.c_double) for n in SERVE_THROUGHPUT_FIELDS[:3]] + \
               [(n, C.c_int64) for n in SERVE_THROUGHPUT_FIELDS[3:]]


class ForgeShapeInfo(C.Structure):
    _fields_ = [("M", C.c_int64), ("N", C.c_int64), ("K", C.c_int64), ("batch", C.c_int64)]


class ForgeArgs(C.Structure):
    _fields_ = [("farr_ids", C.c_int64 * 8), ("count", C.c_int)]


class HexaFarrBf16(C.Structure):
    """Same layout for HexaFarrF32 / HexaFarrI32 (4-byte elements)."""
    _fields_ = [("h_buf", C.c_void_p), ("d_buf", C.c_void_p), ("len", C.c_int64), ("loc", C.c_int),
                ("owns", C.c_int)]


HexaFarrF32 = HexaFarrI32 = HexaFarrBf16


class HexaFarrW(C.Structure):
    _fields_ = [("d_tiles", C.c_void_p), ("d_scales", C.c_void_p), ("rows", C.c_int64), ("cols", C.c_int64),
                ("tile_bytes", C.c_int64), ("scale_bytes", C.c_int64), ("kind", C.c_int32), ("group", C.c_int32),
                ("packed", C.c_int32), ("owns", C.c_int32)]


class HexaKvCache(C.Structure):
    _fields_ = [("d_k", C.c_void_p), ("d_v", C.c_void_p), ("d_pos", C.c_void_p), ("n_layer", C.c_int64),
                ("batch", C.c_int64), ("n_kv_head", C.c_int64), ("max_ctx", C.c_int64), ("head_dim", C.c_int64),
                ("owns", C.c_int), ("reserved", C.c_int)]


# v1 / v2 constants (include/forge_tier_v1.h, include/forge_b200.h)
FORGE_OK, FORGE_FALLBACK_USED, FORGE_KERNEL_UNSUPPORTED = 0, 1, -1
FORGE_REGIME_UNSUPPORTED, FORGE_PRECISION_UNSUPPORTED, FORGE_INVALID_ARGS, FORGE_ABI_MISMATCH = -2, -3, -4, -5
FORGE_KERNEL_MATMUL, FORGE_KERNEL_FFN_FUSED, FORGE_KERNEL_FWD_BWD_LINEAR = 1, 2, 3
FORGE_KERNEL_ATTN_DT_FWD, FORGE_KERNEL_ATTN_DT_BWD, FORGE_KERNEL_RMSNORM_MH = 4, 5, 6
FORGE_KERNEL_SILU_GATE, FORGE_KERNEL_ROPE_MH = 7, 8
FORGE_KERNEL_GEMV_W4A16_G128, FORGE_KERNEL_GEMV_BF16, FORGE_KERNEL_QKV_ROPE_FUSED = 16, 17, 18
FORGE_KERNEL_FLASH_DECODE, FORGE_KERNEL_SWIGLU_FUSED, FORGE_KERNEL_LMHEAD_ARGMAX = 19, 20, 21
FORGE_KERNEL_FLASH_PREFILL, FORGE_KERNEL_DECODE_STEP = 22, 23
FORGE_PREC_FP64, FORGE_PREC_LAYERCAST_BF16_FP32, FORGE_PREC_PURE_BF16, FORGE_PREC_W4A16_G128_BF16 = 0, 1, 2, 3
FORGE_DET_DEFAULT, FORGE_DET_PEDANTIC = 0, 1
HEXA_FARR_W_BF16, HEXA_FARR_W_Q4_G128 = 0, 1


def forge_args(*slots) -> ForgeArgs:
    """ForgeArgs from descriptor pointers (ctypes objects or ints)."""
    a = ForgeArgs()
    for i, v in enumerate(slots):
        if v is None:
            v = 0
        elif not isinstance(v, int):
            v = C.cast(v, C.c_void_p).value or 0
        a.farr_ids[i] = v
    a.count = len(slots)
    return a


def build(force: bool = False) -> str:
    """Compiles libforge_b200.so for sm_100a with nvcc (no GPU needed)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-C", os.path.join(HERE, "csrc"), "-j8"], check=True,
                       stdout=subprocess.DEVNULL)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it (make -C hexa-lang_b200/csrc)")
        L = C.CDLL(LIB_PATH)
        vp, i64, i32 = C.c_void_p, C.c_int64, C.c_int
        sig = {
            "forge_b200_create": (i32, [C.POINTER(ForgeModelDesc), i32, C.POINTER(vp)]),
            "forge_b200_destroy": (None, [vp]),
            "forge_b200_create_tp": (i32, [C.POINTER(ForgeModelDesc), i32, vp, C.POINTER(vp)]),
            "forge_b200_tp_unique_id": (i32, [vp]),
            "forge_tp_split": (i32, [i64, i64, i32, i32, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
            "forge_b200_last_error": (C.c_char_p, []),
            "forge_b200_stream": (vp, [vp]),
            "forge_b200_load_layer": (i32, [vp, i32, C.POINTER(ForgeLayerWeights)]),
            "forge_b200_load_embedding": (i32, [vp, vp, vp, vp]),
            "forge_b200_init_synthetic": (i32, [vp, C.c_uint64, C.c_float]),
            "forge_b200_reset": (i32, [vp]),
            "forge_b200_fill_kv_synthetic": (i32, [vp, C.c_uint64, i32, C.c_float]),
            "forge_b200_set_positions": (i32, [vp, vp, i32]),
            "forge_b200_get_kv": (i32, [vp, i32, i32, vp, vp]),
            "forge_b200_decode_step": (i32, [vp, i32, vp, vp, vp]),
            "forge_b200_decode_device": (i32, [vp, i32, i32]),
            "forge_b200_generate": (i32, [vp, i32, vp, i32, i32, vp]),
            "forge_b200_sync": (i32, [vp]),
            "forge_b200_step_bytes": (i64, [vp, i32, i32]),
            "forge_b200_prefill": (i32, [vp, i32, vp, i32, i32, vp, vp]),
            "forge_b200_forward_rows": (i32, [vp, i32, vp, vp, vp, i32, vp, i32, vp, vp]),
            "forge_b200_get_kv_rows": (i32, [vp, i32, i32, vp, vp, i32]),
            "forge_b200_get_desc": (i32, [vp, C.POINTER(ForgeModelDesc)]),
            "forge_b200_init_synthetic_d": (i32, [vp, C.c_uint64, C.c_double]),
            "forge_serve_create": (i32, [vp, i32, i64, C.POINTER(vp)]),
            "forge_serve_destroy": (i32, [vp]),
            "forge_serve_set_eos": (i32, [vp, i32]),
            "forge_serve_add_request": (i32, [vp, i64, vp, i64, i64, i64, i64]),
            "forge_serve_run_step": (i32, [vp, i64]),
            "forge_serve_run_until_done": (i32, [vp, i64]),
            "forge_serve_check_deadlines": (i32, [vp, i64]),
            "forge_serve_preempt": (i32, [vp, i64]),
            "forge_serve_preempt_for_room": (i32, [vp, i64]),
            "forge_serve_swap_out": (i32, [vp, i64]),
            "forge_serve_swap_in": (i32, [vp, i64]),
            "forge_serve_peek_queue": (i32, [vp, C.POINTER(ForgeServeRequest)]),
            "forge_serve_find_request": (i32, [vp, i64, C.POINTER(ForgeServeRequest)]),
            "forge_serve_count_by_phase": (i64, [vp, i64]),
            "forge_serve_stats": (i32, [vp, C.POINTER(ForgeServeStats)]),
            "forge_serve_throughput": (i32, [vp, C.POINTER(ForgeServeThroughput)]),
            "forge_serve_output": (i32, [vp, i64, vp, i64, C.POINTER(C.c_int64)]),
            "forge_serve_engine_time": (i32, [vp, C.POINTER(C.c_double), C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
            "forge_tp_selftest_absent_peer": (i32, [i32, i32, C.c_uint64, vp, vp]),
            "forge_train_rmsnorm_rows": (i32, [vp, i64, i64, C.c_double, vp, vp]),
            "forge_train_rmsnorm_bwd_rows": (i32, [vp, vp, i64, i64, vp, vp]),
            "forge_train_adamw_step": (i32, [vp, vp, vp, vp, i64] + [C.c_double] * 5 + [i64, vp, vp]),
            "forge_train_rope": (i32, [vp, vp, vp, i64, i64, i64, i32, vp, vp]),
            "forge_train_silu": (i32, [vp, vp, i64, i32, vp, vp]),
            "forge_train_attn_fwd": (i32, [vp, vp, vp, i64, i64, i64, i64, vp, vp, vp]),
            "forge_train_attn_bwd": (i32, [vp, vp, vp, vp, vp, i64, i64, i64, i64, vp, vp, vp, vp, vp]),
            "forge_b200_launches_per_step": (i32, [vp, i32]),
            "forge_b200_step_trace": (i32, [vp, vp, i32]),
            "forge_b200_uses_fused_step": (i32, [vp, i32]),
            "forge_gemv_w4a16_g128": (i32, [vp, vp, i64, i64, vp, i32, vp, i32, vp]),
            "forge_gemv_bf16": (i32, [vp, i64, i64, vp, i32, vp, i32, vp]),
            "forge_flash_decode_workspace_bytes": (i64, [i32, i32, i32, i32, i32]),
            "forge_flash_decode": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, vp, vp]),
            "forge_flash_decode_noalloc": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, vp]),
            "forge_flash_decode_noalloc_capacity": (i64, []),
            "forge_flash_decode_noalloc_status": (i32, []),
            "forge_fill_normal_bf16": (i32, [vp, i64, C.c_uint64, C.c_uint64, C.c_float, vp]),
            "forge_fill_f32": (i32, [vp, i64, C.c_float, vp]),
            "forge_q4_quantize_bf16": (i32, [vp, i64, i64, i32, vp, vp, vp]),
            "forge_permute_rows_bf16": (i32, [vp, vp, i64, i64, i32, i64, vp]),
            "forge_bf16_pack_tiles": (i32, [vp, i64, i64, vp, vp]),
            "forge_q4_pack_tiles": (i32, [vp, vp, i64, i64, i32, vp, vp, vp]),
            "forge_q4_unpack_tiles": (i32, [vp, vp, i64, i64, i32, vp, vp, vp]),
            "forge_q4_tile_bytes": (i64, [i64, i64]),
            "forge_q4_scale_tile_bytes": (i64, [i64, i64, i32]),
            "forge_ops_check": (i32, []),
            "forge_flash_prefill": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
            "forge_api_version_v1": (C.c_uint32, []),
            "forge_tier_dispatch_v1": (i32, [i32, C.POINTER(ForgeShapeInfo), i32, i32, i32,
                                             C.POINTER(ForgeArgs), C.POINTER(ForgeArgs)]),
            "forge_tier_dispatch_v2": (i32, [i32, C.POINTER(ForgeShapeInfo), i32, i32, i32,
                                             C.POINTER(ForgeArgs), C.POINTER(ForgeArgs)]),
            "forge_register_specialized_v1": (i32, [i32, C.POINTER(ForgeShapeInfo), i32, i32, vp]),
            "forge_b200_embed": (i32, [vp, i32, vp, vp]),
            "forge_b200_qkv_rope": (i32, [vp, i32, i32, vp, vp]),
            "forge_b200_attention": (i32, [vp, i32, i32, vp, vp]),
            "forge_b200_o_proj": (i32, [vp, i32, i32, vp, vp]),
            "forge_b200_mlp": (i32, [vp, i32, i32, vp, vp]),
            "forge_b200_lm_head": (i32, [vp, i32, vp, vp, vp]),
            "forge_b200_advance": (i32, [vp, i32]),
            "forge_b200_set_kv": (i32, [vp, i32, i32, vp, vp, i32]),
            "hexa_farr_bf16_alloc": (C.POINTER(HexaFarrBf16), [i64]),
            "hexa_farr_bf16_free": (None, [C.POINTER(HexaFarrBf16)]),
            "hexa_farr_bf16_from_f64": (i32, [vp, C.POINTER(HexaFarrBf16), i64]),
            "hexa_farr_bf16_to_f64": (i32, [C.POINTER(HexaFarrBf16), vp, i64]),
            "hexa_farr_bf16_to_device": (i32, [C.POINTER(HexaFarrBf16)]),
            "hexa_farr_bf16_to_host": (i32, [C.POINTER(HexaFarrBf16)]),
            "hexa_farr_f32_alloc": (C.POINTER(HexaFarrF32), [i64]),
            "hexa_farr_f32_free": (None, [C.POINTER(HexaFarrF32)]),
            "hexa_farr_f32_to_device": (i32, [C.POINTER(HexaFarrF32)]),
            "hexa_farr_f32_to_host": (i32, [C.POINTER(HexaFarrF32)]),
            "hexa_farr_i32_alloc": (C.POINTER(HexaFarrI32), [i64]),
            "hexa_farr_i32_free": (None, [C.POINTER(HexaFarrI32)]),
            "hexa_farr_i32_to_device": (i32, [C.POINTER(HexaFarrI32)]),
            "hexa_farr_i32_to_host": (i32, [C.POINTER(HexaFarrI32)]),
            "hexa_farr_w_alloc": (C.POINTER(HexaFarrW), [i32, i64, i64]),
            "hexa_farr_q4_alloc": (C.POINTER(HexaFarrW), [i64, i64, i32]),
            "hexa_farr_w_pack": (i32, [C.POINTER(HexaFarrW), C.POINTER(HexaFarrBf16)]),
            "hexa_farr_q4_unpack": (i32, [C.POINTER(HexaFarrW), vp, vp]),
            "hexa_farr_w_free": (None, [C.POINTER(HexaFarrW)]),
            "hexa_kv_alloc": (C.POINTER(HexaKvCache), [i64, i64, i64, i64, i64]),
            "hexa_kv_free": (None, [C.POINTER(HexaKvCache)]),
            "hexa_kv_set_positions": (i32, [C.POINTER(HexaKvCache), vp, i64]),
            "hexa_kv_write": (i32, [C.POINTER(HexaKvCache), i64, i64, vp, vp, i64]),
            "forge_api_version_v2": (C.c_uint32, []),
            "forge_sample": (i32, [vp, i64, i32, i32, C.c_double, i32, C.c_double, vp, vp, vp, vp]),
            "forge_b200_decode_step_sampled": (i32, [vp, i32, vp, vp, C.c_double, i32, C.c_double, vp]),
            "forge_b200_desc_from_packed": (i32, [vp, C.POINTER(ForgeModelDesc)]),
            "forge_b200_create_packed": (i32, [vp]),
            "forge_b200_decode_step_sampled_packed": (i32, [vp]),
            "forge_paged_kv_create": (i32, [i32, i32, i32, C.POINTER(vp)]),
            "forge_paged_kv_destroy": (None, [vp]),
            "forge_paged_kv_free_count": (i32, [vp]),
            "forge_paged_kv_used_count": (i32, [vp]),
            "forge_paged_kv_seq_count": (i32, [vp]),
            "forge_paged_kv_register_seq": (i32, [vp, i64]),
            "forge_paged_kv_alloc_page": (i32, [vp, i64]),
            "forge_paged_kv_release_page": (i32, [vp, i64, i32]),
            "forge_paged_kv_release_seq": (i32, [vp, i64]),
            "forge_paged_kv_page_table": (i32, [vp, i64, vp, i32]),
            "forge_paged_kv_stats": (i32, [vp, C.POINTER(ForgePagedKvStats)]),
            "forge_flash_decode_paged": (i32, [vp, vp, vp, i32, vp, i32, i32, vp, i32, i32, i32, i32, vp, vp, vp]),
            "forge_clm_open": (i32, [C.c_char_p, C.POINTER(vp)]),
            "forge_clm_close": (None, [vp]),
            "forge_clm_count": (i32, [vp]),
            "forge_clm_block": (i32, [vp, i32, C.POINTER(ForgeClmBlock)]),
            "forge_clm_block_levels": (i32, [vp, i32, vp, vp]),
            "forge_clm_block_to_q4g128": (i32, [vp, i32, vp, vp]),
            "forge_st_open": (i32, [C.c_char_p, C.POINTER(vp)]),
            "forge_st_close": (i32, [vp]),
            "forge_st_header": (vp, [vp, C.POINTER(C.c_int64)]),
            "forge_st_data_offset": (i64, [vp]),
            "forge_st_size": (i64, [vp]),
            "forge_st_count": (i32, [vp]),
            "forge_st_total_bytes": (i64, [vp]),
            "forge_st_tensor_at": (i32, [vp, i32, C.POINTER(ForgeStTensor)]),
            "forge_st_find": (i32, [vp, C.c_char_p, C.POINTER(ForgeStTensor)]),
            "forge_st_metadata": (C.c_char_p, [vp, C.c_char_p]),
            "forge_st_view_u8": (i32, [C.POINTER(ForgeStTensor), i64]),
            "forge_st_read_bytes": (i64, [vp, i64, i64, vp]),
            "forge_st_read_f32": (i64, [vp, i64, i64, vp]),
            "forge_st_read_bf16_to_f32": (i64, [vp, i64, i64, vp]),
            "forge_st_tensor_to_bf16": (i32, [C.POINTER(ForgeStTensor), vp, i64]),
            "forge_st_tensor_to_f32": (i32, [C.POINTER(ForgeStTensor), vp, i64]),
            "forge_b200_load_safetensors": (i32, [vp, i32, C.POINTER(C.c_char_p)]),
            "forge_safetensors_check_llama": (i32, [C.POINTER(ForgeModelDesc), i32, C.POINTER(C.c_char_p)]),
        }
        for name, (res, args) in sig.items():
            if hasattr(L, name):
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
        _lib = L
    return _lib


class ForgeError(RuntimeError):
    pass


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().forge_b200_last_error().decode(errors="replace")
        raise ForgeError(f"{what} failed ({rc}): {msg}")


def _ptr(a) -> int:
    """Data pointer of a numpy array or a torch tensor."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


class PagedKv:
    """Host page allocator of the paged KV cache (forge_paged_kv_*; the
    contract of self/alloc/paged_kv.hexa)."""

    def __init__(self, num_pages=64, page_tokens=16, head_dim=64):
        h = C.c_void_p()
        check(lib().forge_paged_kv_create(num_pages, page_tokens, head_dim, C.byref(h)), "forge_paged_kv_create")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().forge_paged_kv_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    free_count = property(lambda self: lib().forge_paged_kv_free_count(self.h))
    used_count = property(lambda self: lib().forge_paged_kv_used_count(self.h))
    seq_count = property(lambda self: lib().forge_paged_kv_seq_count(self.h))

    def register_seq(self, seq):
        check(lib().forge_paged_kv_register_seq(self.h, seq), "register_seq")

    def alloc_page(self, seq):
        return lib().forge_paged_kv_alloc_page(self.h, seq)

    def release_page(self, seq, page_id):
        return lib().forge_paged_kv_release_page(self.h, seq, page_id) == 0

    def release_seq(self, seq):
        return lib().forge_paged_kv_release_seq(self.h, seq) == 0

    def page_table(self, seq):
        import numpy as np
        n = lib().forge_paged_kv_page_table(self.h, seq, None, 0)
        out = np.zeros(n, np.int32)
        lib().forge_paged_kv_page_table(self.h, seq, out.ctypes.data if n else None, n)
        return out.tolist()

    def seq_pages(self, seq):
        return lib().forge_paged_kv_page_table(self.h, seq, None, 0)

    def stats(self):
        s = ForgePagedKvStats()
        check(lib().forge_paged_kv_stats(self.h, C.byref(s)), "stats")
        return s


class Clm:
    """A .clm int4 checkpoint (forge_clm_*; stdlib/flame/clm_ckpt.hexa)."""

    def __init__(self, path):
        h = C.c_void_p()
        check(lib().forge_clm_open(os.fsencode(path), C.byref(h)), f"forge_clm_open({path})")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().forge_clm_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self):
        return lib().forge_clm_count(self.h)

    def block(self, i):
        b = ForgeClmBlock()
        check(lib().forge_clm_block(self.h, i, C.byref(b)), "forge_clm_block")
        return b

    def levels(self, i):
        """(q int8 [Cout][rest], scale fp32 [Cout]) as stored."""
        import numpy as np
        b = self.block(i)
        q = np.empty((b.cout, b.rest), np.int8)
        s = np.empty(b.cout, np.float32)
        check(lib().forge_clm_block_levels(self.h, i, q.ctypes.data, s.ctypes.data), "forge_clm_block_levels")
        return q, s

    def to_q4g128(self, i):
        """(codes u8 [Cout][rest], bf16 scales [Cout][rest / 128]) of the group-128 format."""
        import numpy as np
        b = self.block(i)
        codes = np.empty((b.cout, b.rest), np.uint8)
        sc = np.empty((b.cout, b.rest // 128), np.uint16)
        check(lib().forge_clm_block_to_q4g128(self.h, i, codes.ctypes.data, sc.ctypes.data), "forge_clm_block_to_q4g128")
        return codes, sc


class Safetensors:
    """Read-only mapped safetensors file (forge_st_*; the hexa runtime's
    safetensors_mmap_* builtins, self/runtime.h:1068-1082). Host only."""

    def __init__(self, path):
        h = C.c_void_p()
        check(lib().forge_st_open(os.fsencode(path), C.byref(h)), f"forge_st_open({path})")
        self.h = h

    def close(self):
        rc = 0
        if getattr(self, "h", None):
            rc = lib().forge_st_close(self.h)
            self.h = None
        return rc

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def header(self) -> bytes:
        n = C.c_int64()
        p = lib().forge_st_header(self.h, C.byref(n))
        return C.string_at(p, n.value)

    @property
    def data_offset(self):
        return lib().forge_st_data_offset(self.h)

    @property
    def size(self):
        return lib().forge_st_size(self.h)

    @property
    def total_bytes(self):
        return lib().forge_st_total_bytes(self.h)

    def __len__(self):
        return lib().forge_st_count(self.h)

    def tensor_at(self, i) -> ForgeStTensor:
        v = ForgeStTensor()
        check(lib().forge_st_tensor_at(self.h, i, C.byref(v)), "forge_st_tensor_at")
        return v

    def names(self):
        return [self.tensor_at(i).name.decode() for i in range(len(self))]

    def find(self, name):
        """The tensor view, or None when the file has no such tensor."""
        v = ForgeStTensor()
        rc = lib().forge_st_find(self.h, name.encode(), C.byref(v))
        if rc == FORGE_ST_NOT_FOUND:
            return None
        check(rc, "forge_st_find")
        return v

    def metadata(self, key):
        r = lib().forge_st_metadata(self.h, key.encode())
        return None if r is None else r.decode()

    def read_bytes(self, off, n) -> bytes:
        buf = C.create_string_buffer(max(n, 1))
        r = lib().forge_st_read_bytes(self.h, off, n, buf)
        if r < 0:
            check(r, "forge_st_read_bytes")
        return buf.raw[:n]

    def _read_f(self, fn, off, n):
        import numpy as np
        out = np.empty(n, np.float32)
        r = fn(self.h, off, n, out.ctypes.data)
        if r < 0:
            check(r, fn.__name__)
        return out

    def read_f32(self, off, n):
        return self._read_f(lib().forge_st_read_f32, off, n)

    def read_bf16_to_f32(self, off, n):
        return self._read_f(lib().forge_st_read_bf16_to_f32, off, n)

    def to_bf16(self, v):
        """The tensor as bf16 bit patterns (uint16), rounded to nearest even."""
        import numpy as np
        n = int(np.prod([v.shape[i] for i in range(v.ndim)], dtype=np.int64))
        out = np.empty(n, np.uint16)
        check(lib().forge_st_tensor_to_bf16(C.byref(v), out.ctypes.data, n), "forge_st_tensor_to_bf16")
        return out

    def to_f32(self, v):
        import numpy as np
        n = int(np.prod([v.shape[i] for i in range(v.ndim)], dtype=np.int64))
        out = np.empty(n, np.float32)
        check(lib().forge_st_tensor_to_f32(C.byref(v), out.ctypes.data, n), "forge_st_tensor_to_f32")
        return out


class ForgeModel:
    """One decode engine on one GPU (forge_b200_create / ..._destroy)."""

    def __init__(self, n_layer, d_model, n_head, n_kv_head, head_dim, ffn, vocab, *,
                 weight_kind=FORGE_WEIGHT_BF16, tied_head=False, max_batch=1, max_ctx=256,
                 rms_eps=1e-5, rope_theta=10000.0, act_mode=0, device=0, tp_rank=0, tp_size=1, nccl_id=None):
        self.desc = ForgeModelDesc(n_layer, d_model, n_head, n_kv_head, head_dim, ffn, vocab,
                                   rms_eps, rope_theta, weight_kind, int(tied_head), max_batch,
                                   max_ctx, tp_rank, tp_size, act_mode)
        h = C.c_void_p()
        if tp_size > 1:
            idb = C.create_string_buffer(bytes(nccl_id), 128)
            check(lib().forge_b200_create_tp(C.byref(self.desc), device, idb, C.byref(h)), "forge_b200_create_tp")
        else:
            check(lib().forge_b200_create(C.byref(self.desc), device, C.byref(h)), "forge_b200_create")
        self.h = h
        self.vocab = vocab

    def close(self):
        if getattr(self, "h", None):
            lib().forge_b200_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_synthetic(self, seed=1234, std=0.02):
        check(lib().forge_b200_init_synthetic(self.h, seed, std), "init_synthetic")

    def load_layer(self, layer, wq, wk, wv, wo, wg, wu, wd, g1, g2):
        w = ForgeLayerWeights(*[_ptr(a) for a in (wq, wk, wv, wo, wg, wu, wd, g1, g2)])
        check(lib().forge_b200_load_layer(self.h, layer, C.byref(w)), "load_layer")

    def load_embedding(self, emb, gF, head=None):
        check(lib().forge_b200_load_embedding(self.h, _ptr(emb), _ptr(gF), _ptr(head)), "load_embedding")

    def load_safetensors(self, paths):
        """Llama-layout checkpoint from one or more .safetensors shards."""
        if isinstance(paths, (str, bytes, os.PathLike)):
            paths = [paths]
        arr = (C.c_char_p * len(paths))(*[os.fsencode(p) for p in paths])
        check(lib().forge_b200_load_safetensors(self.h, len(paths), arr), "load_safetensors")

    def reset(self):
        check(lib().forge_b200_reset(self.h), "reset")

    def fill_kv_synthetic(self, seed, ctx_len, std=0.5):
        check(lib().forge_b200_fill_kv_synthetic(self.h, seed, ctx_len, std), "fill_kv_synthetic")

    def set_positions(self, pos):
        import numpy as np
        p = np.ascontiguousarray(pos, dtype=np.int32)
        check(lib().forge_b200_set_positions(self.h, _ptr(p), len(p)), "set_positions")

    def get_kv(self, layer, seq, n_kv, max_ctx, hd):
        import numpy as np
        k = np.zeros((n_kv, max_ctx, hd), np.uint16)
        v = np.zeros_like(k)
        check(lib().forge_b200_get_kv(self.h, layer, seq, _ptr(k), _ptr(v)), "get_kv")
        return k, v

    def set_kv(self, layer, seq, k, v):
        """k, v: host bf16 bit patterns [n_kv_head][n_pos][head_dim]."""
        import numpy as np
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        check(lib().forge_b200_set_kv(self.h, layer, seq, _ptr(k), _ptr(v), k.shape[1]), "set_kv")

    # block-level entries on device arrays (torch CUDA tensors), handle stream
    def embed(self, batch, tok, x):
        check(lib().forge_b200_embed(self.h, batch, _ptr(tok), _ptr(x)), "embed")

    def qkv_rope(self, layer, batch, x, q):
        check(lib().forge_b200_qkv_rope(self.h, layer, batch, _ptr(x), _ptr(q)), "qkv_rope")

    def attention(self, layer, batch, q, ctx):
        check(lib().forge_b200_attention(self.h, layer, batch, _ptr(q), _ptr(ctx)), "attention")

    def o_proj(self, layer, batch, ctx, x):
        check(lib().forge_b200_o_proj(self.h, layer, batch, _ptr(ctx), _ptr(x)), "o_proj")

    def mlp(self, layer, batch, x, y):
        check(lib().forge_b200_mlp(self.h, layer, batch, _ptr(x), _ptr(y)), "mlp")

    def lm_head(self, batch, x, tok, logits=None):
        check(lib().forge_b200_lm_head(self.h, batch, _ptr(x), _ptr(tok), _ptr(logits)), "lm_head")

    def advance(self, batch):
        check(lib().forge_b200_advance(self.h, batch), "advance")

    def step(self, tokens, want_logits=False):
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = np.zeros(len(t), np.int32)
        lg = np.zeros((len(t), self.vocab), np.float32) if want_logits else None
        check(lib().forge_b200_decode_step(self.h, len(t), _ptr(t), _ptr(nxt), _ptr(lg)), "decode_step")
        return (nxt, lg) if want_logits else nxt

    def step_sampled(self, tokens, rng_state, temperature=0.7, top_k=40, top_p=0.9):
        """One step with the reference sampler (defaults: gpu_sampler_default);
        rng_state is an int64 array [batch], advanced in place."""
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        assert rng_state.dtype == np.int64 and rng_state.flags.c_contiguous and rng_state.size >= len(t)
        nxt = np.zeros(len(t), np.int32)
        check(lib().forge_b200_decode_step_sampled(self.h, len(t), _ptr(t), _ptr(nxt), float(temperature),
                                                    int(top_k), float(top_p), _ptr(rng_state)), "decode_step_sampled")
        return nxt

    def decode_device(self, batch, n_steps):
        check(lib().forge_b200_decode_device(self.h, batch, n_steps), "decode_device")

    def sync(self):
        check(lib().forge_b200_sync(self.h), "sync")

    def prefill(self, prompt, exact=1, want_logits=False):
        """All prompt positions in one pass; returns the next token of every
        sequence (and its logits). prompt: [batch][n] (or [n])."""
        import numpy as np
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        if p.ndim == 1:
            p = p[None, :]
        nxt = np.zeros(p.shape[0], np.int32)
        lg = np.zeros((p.shape[0], self.vocab), np.float32) if want_logits else None
        check(lib().forge_b200_prefill(self.h, p.shape[0], _ptr(p), p.shape[1], int(exact), _ptr(nxt), _ptr(lg)),
              "prefill")
        return (nxt, lg) if want_logits else nxt

    def forward_rows(self, tok, pos, seq, out_rows, exact=1, want_logits=False):
        """One pass over ragged rows (token, position, sequence slot); the
        argmax (and logits) of the rows out_rows."""
        import numpy as np
        t, p, q, o = (np.ascontiguousarray(a, dtype=np.int32) for a in (tok, pos, seq, out_rows))
        nxt = np.zeros(len(o), np.int32)
        lg = np.zeros((len(o), self.vocab), np.float32) if want_logits else None
        check(lib().forge_b200_forward_rows(self.h, len(t), _ptr(t), _ptr(p), _ptr(q), len(o), _ptr(o), int(exact),
                                            _ptr(nxt), _ptr(lg)), "forward_rows")
        return (nxt, lg) if want_logits else nxt

    def generate(self, prompt, n_gen):
        import numpy as np
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        if p.ndim == 1:
            p = p[None, :]
        out = np.zeros((p.shape[0], n_gen), np.int32)
        check(lib().forge_b200_generate(self.h, p.shape[0], _ptr(p), p.shape[1], n_gen, _ptr(out)),
              "generate")
        return out

    def step_bytes(self, batch, ctx):
        return lib().forge_b200_step_bytes(self.h, batch, ctx)

    def uses_fused_step(self, batch):
        return lib().forge_b200_uses_fused_step(self.h, batch) == 1

    def launches_per_step(self, batch):
        return lib().forge_b200_launches_per_step(self.h, batch)

    @property
    def stream(self):
        return lib().forge_b200_stream(self.h)


def tp_heartbeat(store, rank, world, step, timeout_s=5.0):
    """Host-side liveness check of a tensor-parallel group before a step is
    launched: every rank posts forge_hb/<step>/<rank> in a shared key-value
    store (a torch.distributed Store) and waits for the other ranks' keys of
    the same step. A rank that left between steps (exited, crashed, stopped)
    is found here, on the host, before any kernel or collective of the step
    is launched — a device collective with a missing peer would otherwise
    wait on the GPU until its own bounded wait (FORGE_WAIT_NS) ran out.
    Raises ForgeError naming the ranks that are missing."""
    import datetime
    store.set(f"forge_hb/{step}/{rank}", "1")
    keys = [f"forge_hb/{step}/{r}" for r in range(world)]
    try:
        store.wait(keys, datetime.timedelta(seconds=timeout_s))
    except Exception:
        missing = [r for r in range(world) if not store.check([f"forge_hb/{step}/{r}"])]
        raise ForgeError(f"tensor-parallel rank(s) {missing} missed the heartbeat of step {step}")


def tp_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id for forge_b200_create_tp."""
    buf = C.create_string_buffer(128)
    check(lib().forge_b200_tp_unique_id(buf), "forge_b200_tp_unique_id")
    return buf.raw


def tp_split(n, gran, rank, size):
    off, ln = C.c_int64(), C.c_int64()
    check(lib().forge_tp_split(n, gran, rank, size, C.byref(off), C.byref(ln)), "forge_tp_split")
    return off.value, ln.value


# ---- per-op helpers on torch CUDA tensors -----------------------------------
def q4_pack(w_bf16_dev, group=128, stream=None):
    """Quantise a logical [N][K] bf16 device tensor (torch.int16/uint16 view)
    and pack it: returns (codes, scales, tiles, scale_tiles) torch tensors."""
    import torch
    N, K = w_bf16_dev.shape
    dev = w_bf16_dev.device
    codes = torch.empty((N, K // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty((N, K // group), dtype=torch.int16, device=dev)
    tiles = torch.empty(lib().forge_q4_tile_bytes(N, K), dtype=torch.uint8, device=dev)
    stiles = torch.empty(lib().forge_q4_scale_tile_bytes(N, K, group), dtype=torch.uint8, device=dev)
    s = stream or 0
    check(lib().forge_q4_quantize_bf16(_ptr(w_bf16_dev), N, K, group, _ptr(codes), _ptr(scales), s), "q4_quantize")
    check(lib().forge_q4_pack_tiles(_ptr(codes), _ptr(scales), N, K, group, _ptr(tiles), _ptr(stiles), s), "q4_pack")
    return codes, scales, tiles, stiles


def bf16_pack(w_bf16_dev, stream=None):
    import torch
    N, K = w_bf16_dev.shape
    tiles = torch.empty(N * K * 2, dtype=torch.uint8, device=w_bf16_dev.device)
    check(lib().forge_bf16_pack_tiles(_ptr(w_bf16_dev), N, K, _ptr(tiles), stream or 0), "bf16_pack")
    return tiles


class ForgeServe:
    """Continuous batching (include/forge_serve.h): the cb2 scheduler of
    self/ml/continuous_batching.hexa; with a ForgeModel every iteration runs
    one ragged engine pass and each request generates greedy tokens, without
    one (model=None) the scheduler keeps the books alone."""

    def __init__(self, model, max_batch, max_kv_slots):
        h = C.c_void_p()
        self.model = model
        check(lib().forge_serve_create(model.h if model is not None else None, max_batch, max_kv_slots,
                                       C.byref(h)), "forge_serve_create")
        self.h = h

    def close(self):
        if self.h:
            lib().forge_serve_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _rc(self, rc, what):
        if rc < 0:
            check(rc, what)
        return rc

    def set_eos(self, eos):
        check(lib().forge_serve_set_eos(self.h, eos), "set_eos")

    def add_request(self, req_id, prompt_len=None, max_gen=1, priority=0, deadline=0, prompt=None):
        import numpy as np
        p = None
        if prompt is not None:
            p = np.ascontiguousarray(prompt, dtype=np.int32)
            prompt_len = len(p)
        check(lib().forge_serve_add_request(self.h, req_id, _ptr(p), prompt_len, max_gen, priority, deadline),
              "add_request")

    def run_step(self, cur_time):
        return self._rc(lib().forge_serve_run_step(self.h, cur_time), "run_step")

    def run_until_done(self, max_steps):
        return self._rc(lib().forge_serve_run_until_done(self.h, max_steps), "run_until_done")

    def check_deadlines(self, cur_time):
        return self._rc(lib().forge_serve_check_deadlines(self.h, cur_time), "check_deadlines")

    def preempt(self, req_id):
        return self._rc(lib().forge_serve_preempt(self.h, req_id), "preempt")

    def preempt_for_room(self, needed):
        return self._rc(lib().forge_serve_preempt_for_room(self.h, needed), "preempt_for_room")

    def swap_out(self, req_id):
        return self._rc(lib().forge_serve_swap_out(self.h, req_id), "swap_out")

    def swap_in(self, req_id):
        return self._rc(lib().forge_serve_swap_in(self.h, req_id), "swap_in")

    @staticmethod
    def _as_dict(st, fields):
        return {n: getattr(st, n) for n in fields}

    def peek_queue(self):
        r = ForgeServeRequest()
        return {} if self._rc(lib().forge_serve_peek_queue(self.h, C.byref(r)), "peek_queue") == 1 else \
            self._as_dict(r, SERVE_REQUEST_FIELDS)

    def find_request(self, req_id):
        r = ForgeServeRequest()
        return {} if self._rc(lib().forge_serve_find_request(self.h, req_id, C.byref(r)), "find_request") == 1 else \
            self._as_dict(r, SERVE_REQUEST_FIELDS)

    def count_by_phase(self, phase):
        return lib().forge_serve_count_by_phase(self.h, phase)

    def stats(self):
        st = ForgeServeStats()
        check(lib().forge_serve_stats(self.h, C.byref(st)), "stats")
        return self._as_dict(st, SERVE_STATS_FIELDS)

    def throughput(self):
        st = ForgeServeThroughput()
        check(lib().forge_serve_throughput(self.h, C.byref(st)), "throughput")
        return self._as_dict(st, SERVE_THROUGHPUT_FIELDS)

    def output(self, req_id):
        import numpy as np
        n = C.c_int64()
        if self._rc(lib().forge_serve_output(self.h, req_id, None, 0, C.byref(n)), "output") == 1:
            return None
        out = np.zeros(n.value, np.int32)
        check(lib().forge_serve_output(self.h, req_id, _ptr(out), n.value, C.byref(n)), "output")
        return out

    def engine_time(self):
        ms, rows, passes = C.c_double(), C.c_int64(), C.c_int64()
        check(lib().forge_serve_engine_time(self.h, C.byref(ms), C.byref(rows), C.byref(passes)), "engine_time")
        return ms.value, rows.value, passes.value
