// farr.cu — device-array descriptors (include/forge_farr.h).
//
// HexaFarrBf16 follows the reference's bf16 storage class
// (self/cuda/runtime_bf16_emit.hexa:292-413): calloc'd host buffer,
// cudaMalloc on first upload, upload only while the host copy is the
// authoritative one (loc == HOST), and RNE rounding from fp64 through fp32
// (_hx_f32_to_bf16_rne, :264-277). The fp32/int32 siblings, the packed
// weight descriptor and the KV-cache descriptor are additions of this
// library. Everything here is host code except the device packing calls.
#include <cstdlib>
#include <cstring>
#include "forge_internal.h"
#include "../../include/forge_b200.h"
#include "../../include/forge_farr.h"

namespace {
uint16_t f32_to_bf16_rne(float v) {
    uint32_t bits;
    std::memcpy(&bits, &v, 4);
    if (((bits >> 23) & 0xFF) == 0xFF && (bits & 0x7FFFFF)) return (uint16_t)((bits >> 16) | 0x40);
    return (uint16_t)((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
}
float bf16_to_f32(uint16_t b) {
    const uint32_t bits = (uint32_t)b << 16;
    float v;
    std::memcpy(&v, &bits, 4);
    return v;
}

// The three plain descriptors share one layout; these helpers work on any
// of them given the element size.
struct Plain {
    void* h_buf;
    void* d_buf;
    int64_t len;
    int loc;
    int owns;
};
static_assert(sizeof(Plain) == sizeof(HexaFarrBf16) && sizeof(Plain) == sizeof(HexaFarrF32) &&
                  sizeof(Plain) == sizeof(HexaFarrI32), "descriptor layout");

Plain* plain_alloc(int64_t len, size_t elem) {
    if (len < 0) {
        forge_fail(FORGE_INVALID_ARGS, "farr alloc: negative length");
        return nullptr;
    }
    Plain* f = (Plain*)std::calloc(1, sizeof(Plain));
    if (!f) return nullptr;
    f->h_buf = len > 0 ? std::calloc((size_t)len, elem) : nullptr;
    if (len > 0 && !f->h_buf) {
        std::free(f);
        forge_fail(-1, "farr alloc: host allocation of %lld elements failed", (long long)len);
        return nullptr;
    }
    f->len = len;
    f->loc = FARR_BF16_LOC_HOST;
    f->owns = 1;
    return f;
}

void plain_free(Plain* f) {
    if (!f) return;
    if (f->owns) {
        std::free(f->h_buf);
        if (f->d_buf) cudaFree(f->d_buf);
    }
    std::free(f);
}

int plain_to_device(Plain* f, size_t elem, const char* what) {
    if (!f || f->len < 0) return forge_fail(-1, "%s_to_device: bad descriptor", what);
    const size_t bytes = (size_t)f->len * elem;
    if (!f->d_buf && f->len > 0) {
        cudaError_t e = cudaMalloc(&f->d_buf, bytes);
        if (e != cudaSuccess) {
            f->d_buf = nullptr;
            return forge_fail(-1, "%s_to_device: cudaMalloc %zu B: %s", what, bytes, cudaGetErrorString(e));
        }
    }
    if (f->len > 0 && f->h_buf && f->loc == FARR_BF16_LOC_HOST) {
        cudaError_t e = cudaMemcpy(f->d_buf, f->h_buf, bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return forge_fail(-1, "%s_to_device: H2D: %s", what, cudaGetErrorString(e));
    }
    f->loc = FARR_BF16_LOC_MIRROR;
    return 0;
}

int plain_to_host(Plain* f, size_t elem, const char* what) {
    if (!f || f->len < 0 || !f->d_buf || !f->h_buf) return forge_fail(-1, "%s_to_host: bad descriptor", what);
    cudaError_t e = cudaMemcpy(f->h_buf, f->d_buf, (size_t)f->len * elem, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return forge_fail(-1, "%s_to_host: D2H: %s", what, cudaGetErrorString(e));
    f->loc = FARR_BF16_LOC_MIRROR;
    return 0;
}
}  // namespace

extern "C" {
// ---- bf16 ----------------------------------------------------------------
FORGE_API HexaFarrBf16* hexa_farr_bf16_alloc(int64_t len) { return (HexaFarrBf16*)plain_alloc(len, 2); }
FORGE_API void hexa_farr_bf16_free(HexaFarrBf16* f) { plain_free((Plain*)f); }

FORGE_API int hexa_farr_bf16_from_f64(const double* src, HexaFarrBf16* dst, int64_t n) {
    if (!src || !dst || !dst->h_buf || n < 0 || n > dst->len) return forge_fail(-1, "hexa_farr_bf16_from_f64: bad args");
    uint16_t* hb = (uint16_t*)dst->h_buf;
    for (int64_t i = 0; i < n; ++i) hb[i] = f32_to_bf16_rne((float)src[i]);
    dst->loc = FARR_BF16_LOC_HOST;
    return 0;
}

FORGE_API int hexa_farr_bf16_to_f64(const HexaFarrBf16* src, double* dst, int64_t n) {
    if (!src || !src->h_buf || !dst || n < 0 || n > src->len) return forge_fail(-1, "hexa_farr_bf16_to_f64: bad args");
    const uint16_t* hb = (const uint16_t*)src->h_buf;
    for (int64_t i = 0; i < n; ++i) dst[i] = (double)bf16_to_f32(hb[i]);
    return 0;
}

FORGE_API int hexa_farr_bf16_to_device(HexaFarrBf16* f) { return plain_to_device((Plain*)f, 2, "hexa_farr_bf16"); }
FORGE_API int hexa_farr_bf16_to_host(HexaFarrBf16* f) { return plain_to_host((Plain*)f, 2, "hexa_farr_bf16"); }

// ---- fp32 / int32 -------------------------------------------------------------
FORGE_API HexaFarrF32* hexa_farr_f32_alloc(int64_t len) { return (HexaFarrF32*)plain_alloc(len, 4); }
FORGE_API void hexa_farr_f32_free(HexaFarrF32* f) { plain_free((Plain*)f); }
FORGE_API int hexa_farr_f32_to_device(HexaFarrF32* f) { return plain_to_device((Plain*)f, 4, "hexa_farr_f32"); }
FORGE_API int hexa_farr_f32_to_host(HexaFarrF32* f) { return plain_to_host((Plain*)f, 4, "hexa_farr_f32"); }
FORGE_API HexaFarrI32* hexa_farr_i32_alloc(int64_t len) { return (HexaFarrI32*)plain_alloc(len, 4); }
FORGE_API void hexa_farr_i32_free(HexaFarrI32* f) { plain_free((Plain*)f); }
FORGE_API int hexa_farr_i32_to_device(HexaFarrI32* f) { return plain_to_device((Plain*)f, 4, "hexa_farr_i32"); }
FORGE_API int hexa_farr_i32_to_host(HexaFarrI32* f) { return plain_to_host((Plain*)f, 4, "hexa_farr_i32"); }

// ---- packed weights ------------------------------------------------------------
FORGE_API HexaFarrW* hexa_farr_w_alloc(int kind, int64_t rows, int64_t K) {
    if ((kind != HEXA_FARR_W_BF16 && kind != HEXA_FARR_W_Q4_G128) || rows <= 0 || K <= 0 || rows % 16 ||
        (kind == HEXA_FARR_W_BF16 ? K % 16 : K % 128)) {
        forge_fail(FORGE_INVALID_ARGS, "hexa_farr_w_alloc: kind %d rows %lld K %lld (rows %% 16, K %% 16 bf16 / "
                   "%% 128 int4)", kind, (long long)rows, (long long)K);
        return nullptr;
    }
    HexaFarrW* w = (HexaFarrW*)std::calloc(1, sizeof(HexaFarrW));
    if (!w) return nullptr;
    w->rows = rows;
    w->cols = K;
    w->kind = kind;
    w->group = kind == HEXA_FARR_W_Q4_G128 ? 128 : 0;
    w->owns = 1;
    w->tile_bytes = kind == HEXA_FARR_W_Q4_G128 ? forge_q4_tile_bytes(rows, K) : rows * K * 2;
    w->scale_bytes = kind == HEXA_FARR_W_Q4_G128 ? forge_q4_scale_tile_bytes(rows, K, 128) : 0;
    if (cudaMalloc(&w->d_tiles, (size_t)w->tile_bytes) != cudaSuccess ||
        (w->scale_bytes && cudaMalloc(&w->d_scales, (size_t)w->scale_bytes) != cudaSuccess)) {
        cudaGetLastError();
        hexa_farr_w_free(w);
        forge_fail(-1, "hexa_farr_w_alloc: device allocation failed");
        return nullptr;
    }
    return w;
}

FORGE_API HexaFarrW* hexa_farr_q4_alloc(int64_t rows, int64_t K, int group) {
    if (group != 128) {
        forge_fail(FORGE_PRECISION_UNSUPPORTED, "hexa_farr_q4_alloc: group %d (only 128)", group);
        return nullptr;
    }
    return hexa_farr_w_alloc(HEXA_FARR_W_Q4_G128, rows, K);
}

FORGE_API int hexa_farr_w_pack(HexaFarrW* w, HexaFarrBf16* logical) {
    if (!w || !logical || logical->len != w->rows * w->cols)
        return forge_fail(FORGE_INVALID_ARGS, "hexa_farr_w_pack: descriptor sizes differ");
    if (hexa_farr_bf16_to_device(logical)) return -1;
    const uint16_t* src = (const uint16_t*)logical->d_buf;
    int rc = 0;
    if (w->kind == HEXA_FARR_W_BF16) {
        rc = forge_bf16_pack_tiles(src, w->rows, w->cols, w->d_tiles, nullptr);
    } else {
        uint8_t* codes = nullptr;
        uint16_t* scales = nullptr;
        const int64_t G = w->cols / 128;
        if (cudaMalloc(&codes, (size_t)(w->rows * w->cols)) != cudaSuccess ||
            cudaMalloc(&scales, (size_t)(w->rows * G * 2)) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(codes);
            return forge_fail(-1, "hexa_farr_w_pack: staging allocation failed");
        }
        rc = forge_q4_quantize_bf16(src, w->rows, w->cols, 128, codes, scales, nullptr);
        if (!rc) rc = forge_q4_pack_tiles(codes, scales, w->rows, w->cols, 128, w->d_tiles, w->d_scales, nullptr);
        cudaError_t e = cudaDeviceSynchronize();
        cudaFree(codes);
        cudaFree(scales);
        if (!rc && e != cudaSuccess) rc = forge_fail(-1, "hexa_farr_w_pack: %s", cudaGetErrorString(e));
    }
    if (!rc) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) rc = forge_fail(-1, "hexa_farr_w_pack: %s", cudaGetErrorString(e));
    }
    w->packed = rc == 0;
    return rc ? -1 : 0;
}

FORGE_API int hexa_farr_q4_unpack(const HexaFarrW* w, uint8_t* codes, uint16_t* scales) {
    if (!w || w->kind != HEXA_FARR_W_Q4_G128 || !w->packed || !codes || !scales)
        return forge_fail(FORGE_INVALID_ARGS, "hexa_farr_q4_unpack: not a packed int4 descriptor");
    const int64_t G = w->cols / 128;
    uint8_t* dc = nullptr;
    uint16_t* ds = nullptr;
    if (cudaMalloc(&dc, (size_t)(w->rows * w->cols / 2)) != cudaSuccess ||
        cudaMalloc(&ds, (size_t)(w->rows * G * 2)) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(dc);
        return forge_fail(-1, "hexa_farr_q4_unpack: staging allocation failed");
    }
    int rc = forge_q4_unpack_tiles(w->d_tiles, w->d_scales, w->rows, w->cols, 128, dc, ds, nullptr);
    if (!rc && (cudaMemcpy(codes, dc, (size_t)(w->rows * w->cols / 2), cudaMemcpyDeviceToHost) != cudaSuccess ||
                cudaMemcpy(scales, ds, (size_t)(w->rows * G * 2), cudaMemcpyDeviceToHost) != cudaSuccess))
        rc = forge_fail(-1, "hexa_farr_q4_unpack: D2H: %s", cudaGetErrorString(cudaGetLastError()));
    cudaFree(dc);
    cudaFree(ds);
    return rc ? -1 : 0;
}

FORGE_API void hexa_farr_w_free(HexaFarrW* w) {
    if (!w) return;
    if (w->owns) {
        if (w->d_tiles) cudaFree(w->d_tiles);
        if (w->d_scales) cudaFree(w->d_scales);
    }
    std::free(w);
}

// ---- KV cache ------------------------------------------------------------------
FORGE_API HexaKvCache* hexa_kv_alloc(int64_t n_layer, int64_t batch, int64_t n_kv_head, int64_t max_ctx,
                                     int64_t head_dim) {
    if (n_layer <= 0 || batch <= 0 || n_kv_head <= 0 || max_ctx <= 0 || (head_dim != 64 && head_dim != 128)) {
        forge_fail(FORGE_INVALID_ARGS, "hexa_kv_alloc: bad shape (head_dim 64 or 128)");
        return nullptr;
    }
    HexaKvCache* kv = (HexaKvCache*)std::calloc(1, sizeof(HexaKvCache));
    if (!kv) return nullptr;
    kv->n_layer = n_layer; kv->batch = batch; kv->n_kv_head = n_kv_head; kv->max_ctx = max_ctx;
    kv->head_dim = head_dim; kv->owns = 1;
    const size_t bytes = (size_t)(n_layer * batch * n_kv_head * max_ctx * head_dim * 2);
    if (cudaMalloc(&kv->d_k, bytes) != cudaSuccess || cudaMalloc(&kv->d_v, bytes) != cudaSuccess ||
        cudaMalloc(&kv->d_pos, (size_t)batch * 4) != cudaSuccess || cudaMemset(kv->d_k, 0, bytes) != cudaSuccess ||
        cudaMemset(kv->d_v, 0, bytes) != cudaSuccess || cudaMemset(kv->d_pos, 0, (size_t)batch * 4) != cudaSuccess) {
        cudaGetLastError();
        hexa_kv_free(kv);
        forge_fail(-1, "hexa_kv_alloc: device allocation of 2 x %zu bytes failed", bytes);
        return nullptr;
    }
    return kv;
}

FORGE_API void hexa_kv_free(HexaKvCache* kv) {
    if (!kv) return;
    if (kv->owns) {
        if (kv->d_k) cudaFree(kv->d_k);
        if (kv->d_v) cudaFree(kv->d_v);
        if (kv->d_pos) cudaFree(kv->d_pos);
    }
    std::free(kv);
}

FORGE_API int hexa_kv_write(HexaKvCache* kv, int64_t layer, int64_t seq, const uint16_t* k, const uint16_t* v,
                             int64_t n_pos) {
    if (!kv || !k || !v || layer < 0 || layer >= kv->n_layer || seq < 0 || seq >= kv->batch || n_pos < 0 ||
        n_pos > kv->max_ctx)
        return forge_fail(FORGE_INVALID_ARGS, "hexa_kv_write: bad args");
    if (!n_pos) return 0;
    const size_t row = (size_t)kv->head_dim * 2, pitch = (size_t)kv->max_ctx * row;
    const size_t off = ((size_t)layer * kv->batch + seq) * kv->n_kv_head * pitch;
    if (cudaMemcpy2D((char*)kv->d_k + off, pitch, k, (size_t)n_pos * row, (size_t)n_pos * row, kv->n_kv_head,
                     cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy2D((char*)kv->d_v + off, pitch, v, (size_t)n_pos * row, (size_t)n_pos * row, kv->n_kv_head,
                     cudaMemcpyHostToDevice) != cudaSuccess)
        return forge_fail(-1, "hexa_kv_write: H2D: %s", cudaGetErrorString(cudaGetLastError()));
    return 0;
}

FORGE_API int hexa_kv_set_positions(HexaKvCache* kv, const int32_t* pos, int64_t batch) {
    if (!kv || !pos || batch <= 0 || batch > kv->batch) return forge_fail(FORGE_INVALID_ARGS, "hexa_kv_set_positions: bad args");
    for (int64_t b = 0; b < batch; ++b)
        if (pos[b] < 0 || pos[b] >= kv->max_ctx)
            return forge_fail(FORGE_INVALID_ARGS, "hexa_kv_set_positions: position %d outside the cache", pos[b]);
    cudaError_t e = cudaMemcpy(kv->d_pos, pos, (size_t)batch * 4, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? 0 : forge_fail(-1, "hexa_kv_set_positions: %s", cudaGetErrorString(e));
}
}  // extern "C"
