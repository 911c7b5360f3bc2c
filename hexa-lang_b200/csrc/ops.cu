// ops.cu — per-op C-ABI entries on caller-owned device memory: the decode
// GEMVs and split-K flash-decode as standalone kernels (the B200 siblings of
// forge's _hx_cuda_farr_packed_gemv_offset_gpu, runtime_cuda_emit.hexa:1858,
// and of the attention kernel entry, :2819). No hidden allocation beyond one
// 16-byte device error word per device, created on first use.
#include <mutex>
#include "forge_internal.h"
#include "../../include/forge_paged_kv.h"
#include "../../include/forge_b200.h"

namespace {
uint32_t* g_err[64] = {nullptr};
std::mutex g_err_mu;

uint32_t* err_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_err_mu);
    if (!g_err[dev]) {
        void* p = nullptr;
        if (cudaMalloc(&p, 16) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, 16);
        g_err[dev] = (uint32_t*)p;
    }
    return g_err[dev];
}

}  // namespace

uint32_t* forge_ops_err_word() { return err_word(); }

namespace {
int gemv_entry(int wkind, const void* tiles, const void* stiles, int64_t N, int64_t K, const float* x, int batch,
               float* y, int exact, void* stream) {
    if (!tiles || !x || !y || batch <= 0 || N <= 0 || K <= 0 || N > (1ll << 30) || K > (1ll << 30))
        return forge_fail(FORGE_INVALID_ARGS, "forge_gemv: bad args");
    uint32_t* err = err_word();
    if (!err) return forge_fail(-1, "forge_gemv: no device");
    if (forge_gemv_configure()) return -1;
    ForgeGemvArgs a{};
    a.w = tiles; a.s = stiles; a.N = (int32_t)N; a.K = (int32_t)K; a.wkind = wkind;
    a.batch = batch; a.split = exact ? 1 : 0; a.x = x; a.x_stride = (int32_t)K;
    a.pro = FORGE_PRO_PLAIN; a.epi = FORGE_EPI_STORE; a.y = y; a.y_stride = (int32_t)N; a.err = err;
    if (batch > 4 && (wkind == FORGE_W_Q4 || !exact)) {
        // batched path: library-owned activation scratch, grown on demand
        static std::mutex mu;
        static void* buf[64] = {nullptr};
        static int64_t cap[64] = {0};
        int dev = 0;
        cudaGetDevice(&dev);
        if (forge_gemv_b_configure()) return -1;
        std::lock_guard<std::mutex> lk(mu);
        const int64_t need = forge_gemv_b_scratch_bytes((int)K);
        if (need > cap[dev]) {
            if (buf[dev]) {
                cudaStreamSynchronize((cudaStream_t)stream);
                cudaFree(buf[dev]);
            }
            buf[dev] = nullptr;
            cap[dev] = 0;
            if (cudaMalloc(&buf[dev], (size_t)need) != cudaSuccess || cudaMemset(buf[dev], 0, (size_t)need) != cudaSuccess) {
                cudaGetLastError();
                if (buf[dev]) cudaFree(buf[dev]);
                buf[dev] = nullptr;
                return forge_fail(-1, "forge_gemv: batched scratch of %lld bytes", (long long)need);
            }
            cap[dev] = need;
        }
        a.bscratch = buf[dev];
        return forge_gemv_launch(a, (cudaStream_t)stream, false) ? FORGE_INVALID_ARGS : 0;
    }
    int rc = forge_gemv_launch(a, (cudaStream_t)stream, false);
    return rc ? FORGE_INVALID_ARGS : 0;
}
}  // namespace

extern "C" {
FORGE_API int forge_gemv_w4a16_g128(const void* tiles, const void* scale_tiles, int64_t N, int64_t K,
                                    const float* x, int batch, float* y, int exact, void* stream) {
    if (!scale_tiles) return forge_fail(FORGE_INVALID_ARGS, "forge_gemv_w4a16_g128: null scales");
    return gemv_entry(FORGE_W_Q4, tiles, scale_tiles, N, K, x, batch, y, exact, stream);
}
FORGE_API int forge_gemv_bf16(const void* tiles, int64_t N, int64_t K, const float* x, int batch, float* y,
                              int exact, void* stream) {
    return gemv_entry(FORGE_W_BF16, tiles, nullptr, N, K, x, batch, y, exact, stream);
}

FORGE_API int64_t forge_flash_decode_workspace_bytes(int B, int H, int Hkv, int hd, int lmax) {
    if (B <= 0 || H <= 0 || Hkv <= 0 || hd <= 0 || lmax <= 0) return -1;
    const int ns = forge_attn_pick_splits(B, Hkv, lmax);
    const int64_t counters = ((int64_t)B * Hkv * 4 + 255) / 256 * 256;
    return counters + 4 * forge_attn_partial_floats(B, H, hd, ns);
}

FORGE_API int forge_flash_decode(const float* q, const uint16_t* kc, const uint16_t* vc, const int32_t* pos, int B,
                                 int H, int Hkv, int hd, int lmax, float* out, void* workspace, void* stream) {
    if (!q || !kc || !vc || !pos || !out || !workspace || B <= 0 || H <= 0 || Hkv <= 0 || lmax <= 0)
        return forge_fail(FORGE_INVALID_ARGS, "forge_flash_decode: bad args");
    uint32_t* err = err_word();
    if (!err) return forge_fail(-1, "forge_flash_decode: no device");
    if (forge_attn_configure()) return -1;
    ForgeAttnArgs a{};
    a.q = q; a.kc = kc; a.vc = vc; a.pos = pos; a.B = B; a.H = H; a.Hkv = Hkv; a.hd = hd; a.lmax = lmax;
    a.nsplit = forge_attn_pick_splits(B, Hkv, lmax);
    const int64_t counters = ((int64_t)B * Hkv * 4 + 255) / 256 * 256;
    a.counters = (uint32_t*)workspace;
    a.partial = (float*)((char*)workspace + counters);
    a.out = out; a.err = err;
    return forge_attn_launch(a, (cudaStream_t)stream, false) ? FORGE_INVALID_ARGS : 0;
}

FORGE_API int forge_flash_decode_paged(const float* q, const uint16_t* k_pool, const uint16_t* v_pool, int num_pages,
                                       const int32_t* block_table, int max_pages, int page_tokens, const int32_t* pos,
                                       int B, int H, int Hkv, int hd, float* out, void* workspace, void* stream) {
    if (!q || !k_pool || !v_pool || !block_table || !pos || !out || !workspace || B <= 0 || H <= 0 || Hkv <= 0 ||
        num_pages <= 0 || max_pages <= 0 || page_tokens <= 0 || (int64_t)max_pages * page_tokens > (1 << 30))
        return forge_fail(FORGE_INVALID_ARGS, "forge_flash_decode_paged: bad args");
    uint32_t* err = err_word();
    if (!err) return forge_fail(-1, "forge_flash_decode_paged: no device");
    if (forge_attn_configure()) return -1;
    ForgeAttnArgs a{};
    a.q = q; a.kc = k_pool; a.vc = v_pool; a.pos = pos; a.B = B; a.H = H; a.Hkv = Hkv; a.hd = hd;
    a.lmax = max_pages * page_tokens;
    a.table = block_table; a.max_pages = max_pages; a.page_tokens = page_tokens; a.num_pages = num_pages;
    a.nsplit = forge_attn_pick_splits(B, Hkv, a.lmax);
    const int64_t counters = ((int64_t)B * Hkv * 4 + 255) / 256 * 256;
    a.counters = (uint32_t*)workspace;
    a.partial = (float*)((char*)workspace + counters);
    a.out = out; a.err = err;
    return forge_attn_launch(a, (cudaStream_t)stream, false) ? FORGE_INVALID_ARGS : 0;
}

// Reads and clears the per-device error word of the per-op entries.
FORGE_API int forge_ops_check(void) {
    uint32_t* err = err_word();
    if (!err) return forge_fail(-1, "forge_ops_check: no device");
    uint32_t e = 0;
    if (cudaMemcpy(&e, err, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return forge_fail(-1, "forge_ops_check: %s", cudaGetErrorString(cudaGetLastError()));
    if (e) {
        cudaMemset(err, 0, 4);
        return forge_fail(-1, "forge_ops_check: kernel error word 0x%x", e);
    }
    return 0;
}
}  // extern "C"
