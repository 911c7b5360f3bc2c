// abi.cu — forge's dispatch entries: the frozen v1 surface and the v2
// families of this library.
//
// v1 (include/forge_tier_v1.h, reference self/forge/forge_tier_v1.h:24-130
// with the dispatcher in self/forge/forge_tier_v1_emit.hexa:87-375):
//   * forge_api_version_v1 returns 0x00010000;
//   * forge_register_specialized_v1 remembers up to 64 registrations in
//     memory and otherwise does nothing, as the reference's stub does;
//   * forge_tier_dispatch_v1 validates in the reference's order (pedantic
//     determinism needs FP64, unknown precision, unknown family) and then
//     routes the bf16 precisions: PURE_BF16 MATMUL / FFN_FUSED / RMSNORM_MH
//     / SILU_GATE / ROPE_MH run the kernels below on HexaFarrBf16 slots
//     (where the reference implements MATMUL and FFN_FUSED with cuBLAS and
//     leaves the other three unsupported); LAYERCAST_BF16_FP32 stays
//     FORGE_KERNEL_UNSUPPORTED as in the reference (its operands are plain
//     float arrays that do not fit the slot model). FP64 returns
//     FORGE_KERNEL_UNSUPPORTED: the reference's FP64 MATMUL runs the hexa
//     runtime's own farr table and CPU/Dgemm path, which this library does
//     not contain and does not fall back to.
// v2 (include/forge_b200.h): the decode families, on the descriptors of
// include/forge_farr.h or on a ForgeB200 handle.
//
// The v1 kernels run on the legacy default stream, so the synchronous
// hexa_farr_*_to_host copies order after them without an explicit sync.
#include <cublas_v2.h>
#include <dlfcn.h>
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include "common.cuh"
#include "forge_internal.h"
#include "../../include/forge_b200.h"
#include "../../include/forge_farr.h"

namespace {
// ---------------------------------------------------------------------------
// v1 bf16 kernels
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ld_bf16(const uint16_t* p, int64_t i) { return bf16_bits_to_f32(p[i]); }

// C[M][N] = A[M][K] B[K][N], row-major bf16, fp32 accumulation, bf16 (RNE)
// result. EPI 1 applies the reference FFN's activation to the rounded
// product: h = bf16(acc), out = bf16(silu(h)). 64x64 output tile per CTA,
// 256 threads with 4x4 outputs each, K in steps of 16 through shared memory.
template <int EPI>
__global__ void __launch_bounds__(256) k_matmul_bf16(const uint16_t* __restrict__ A, const uint16_t* __restrict__ B,
                                                     uint16_t* __restrict__ C, int64_t M, int64_t N, int64_t K) {
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * 64, n0 = (int64_t)blockIdx.x * 64;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < K; k0 += 16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = tid + i * 256;           // 0..1023
            const int am = e >> 4, ak = e & 15;    // A tile 64 x 16
            const int64_t gm = m0 + am, gk = k0 + ak;
            As[ak][am] = (gm < M && gk < K) ? ld_bf16(A, gm * K + gk) : 0.f;
            const int bk = e >> 6, bn = e & 63;    // B tile 16 x 64
            const int64_t gk2 = k0 + bk, gn = n0 + bn;
            Bs[bk][bn] = (gk2 < K && gn < N) ? ld_bf16(B, gk2 * N + gn) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t gm = m0 + ty * 4 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t gn = n0 + tx * 4 + j;
            if (gn >= N) continue;
            float v = acc[i][j];
            if (EPI == 1) {
                const float h = bf16_bits_to_f32(f32_to_bf16_bits(v));
                v = h / (1.0f + expf(-h));
            }
            C[gm * N + gn] = f32_to_bf16_bits(v);
        }
    }
}

// h = bf16(silu(h)) in place: the FFN's activation on the rounded product.
__global__ void k_silu_bf16_inplace(uint16_t* __restrict__ h, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = bf16_bits_to_f32(h[i]);
        h[i] = f32_to_bf16_bits(v / (1.0f + expf(-v)));
    }
}

// cuBLAS, opened at run time as the reference reaches it (cublasGemmEx with
// bf16 operands and fp32 compute, runtime_bf16_emit.hexa:487-540): the
// tensor-core GEMM for the v1 MATMUL and FFN_FUSED families. One handle per
// device on the legacy default stream. When the library cannot be opened
// the 64 x 64 tile kernel above runs instead (one line on stderr).
struct Blas {
    void* lib = nullptr;
    decltype(&cublasCreate_v2) create = nullptr;
    cublasStatus_t (*gemm)(cublasHandle_t, cublasOperation_t, cublasOperation_t, int, int, int, const void*,
                           const void*, cudaDataType, int, const void*, cudaDataType, int, const void*, void*,
                           cudaDataType, int, cublasComputeType_t, cublasGemmAlgo_t) = nullptr;
    cublasHandle_t handle[64] = {};
};
std::mutex g_blas_mu;
Blas g_blas;
bool g_blas_tried = false;

// The handle of the current device, or nullptr when cuBLAS is unavailable.
cublasHandle_t blas_handle() {
    std::lock_guard<std::mutex> lk(g_blas_mu);
    if (!g_blas_tried) {
        g_blas_tried = true;
        const char* path = getenv("FORGE_CUBLAS_LIB");
        g_blas.lib = dlopen(path && *path ? path : "libcublas.so.12", RTLD_NOW | RTLD_GLOBAL);
        if (g_blas.lib) {
            g_blas.create = (decltype(g_blas.create))dlsym(g_blas.lib, "cublasCreate_v2");
            g_blas.gemm = (decltype(g_blas.gemm))dlsym(g_blas.lib, "cublasGemmEx");
        }
        if (!g_blas.create || !g_blas.gemm)
            fprintf(stderr, "[forge_b200] cuBLAS not available (%s): v1 MATMUL / FFN_FUSED use the tile kernel\n",
                    g_blas.lib ? "missing symbols" : dlerror());
    }
    if (!g_blas.create || !g_blas.gemm) return nullptr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!g_blas.handle[dev] && g_blas.create(&g_blas.handle[dev]) != CUBLAS_STATUS_SUCCESS) {
        g_blas.handle[dev] = nullptr;
        return nullptr;
    }
    return g_blas.handle[dev];
}

// C[M][N] = A[M][K] B[K][N] (row-major bf16, fp32 accumulation, bf16 RNE
// result): the column-major product C^T = B^T A^T. Returns 1 when cuBLAS is
// unavailable or a dimension exceeds its int range.
int matmul_bf16(const uint16_t* A, const uint16_t* B, uint16_t* C, int64_t M, int64_t N, int64_t K) {
    const int64_t lim = (1ll << 31) - 1;
    cublasHandle_t hd = (M <= lim && N <= lim && K <= lim) ? blas_handle() : nullptr;
    if (!hd) {
        k_matmul_bf16<0><<<dim3((unsigned)((N + 63) / 64), (unsigned)((M + 63) / 64)), 256>>>(A, B, C, M, N, K);
        return 0;
    }
    const float one = 1.0f, zero = 0.0f;
    const cublasStatus_t st = g_blas.gemm(hd, CUBLAS_OP_N, CUBLAS_OP_N, (int)N, (int)M, (int)K, &one, B, CUDA_R_16BF,
                                          (int)N, A, CUDA_R_16BF, (int)K, &zero, C, CUDA_R_16BF, (int)N,
                                          CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    return st == CUBLAS_STATUS_SUCCESS ? 0 : forge_fail(FORGE_KERNEL_UNSUPPORTED, "cublasGemmEx failed (%d)", (int)st);
}

// Row RMSNorm (reference _hx_cuda_kern_rmsnorm_mh, runtime_cuda_emit.hexa:
// 2748-2771, eps 1e-6): inv = 1/sqrt(sum(x^2)/d + eps), xn = x*inv,
// y = g*xn; optional outputs xn [T][d] and inv [T]. One CTA per row, fp32.
__global__ void __launch_bounds__(256) k_rmsnorm_bf16(const uint16_t* __restrict__ X, const uint16_t* __restrict__ G,
                                                      uint16_t* __restrict__ Y, uint16_t* __restrict__ XN,
                                                      uint16_t* __restrict__ I, int64_t d) {
    __shared__ float red[8];
    const int64_t row = blockIdx.x;
    const uint16_t* x = X + row * d;
    float ss = 0.f;
    for (int64_t c = threadIdx.x; c < d; c += 256) {
        const float v = bf16_bits_to_f32(x[c]);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    const float inv = 1.0f / sqrtf(tot / (float)d + 1e-6f);
    if (I && threadIdx.x == 0) I[row] = f32_to_bf16_bits(inv);
    for (int64_t c = threadIdx.x; c < d; c += 256) {
        const float xn = bf16_bits_to_f32(x[c]) * inv;
        if (XN) XN[row * d + c] = f32_to_bf16_bits(xn);
        Y[row * d + c] = f32_to_bf16_bits(bf16_bits_to_f32(G[c]) * xn);
    }
}

// O = (a * sigmoid(a)) * b (reference _hx_cuda_kern_silu_gate, :3033-3045).
__global__ void k_silu_gate_bf16(const uint16_t* __restrict__ A, const uint16_t* __restrict__ B,
                                 uint16_t* __restrict__ O, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float a = bf16_bits_to_f32(A[i]);
        const float sig = 1.0f / (1.0f + expf(-a));
        O[i] = f32_to_bf16_bits(__fmul_rn(__fmul_rn(a, sig), bf16_bits_to_f32(B[i])));
    }
}

// Rotate-half RoPE (reference _hx_cuda_kern_rope_fwd, :2232-2256):
// y[c] = x[c] cos[t][c] + rh(x)[c] sin[t][c], rh = [-x2, x1], two roundings
// (no fused multiply-add). X [T][nheads][hd], COS/SIN [T][hd].
__global__ void k_rope_bf16(const uint16_t* __restrict__ X, const uint16_t* __restrict__ COS,
                            const uint16_t* __restrict__ SIN, uint16_t* __restrict__ Y, int64_t T, int64_t nh,
                            int64_t hd) {
    const int64_t total = T * nh * hd, half = hd / 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = i % hd, row = i - c, t = i / (nh * hd);
        const float rh = c < half ? -bf16_bits_to_f32(X[row + half + c]) : bf16_bits_to_f32(X[row + c - half]);
        const float v = __fadd_rn(__fmul_rn(bf16_bits_to_f32(X[i]), bf16_bits_to_f32(COS[t * hd + c])),
                                  __fmul_rn(rh, bf16_bits_to_f32(SIN[t * hd + c])));
        Y[i] = f32_to_bf16_bits(v);
    }
}

int grid_for(int64_t n) {
    const int64_t g = (n + 255) / 256;
    const int64_t cap = (int64_t)forge_sm_count() * 8;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

// ---------------------------------------------------------------------------
// slot helpers
// ---------------------------------------------------------------------------
template <class T>
T* slot(const ForgeArgs* a, int i) {
    return (T*)(intptr_t)a->farr_ids[i];
}

// Device pointer of an operand descriptor holding at least `need` elements;
// uploads it when only its host copy is current.
const uint16_t* bf16_in(HexaFarrBf16* f, int64_t need) {
    if (!f || f->len < need) return nullptr;
    if (hexa_farr_bf16_to_device(f)) return nullptr;
    return (const uint16_t*)f->d_buf;
}
// Device pointer of a result descriptor (allocated on first use); the
// device copy becomes the authoritative one.
uint16_t* bf16_out(HexaFarrBf16* f, int64_t need) {
    if (!f || f->len < need) return nullptr;
    if (!f->d_buf) {
        if (cudaMalloc(&f->d_buf, (size_t)f->len * 2) != cudaSuccess) {
            cudaGetLastError();
            f->d_buf = nullptr;
            return nullptr;
        }
    }
    f->loc = FARR_BF16_LOC_DEVICE;
    return (uint16_t*)f->d_buf;
}
template <class F>
float* f32_dev(F* f, int64_t need, bool output) {
    if (!f || f->len < need) return nullptr;
    if (output) {
        if (!f->d_buf && cudaMalloc(&f->d_buf, (size_t)f->len * 4) != cudaSuccess) {
            cudaGetLastError();
            f->d_buf = nullptr;
            return nullptr;
        }
        f->loc = FARR_BF16_LOC_DEVICE;
        return (float*)f->d_buf;
    }
    if (hexa_farr_f32_to_device((HexaFarrF32*)f)) return nullptr;
    return (float*)f->d_buf;
}

int launched(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        forge_fail(FORGE_KERNEL_UNSUPPORTED, "%s: %s", what, cudaGetErrorString(e));
        return FORGE_KERNEL_UNSUPPORTED;
    }
    return FORGE_OK;
}

// ---- v1 families, PURE_BF16 ----------------------------------------------------
int v1_matmul(const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out) {
    if (in->count < 2 || out->count < 1 || s->M <= 0 || s->N <= 0 || s->K <= 0) return FORGE_INVALID_ARGS;
    const uint16_t* A = bf16_in(slot<HexaFarrBf16>(in, 0), s->M * s->K);
    const uint16_t* B = bf16_in(slot<HexaFarrBf16>(in, 1), s->K * s->N);
    uint16_t* C = bf16_out(slot<HexaFarrBf16>(out, 0), s->M * s->N);
    if (!A || !B || !C) return FORGE_INVALID_ARGS;
    if (matmul_bf16(A, B, C, s->M, s->N, s->K)) return FORGE_KERNEL_UNSUPPORTED;
    return launched("v1 MATMUL");
}

// FFN_FUSED: Y = SiLU(X W1) W2 with M = shape.M, D = shape.K, FD = shape.N
// (reference forge_tier_v1_emit.hexa:236-263); the hidden activation
// [M][FD] lives in a library-owned scratch grown on demand, as in the
// reference's hexa_farr_ffn_bf16_gpu (runtime_bf16_emit.hexa:543-640).
int v1_ffn(const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out) {
    if (in->count < 3 || out->count < 1 || s->M <= 0 || s->N <= 0 || s->K <= 0) return FORGE_INVALID_ARGS;
    const int64_t M = s->M, D = s->K, FD = s->N;
    const uint16_t* X = bf16_in(slot<HexaFarrBf16>(in, 0), M * D);
    const uint16_t* W1 = bf16_in(slot<HexaFarrBf16>(in, 1), D * FD);
    const uint16_t* W2 = bf16_in(slot<HexaFarrBf16>(in, 2), FD * D);
    uint16_t* Y = bf16_out(slot<HexaFarrBf16>(out, 0), M * D);
    if (!X || !W1 || !W2 || !Y) return FORGE_INVALID_ARGS;
    static std::mutex mu;
    static uint16_t* hbuf[64] = {nullptr};
    static size_t hbytes[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return FORGE_INVALID_ARGS;
    uint16_t* Hd = nullptr;
    {
        std::lock_guard<std::mutex> lk(mu);
        const size_t need = (size_t)(M * FD * 2);
        if (need > hbytes[dev]) {
            if (hbuf[dev]) cudaFree(hbuf[dev]);
            hbuf[dev] = nullptr;
            hbytes[dev] = 0;
            if (cudaMalloc(&hbuf[dev], need) != cudaSuccess) {
                cudaGetLastError();
                forge_fail(FORGE_KERNEL_UNSUPPORTED, "v1 FFN_FUSED: scratch of %zu bytes", need);
                return FORGE_KERNEL_UNSUPPORTED;
            }
            hbytes[dev] = need;
        }
        Hd = hbuf[dev];
    }
    if (matmul_bf16(X, W1, Hd, M, FD, D)) return FORGE_KERNEL_UNSUPPORTED;
    const int64_t nh = M * FD;
    k_silu_bf16_inplace<<<(unsigned)std::min<int64_t>((nh + 255) / 256, 4 * 148), 256>>>(Hd, nh);
    if (matmul_bf16(Hd, W2, Y, M, D, FD)) return FORGE_KERNEL_UNSUPPORTED;
    return launched("v1 FFN_FUSED");
}

// RMSNORM_MH: in = [X [T][d], G [d]], out = [Y [T][d], optional XN [T][d],
// optional inv-rms [T]]; T = shape.M, d = shape.K.
int v1_rmsnorm(const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out) {
    if (in->count < 2 || out->count < 1 || s->M <= 0 || s->K <= 0) return FORGE_INVALID_ARGS;
    const int64_t T = s->M, d = s->K;
    const uint16_t* X = bf16_in(slot<HexaFarrBf16>(in, 0), T * d);
    const uint16_t* G = bf16_in(slot<HexaFarrBf16>(in, 1), d);
    uint16_t* Y = bf16_out(slot<HexaFarrBf16>(out, 0), T * d);
    uint16_t* XN = out->count > 1 && out->farr_ids[1] ? bf16_out(slot<HexaFarrBf16>(out, 1), T * d) : nullptr;
    uint16_t* I = out->count > 2 && out->farr_ids[2] ? bf16_out(slot<HexaFarrBf16>(out, 2), T) : nullptr;
    if (!X || !G || !Y || (out->count > 1 && out->farr_ids[1] && !XN) || (out->count > 2 && out->farr_ids[2] && !I))
        return FORGE_INVALID_ARGS;
    if (T > 0x7FFFFFFF) return FORGE_INVALID_ARGS;
    k_rmsnorm_bf16<<<(unsigned)T, 256>>>(X, G, Y, XN, I, d);
    return launched("v1 RMSNORM_MH");
}

// SILU_GATE: in = [A, B], out = [O], n = shape.M * shape.N elements.
int v1_silu_gate(const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out) {
    if (in->count < 2 || out->count < 1 || s->M <= 0 || s->N <= 0) return FORGE_INVALID_ARGS;
    const int64_t n = s->M * s->N;
    const uint16_t* A = bf16_in(slot<HexaFarrBf16>(in, 0), n);
    const uint16_t* B = bf16_in(slot<HexaFarrBf16>(in, 1), n);
    uint16_t* O = bf16_out(slot<HexaFarrBf16>(out, 0), n);
    if (!A || !B || !O) return FORGE_INVALID_ARGS;
    k_silu_gate_bf16<<<grid_for(n), 256>>>(A, B, O, n);
    return launched("v1 SILU_GATE");
}

// ROPE_MH: in = [X [T][nheads][hd], COS [T][hd], SIN [T][hd]], out = [Y];
// T = shape.M, nheads = shape.N, hd = shape.K (even).
int v1_rope(const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out) {
    if (in->count < 3 || out->count < 1 || s->M <= 0 || s->N <= 0 || s->K <= 0 || (s->K & 1)) return FORGE_INVALID_ARGS;
    const int64_t T = s->M, nh = s->N, hd = s->K;
    const uint16_t* X = bf16_in(slot<HexaFarrBf16>(in, 0), T * nh * hd);
    const uint16_t* C = bf16_in(slot<HexaFarrBf16>(in, 1), T * hd);
    const uint16_t* S = bf16_in(slot<HexaFarrBf16>(in, 2), T * hd);
    uint16_t* Y = bf16_out(slot<HexaFarrBf16>(out, 0), T * nh * hd);
    if (!X || !C || !S || !Y) return FORGE_INVALID_ARGS;
    k_rope_bf16<<<grid_for(T * nh * hd), 256>>>(X, C, S, Y, T, nh, hd);
    return launched("v1 ROPE_MH");
}

// ---- registry (reference forge_tier_v1_emit.hexa:96-128) ---------------------
struct Reg {
    int family, precision, regime;
    ForgeShapeInfo shape;
    void* fn;
};
constexpr int kRegCap = 64;
Reg g_reg[kRegCap];
int g_reg_n = 0;
std::mutex g_reg_mu;

// ---- v2 ---------------------------------------------------------------------------
int v2_gemv(int family, const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out) {
    if (in->count < 2 || out->count < 1) return FORGE_INVALID_ARGS;
    HexaFarrW* W = slot<HexaFarrW>(in, 0);
    if (!W || !W->packed || W->kind != (family == FORGE_KERNEL_GEMV_W4A16_G128 ? HEXA_FARR_W_Q4_G128 : HEXA_FARR_W_BF16))
        return FORGE_INVALID_ARGS;
    const int64_t B = s->M > 0 ? s->M : 1;
    if ((s->N && s->N != W->rows) || (s->K && s->K != W->cols) || B > 1024) return FORGE_INVALID_ARGS;
    const float* X = f32_dev(slot<HexaFarrF32>(in, 1), B * W->cols, false);
    float* Y = f32_dev(slot<HexaFarrF32>(out, 0), B * W->rows, true);
    if (!X || !Y) return FORGE_INVALID_ARGS;
    const int rc = family == FORGE_KERNEL_GEMV_W4A16_G128
                       ? forge_gemv_w4a16_g128(W->d_tiles, W->d_scales, W->rows, W->cols, X, (int)B, Y, 1, nullptr)
                       : forge_gemv_bf16(W->d_tiles, W->rows, W->cols, X, (int)B, Y, B <= 4, nullptr);
    return rc ? FORGE_KERNEL_UNSUPPORTED : FORGE_OK;
}

int v2_flash_decode(const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out) {
    if (in->count < 3 || out->count < 1) return FORGE_INVALID_ARGS;
    HexaKvCache* kv = slot<HexaKvCache>(in, 1);
    const int64_t layer = in->farr_ids[2];
    if (!kv || layer < 0 || layer >= kv->n_layer) return FORGE_INVALID_ARGS;
    const int64_t B = s->M, H = s->N, hd = kv->head_dim;
    if (B <= 0 || B > kv->batch || H <= 0 || H % kv->n_kv_head || (s->K && s->K != hd)) return FORGE_INVALID_ARGS;
    const float* Q = f32_dev(slot<HexaFarrF32>(in, 0), B * H * hd, false);
    float* O = f32_dev(slot<HexaFarrF32>(out, 0), B * H * hd, true);
    if (!Q || !O) return FORGE_INVALID_ARGS;
    const size_t per_layer = (size_t)(kv->batch * kv->n_kv_head * kv->max_ctx * hd);
    const uint16_t* kc = (const uint16_t*)kv->d_k + per_layer * layer;
    const uint16_t* vc = (const uint16_t*)kv->d_v + per_layer * layer;
    // the cache's batch stride is kv->batch sequences; the kernel indexes
    // [B][Hkv][lmax][hd] from the layer base, so B <= kv->batch is enough.
    // The split partials live in a workspace this family owns per device
    // (never the allocation-free entry's shared array), and device errors
    // land in the per-op error word that forge_ops_check reads.
    const int64_t need = forge_flash_decode_workspace_bytes((int)B, (int)H, (int)kv->n_kv_head, (int)hd, (int)kv->max_ctx);
    if (need <= 0) return FORGE_INVALID_ARGS;
    static std::mutex mu;
    static void* ws[64] = {nullptr};
    static int64_t wsb[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return FORGE_INVALID_ARGS;
    std::lock_guard<std::mutex> lk(mu);
    if (need > wsb[dev]) {
        if (ws[dev]) cudaFree(ws[dev]);
        ws[dev] = nullptr;
        wsb[dev] = 0;
        if (cudaMalloc(&ws[dev], (size_t)need) != cudaSuccess || cudaMemset(ws[dev], 0, (size_t)need) != cudaSuccess) {
            cudaGetLastError();
            return FORGE_KERNEL_UNSUPPORTED;
        }
        wsb[dev] = need;
    }
    const int rc = forge_flash_decode(Q, kc, vc, kv->d_pos, (int)B, (int)H, (int)kv->n_kv_head, (int)hd,
                                      (int)kv->max_ctx, O, ws[dev], nullptr);
    return rc ? FORGE_KERNEL_UNSUPPORTED : FORGE_OK;
}

int v2_handle(int family, const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out) {
    ForgeB200* h = slot<ForgeB200>(in, 0);
    if (!h) return FORGE_INVALID_ARGS;
    const int B = (int)(s->batch > 0 ? s->batch : (s->M > 0 ? s->M : 1));
    int rc = 0;
    switch (family) {
        case FORGE_KERNEL_QKV_ROPE_FUSED:
        case FORGE_KERNEL_SWIGLU_FUSED: {
            if (in->count < 3 || out->count < 1) return FORGE_INVALID_ARGS;
            const int layer = (int)in->farr_ids[1];
            const int64_t nin = (int64_t)B * forge_b200_width(h, 0);
            const int64_t nout = (int64_t)B * forge_b200_width(h, family == FORGE_KERNEL_QKV_ROPE_FUSED ? 1 : 0);
            const float* x = f32_dev(slot<HexaFarrF32>(in, 2), nin, false);
            float* y = f32_dev(slot<HexaFarrF32>(out, 0), nout, true);
            if (!x || !y) return FORGE_INVALID_ARGS;
            rc = family == FORGE_KERNEL_QKV_ROPE_FUSED ? forge_b200_qkv_rope(h, layer, B, x, y)
                                                       : forge_b200_mlp(h, layer, B, x, y);
            break;
        }
        case FORGE_KERNEL_LMHEAD_ARGMAX: {
            if (in->count < 2 || out->count < 1) return FORGE_INVALID_ARGS;
            const float* x = f32_dev(slot<HexaFarrF32>(in, 1), (int64_t)B * forge_b200_width(h, 0), false);
            float* tok = f32_dev(slot<HexaFarrI32>(out, 0), B, true);
            float* logits = out->count > 1 && out->farr_ids[1]
                                ? f32_dev(slot<HexaFarrF32>(out, 1), (int64_t)B * forge_b200_width(h, 2), true)
                                : nullptr;
            if (!x || !tok || (out->count > 1 && out->farr_ids[1] && !logits)) return FORGE_INVALID_ARGS;
            rc = forge_b200_lm_head(h, B, x, (int32_t*)tok, logits);
            break;
        }
        case FORGE_KERNEL_DECODE_STEP: {
            if (in->count < 2 || out->count < 1) return FORGE_INVALID_ARGS;
            HexaFarrI32* T = slot<HexaFarrI32>(in, 1);
            HexaFarrI32* N = slot<HexaFarrI32>(out, 0);
            HexaFarrF32* Lg = out->count > 1 ? slot<HexaFarrF32>(out, 1) : nullptr;
            if (!T || !N || !T->h_buf || !N->h_buf || T->len < B || N->len < B || (Lg && !Lg->h_buf))
                return FORGE_INVALID_ARGS;
            rc = forge_b200_decode_step(h, B, (const int32_t*)T->h_buf, (int32_t*)N->h_buf,
                                        Lg ? (float*)Lg->h_buf : nullptr);
            if (!rc) {
                N->loc = FARR_BF16_LOC_HOST;
                if (Lg) Lg->loc = FARR_BF16_LOC_HOST;
            }
            break;
        }
        default:
            return FORGE_INVALID_ARGS;
    }
    return rc == FORGE_INVALID_ARGS ? FORGE_INVALID_ARGS : (rc ? FORGE_KERNEL_UNSUPPORTED : FORGE_OK);
}
}  // namespace

extern "C" {
FORGE_API uint32_t forge_api_version_v1(void) { return FORGE_API_VERSION_V1_ENCODED; }

FORGE_API int forge_register_specialized_v1(int kernel_family, const ForgeShapeInfo* shape, int precision_policy,
                                            int regime_hint, void* fn_ptr) {
    if (!shape || !fn_ptr) return FORGE_INVALID_ARGS;
    std::lock_guard<std::mutex> lk(g_reg_mu);
    if (g_reg_n >= kRegCap) return FORGE_INVALID_ARGS;
    g_reg[g_reg_n++] = Reg{kernel_family, precision_policy, regime_hint, *shape, fn_ptr};
    return FORGE_OK;
}

FORGE_API int forge_tier_dispatch_v1(int kernel_family, const ForgeShapeInfo* shape, int regime_hint,
                                     int precision_policy, int det_mode, const ForgeArgs* in, const ForgeArgs* out) {
    (void)regime_hint;
    if (det_mode == FORGE_DET_PEDANTIC && precision_policy != FORGE_PREC_FP64) return FORGE_PRECISION_UNSUPPORTED;
    if (precision_policy != FORGE_PREC_FP64 && precision_policy != FORGE_PREC_PURE_BF16 &&
        precision_policy != FORGE_PREC_LAYERCAST_BF16_FP32)
        return FORGE_PRECISION_UNSUPPORTED;
    if (kernel_family < FORGE_KERNEL_MATMUL || kernel_family > FORGE_KERNEL_ROPE_MH) return FORGE_INVALID_ARGS;
    if (!shape || !in || !out) return FORGE_INVALID_ARGS;
    if (precision_policy != FORGE_PREC_PURE_BF16) return FORGE_KERNEL_UNSUPPORTED;
    switch (kernel_family) {
        case FORGE_KERNEL_MATMUL: return v1_matmul(shape, in, out);
        case FORGE_KERNEL_FFN_FUSED: return v1_ffn(shape, in, out);
        case FORGE_KERNEL_RMSNORM_MH: return v1_rmsnorm(shape, in, out);
        case FORGE_KERNEL_SILU_GATE: return v1_silu_gate(shape, in, out);
        case FORGE_KERNEL_ROPE_MH: return v1_rope(shape, in, out);
        default: return FORGE_KERNEL_UNSUPPORTED;  // FWD_BWD_LINEAR, ATTN_DT_FWD/BWD
    }
}

FORGE_API int forge_tier_dispatch_v2(int kernel_family, const ForgeShapeInfo* shape, int regime_hint,
                                     int precision_policy, int det_mode, const ForgeArgs* in, const ForgeArgs* out) {
    if (kernel_family >= FORGE_KERNEL_MATMUL && kernel_family <= FORGE_KERNEL_ROPE_MH)
        return forge_tier_dispatch_v1(kernel_family, shape, regime_hint, precision_policy, det_mode, in, out);
    if (kernel_family < FORGE_KERNEL_GEMV_W4A16_G128 || kernel_family > FORGE_KERNEL_DECODE_STEP) return FORGE_INVALID_ARGS;
    if (det_mode == FORGE_DET_PEDANTIC) return FORGE_PRECISION_UNSUPPORTED;
    const int want = kernel_family == FORGE_KERNEL_GEMV_W4A16_G128 ? FORGE_PREC_W4A16_G128_BF16 : FORGE_PREC_PURE_BF16;
    const bool engine = kernel_family == FORGE_KERNEL_QKV_ROPE_FUSED || kernel_family == FORGE_KERNEL_SWIGLU_FUSED ||
                        kernel_family == FORGE_KERNEL_LMHEAD_ARGMAX || kernel_family == FORGE_KERNEL_DECODE_STEP;
    // the engine families take the handle's own weight kind, so either precision names them
    if (engine ? (precision_policy != FORGE_PREC_PURE_BF16 && precision_policy != FORGE_PREC_W4A16_G128_BF16)
               : precision_policy != want)
        return FORGE_PRECISION_UNSUPPORTED;
    if (!shape || !in || !out || in->count < 1 || in->count > 8 || out->count < 1 || out->count > 8)
        return FORGE_INVALID_ARGS;
    switch (kernel_family) {
        case FORGE_KERNEL_GEMV_W4A16_G128:
        case FORGE_KERNEL_GEMV_BF16: return v2_gemv(kernel_family, shape, in, out);
        case FORGE_KERNEL_FLASH_DECODE: return v2_flash_decode(shape, in, out);
        case FORGE_KERNEL_FLASH_PREFILL: return forge_prefill_dispatch(shape, in, out);
        default: return v2_handle(kernel_family, shape, in, out);
    }
}
}  // extern "C"
