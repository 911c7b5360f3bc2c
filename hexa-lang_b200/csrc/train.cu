// train.cu — the training-side forge families on B200, in float64 like the
// reference (self/cuda/runtime_cuda_emit.hexa): RMSNorm rows and its
// backward, AdamW, RoPE forward / backward, SiLU / its derivative / the SiLU
// gate, and causal GQA attention forward / backward with the probabilities
// materialised. Caller-owned device arrays, stream-ordered, 0 / error code.
//
// Every output keeps the reference's order of operations: products and sums
// with explicit round-to-nearest intrinsics (no FMA contraction), sums over j
// or c strictly ascending inside one thread, flame's own series for exp and
// sqrt where the reference uses them (dt_exp: range reduction by halving to
// |x| <= 1/4, 12 Taylor terms, squaring back; dt_sqrt, for the attention
// scale 1 / sqrt(hd) computed on the host: 24 Newton steps from max(x, 1)). Parallelism comes from spreading independent outputs over
// threads and warps, not from splitting a sum, so results equal a sequential
// float64 restatement bit for bit — except RMSNorm's two row reductions,
// which are block trees as in the reference kernels (last-bit differences).
#include <cmath>
#include "common.cuh"
#include "forge_internal.h"
#include "../../include/forge_b200.h"

namespace {
constexpr int kRowThreads = 256;

__device__ __forceinline__ double dt_exp(double x) {
    int r = 0;
    double xr = x;
    while ((xr > 0.0 ? xr : 0.0 - xr) > 0.25) {
        xr = xr / 2.0;
        ++r;
    }
    double term = 1.0, acc = 1.0;
    for (int k = 1; k < 12; ++k) {
        term = __ddiv_rn(__dmul_rn(term, xr), (double)k);
        acc = __dadd_rn(acc, term);
    }
    for (int s = 0; s < r; ++s) acc = __dmul_rn(acc, acc);
    return acc;
}

// Sum over a block of kRowThreads: warp shuffles, then warp 0 over the warp sums.
__device__ double block_sum(double v, double* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    double t = 0.0;
    if (w == 0) {
        t = l < kRowThreads / 32 ? red[l] : 0.0;
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (l == 0) red[kRowThreads / 32] = t;
    }
    __syncthreads();
    return red[kRowThreads / 32];
}

// y = x / sqrt(mean(x^2) + eps), one block per row (_hx_k_rmsnorm_rows).
__global__ void __launch_bounds__(kRowThreads) k_rmsnorm_rows(const double* __restrict__ X, double* __restrict__ Y,
                                                              int64_t C, double eps) {
    __shared__ double red[kRowThreads / 32 + 1];
    const double* xr = X + (size_t)blockIdx.x * C;
    double* yr = Y + (size_t)blockIdx.x * C;
    double v = 0.0;
    for (int64_t j = threadIdx.x; j < C; j += kRowThreads) v += xr[j] * xr[j];
    const double ms = block_sum(v, red) / (double)C;
    const double inv = 1.0 / sqrt(ms + eps);
    for (int64_t j = threadIdx.x; j < C; j += kRowThreads) yr[j] = xr[j] * inv;
}

// dx = inv*dxn - (inv^3 x / C) * dot(dxn, x), eps 1e-6 (_hx_k_rmsnorm_bwd_rows).
__global__ void __launch_bounds__(kRowThreads) k_rmsnorm_bwd_rows(const double* __restrict__ X,
                                                                  const double* __restrict__ DXN,
                                                                  double* __restrict__ O, int64_t C) {
    __shared__ double red[kRowThreads / 32 + 1];
    const size_t base = (size_t)blockIdx.x * C;
    double ssq = 0.0, dot = 0.0;
    for (int64_t j = threadIdx.x; j < C; j += kRowThreads) {
        const double x = X[base + j];
        ssq += x * x;
        dot += DXN[base + j] * x;
    }
    const double ms = block_sum(ssq, red) / (double)C;
    const double d = block_sum(dot, red);
    const double inv = 1.0 / sqrt(ms + 1e-6);
    const double coef = (inv * inv * inv) / (double)C;
    for (int64_t i = threadIdx.x; i < C; i += kRowThreads) O[base + i] = inv * DXN[base + i] - coef * X[base + i] * d;
}

// Decoupled-weight-decay AdamW, in place on m and v; out may be w
// (_hx_k_adamw_step / _inplace), no contraction.
__global__ void k_adamw(double* __restrict__ W, double* __restrict__ Mm, double* __restrict__ Vv,
                        const double* __restrict__ G, double* O, int64_t n, double lr, double b1, double b2,
                        double eps, double wd, double c1, double c2) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const double g = G[i], w = W[i];
        const double mi = __dadd_rn(__dmul_rn(b1, Mm[i]), __dmul_rn(1.0 - b1, g));
        const double vi = __dadd_rn(__dmul_rn(b2, Vv[i]), __dmul_rn(__dmul_rn(1.0 - b2, g), g));
        const double mhat = __ddiv_rn(mi, c1), vhat = __ddiv_rn(vi, c2);
        const double denom = __dadd_rn(sqrt(vhat), eps);
        const double wi = __dsub_rn(__dsub_rn(w, __dmul_rn(__dmul_rn(lr, wd), w)), __ddiv_rn(__dmul_rn(lr, mhat), denom));
        Mm[i] = mi;
        Vv[i] = vi;
        O[i] = wi;
    }
}

// Rotate-half RoPE on [T][nheads][hd] with tables [T][hd]
// (_hx_cuda_kern_rope_fwd / _bwd, nn_lib.hexa:541-562 and its transpose).
__global__ void k_rope(const double* __restrict__ X, const double* __restrict__ COS, const double* __restrict__ SIN,
                       double* __restrict__ Y, int64_t T, int64_t nheads, int64_t hd, int bwd) {
    const int64_t total = T * nheads * hd, half = hd / 2;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t c = i % hd, row = i - c, t = i / (nheads * hd), bse = t * hd;
        if (!bwd) {
            const double rh = c < half ? 0.0 - X[row + half + c] : X[row + c - half];
            Y[i] = __dadd_rn(__dmul_rn(X[row + c], COS[bse + c]), __dmul_rn(rh, SIN[bse + c]));
        } else {
            const double gs = c < half ? __dmul_rn(X[row + half + c], SIN[bse + half + c])
                                       : 0.0 - __dmul_rn(X[row + c - half], SIN[bse + c - half]);
            Y[i] = __dadd_rn(__dmul_rn(X[row + c], COS[bse + c]), gs);
        }
    }
}

// mode 0: silu(x) = x / (1 + exp(-x)); 1: its derivative s (1 + x (1 - s));
// 2: the gate silu(a) * b with flame's dt_exp (_hx_cuda_kern_silu[_grad|_gate]).
__global__ void k_silu(const double* __restrict__ A, const double* __restrict__ Bv, double* __restrict__ O,
                       int64_t n, int mode) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const double x = A[i];
        if (mode == 0) {
            O[i] = x * (1.0 / (1.0 + exp(-x)));
        } else if (mode == 1) {
            const double s = 1.0 / (1.0 + exp(-x));
            O[i] = s * (1.0 + x * (1.0 - s));
        } else {
            const double sig = 1.0 / (1.0 + dt_exp(0.0 - x));
            O[i] = __dmul_rn(__dmul_rn(x, sig), Bv[i]);
        }
    }
}

// Causal GQA attention forward with the probabilities kept
// (_hx_cuda_kern_attn_dt_fwd): one warp per (head, query row i); lanes take
// keys j (each dot product over c sequential), the row's maximum by
// shuffles (exact), exponentials per key, the row sum sequential on lane 0,
// then lanes take value dims c2 (each sum over j sequential).
__global__ void k_attn_fwd(const double* __restrict__ Q, const double* __restrict__ K, const double* __restrict__ V,
                           double* __restrict__ P, double* __restrict__ CTX, int64_t T, int64_t nh, int64_t nkv,
                           int64_t hd, double scale) {
    const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= nh * T) return;
    const int64_t hh = wid / T, i = wid % T, kvh = hh / (nh / nkv), L = i + 1, d = nh * hd;
    double* pr = P + (hh * T + i) * T;
    for (int64_t j = lane; j < T; j += 32) {
        if (j >= L) { pr[j] = 0.0; continue; }
        double dot = 0.0;
        for (int64_t c = 0; c < hd; ++c) dot = __dadd_rn(dot, __dmul_rn(Q[(i * nh + hh) * hd + c], K[(j * nkv + kvh) * hd + c]));
        pr[j] = __dmul_rn(dot, scale);
    }
    __syncwarp();
    double mx = -INFINITY;
    for (int64_t j = lane; j < L; j += 32) mx = fmax(mx, pr[j]);
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int64_t j = lane; j < L; j += 32) pr[j] = dt_exp(pr[j] - mx);
    __syncwarp();
    double tot = 0.0;
    if (lane == 0)
        for (int64_t j = 0; j < L; ++j) tot = __dadd_rn(tot, pr[j]);
    tot = __shfl_sync(0xffffffffu, tot, 0);
    for (int64_t j = lane; j < L; j += 32) pr[j] = __ddiv_rn(pr[j], tot);
    __syncwarp();
    for (int64_t c2 = lane; c2 < hd; c2 += 32) {
        double acc = 0.0;
        for (int64_t j = 0; j < L; ++j) acc = __dadd_rn(acc, __dmul_rn(pr[j], V[(j * nkv + kvh) * hd + c2]));
        CTX[i * d + hh * hd + c2] = acc;
    }
}

// Backward step 1: dP_row[hh, i, j] = sum_c dctx[i, hh, c] V[j, kvh, c], j <= i.
__global__ void k_attn_bwd_dprow(const double* __restrict__ V, const double* __restrict__ DCTX,
                                 double* __restrict__ DP, int64_t T, int64_t nh, int64_t nkv, int64_t hd) {
    const int64_t total = nh * T * T, stride = (int64_t)gridDim.x * blockDim.x, d = nh * hd;
    for (int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; f < total; f += stride) {
        const int64_t hh = f / (T * T), r = f - hh * T * T, i = r / T, j = r - i * T;
        if (j > i) { DP[f] = 0.0; continue; }
        const int64_t kvh = hh / (nh / nkv);
        double acc = 0.0;
        for (int64_t c = 0; c < hd; ++c) acc = __dadd_rn(acc, __dmul_rn(DCTX[i * d + hh * hd + c], V[(j * nkv + kvh) * hd + c]));
        DP[f] = acc;
    }
}

// Backward step 2, one warp per (hh, i): sdot = sum_j P dP_row (lane 0,
// sequential), dS = P (dP_row - sdot) scale in place, then lanes over c2:
// dQ[i, hh, c2] = sum_j dS K[j, kvh, c2].
__global__ void k_attn_bwd_ds_dq(const double* __restrict__ K, const double* __restrict__ P, double* __restrict__ DP,
                                 double* __restrict__ DQ, int64_t T, int64_t nh, int64_t nkv, int64_t hd, double scale) {
    const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= nh * T) return;
    const int64_t hh = wid / T, i = wid % T, kvh = hh / (nh / nkv), L = i + 1;
    const double* pr = P + (hh * T + i) * T;
    double* dr = DP + (hh * T + i) * T;
    double sdot = 0.0;
    if (lane == 0)
        for (int64_t j = 0; j < L; ++j) sdot = __dadd_rn(sdot, __dmul_rn(pr[j], dr[j]));
    sdot = __shfl_sync(0xffffffffu, sdot, 0);
    for (int64_t j = lane; j < L; j += 32) dr[j] = __dmul_rn(__dmul_rn(pr[j], dr[j] - sdot), scale);
    __syncwarp();
    for (int64_t c2 = lane; c2 < hd; c2 += 32) {
        double acc = 0.0;
        for (int64_t j = 0; j < L; ++j) acc = __dadd_rn(acc, __dmul_rn(dr[j], K[(j * nkv + kvh) * hd + c2]));
        DQ[(i * nh + hh) * hd + c2] = acc;
    }
}

// Backward step 3: per (j, kvh, c), over the group's heads then i >= j:
// which 0: dV = sum P dctx; 1: dK = sum dS Q.
__global__ void k_attn_bwd_dkv(const double* __restrict__ A, const double* __restrict__ Bm, double* __restrict__ O,
                               int64_t T, int64_t nh, int64_t nkv, int64_t hd, int which) {
    const int64_t total = T * nkv * hd, stride = (int64_t)gridDim.x * blockDim.x, n_rep = nh / nkv, d = nh * hd;
    for (int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; f < total; f += stride) {
        const int64_t j = f / (nkv * hd), r = f - j * (nkv * hd), kvh = r / hd, c = r - kvh * hd;
        double acc = 0.0;
        for (int64_t hh = kvh * n_rep; hh < (kvh + 1) * n_rep; ++hh)
            for (int64_t i = j; i < T; ++i) {
                const double b = which == 0 ? Bm[i * d + hh * hd + c] : Bm[(i * nh + hh) * hd + c];
                acc = __dadd_rn(acc, __dmul_rn(A[(hh * T + i) * T + j], b));
            }
        O[(j * nkv + kvh) * hd + c] = acc;
    }
}

int grid_for(int64_t n, int threads) {
    const int64_t g = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)forge_sm_count() * 16;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}
int done(const char* what) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : forge_fail(-1, "%s: %s", what, cudaGetErrorString(e));
}
}  // namespace

extern "C" {
FORGE_API int forge_train_rmsnorm_rows(const double* x, int64_t R, int64_t C, double eps, double* y, void* stream) {
    if (!x || !y || R <= 0 || C <= 0 || R > INT32_MAX || !(eps >= 0.0))
        return forge_fail(FORGE_INVALID_ARGS, "forge_train_rmsnorm_rows: bad args");
    k_rmsnorm_rows<<<(unsigned)R, kRowThreads, 0, (cudaStream_t)stream>>>(x, y, C, eps);
    return done("forge_train_rmsnorm_rows");
}

FORGE_API int forge_train_rmsnorm_bwd_rows(const double* x, const double* dxn, int64_t R, int64_t C, double* dx,
                                           void* stream) {
    if (!x || !dxn || !dx || R <= 0 || C <= 0 || R > INT32_MAX)
        return forge_fail(FORGE_INVALID_ARGS, "forge_train_rmsnorm_bwd_rows: bad args");
    k_rmsnorm_bwd_rows<<<(unsigned)R, kRowThreads, 0, (cudaStream_t)stream>>>(x, dxn, dx, C);
    return done("forge_train_rmsnorm_bwd_rows");
}

FORGE_API int forge_train_adamw_step(double* w, double* m, double* v, const double* g, int64_t n, double lr, double b1,
                                     double b2, double eps, double wd, int64_t step_t, double* out, void* stream) {
    if (!w || !m || !v || !g || !out || n <= 0 || step_t < 1)
        return forge_fail(FORGE_INVALID_ARGS, "forge_train_adamw_step: bad args");
    // bias corrections by repeated multiplication, as the reference host code
    double b1t = 1.0, b2t = 1.0;
    for (int64_t e = 0; e < step_t; ++e) {
        b1t *= b1;
        b2t *= b2;
    }
    k_adamw<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(w, m, v, g, out, n, lr, b1, b2, eps, wd, 1.0 - b1t,
                                                                 1.0 - b2t);
    return done("forge_train_adamw_step");
}

FORGE_API int forge_train_rope(const double* t, const double* cos_t, const double* sin_t, int64_t T, int64_t nheads,
                               int64_t hd, int bwd, double* out, void* stream) {
    if (!t || !cos_t || !sin_t || !out || T <= 0 || nheads <= 0 || hd <= 0 || (hd & 1))
        return forge_fail(FORGE_INVALID_ARGS, "forge_train_rope: bad args");
    k_rope<<<grid_for(T * nheads * hd, 256), 256, 0, (cudaStream_t)stream>>>(t, cos_t, sin_t, out, T, nheads, hd, bwd);
    return done("forge_train_rope");
}

FORGE_API int forge_train_silu(const double* x, const double* gate_b, int64_t n, int mode, double* out, void* stream) {
    if (!x || !out || n <= 0 || mode < 0 || mode > 2 || (mode == 2 && !gate_b))
        return forge_fail(FORGE_INVALID_ARGS, "forge_train_silu: bad args");
    k_silu<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(x, gate_b, out, n, mode);
    return done("forge_train_silu");
}

FORGE_API int forge_train_attn_fwd(const double* q, const double* k, const double* v, int64_t T, int64_t nh,
                                   int64_t nkv, int64_t hd, double* p, double* ctx, void* stream) {
    if (!q || !k || !v || !p || !ctx || T <= 0 || nh <= 0 || nkv <= 0 || nh % nkv || hd <= 0)
        return forge_fail(FORGE_INVALID_ARGS, "forge_train_attn_fwd: bad args");
    // scale = 1 / dt_sqrt(hd), computed on the host with the same steps
    double g = (double)hd > 1.0 ? (double)hd : 1.0;
    for (int i = 0; i < 24; ++i) g = 0.5 * (g + (double)hd / g);
    const double sc = 1.0 / g;
    const int64_t warps = nh * T;
    k_attn_fwd<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(q, k, v, p, ctx, T, nh, nkv, hd, sc);
    return done("forge_train_attn_fwd");
}

FORGE_API int forge_train_attn_bwd(const double* q, const double* k, const double* v, const double* p,
                                   const double* dctx, int64_t T, int64_t nh, int64_t nkv, int64_t hd, double* dq,
                                   double* dk, double* dv, double* scratch, void* stream) {
    if (!q || !k || !v || !p || !dctx || !dq || !dk || !dv || !scratch || T <= 0 || nh <= 0 || nkv <= 0 ||
        nh % nkv || hd <= 0)
        return forge_fail(FORGE_INVALID_ARGS, "forge_train_attn_bwd: bad args");
    cudaStream_t st = (cudaStream_t)stream;
    double g = (double)hd > 1.0 ? (double)hd : 1.0;
    for (int i = 0; i < 24; ++i) g = 0.5 * (g + (double)hd / g);
    const double sc = 1.0 / g;
    k_attn_bwd_dprow<<<grid_for(nh * T * T, 256), 256, 0, st>>>(v, dctx, scratch, T, nh, nkv, hd);
    k_attn_bwd_ds_dq<<<(unsigned)((nh * T * 32 + 255) / 256), 256, 0, st>>>(k, p, scratch, dq, T, nh, nkv, hd, sc);
    k_attn_bwd_dkv<<<grid_for(T * nkv * hd, 256), 256, 0, st>>>(p, dctx, dv, T, nh, nkv, hd, 0);
    k_attn_bwd_dkv<<<grid_for(T * nkv * hd, 256), 256, 0, st>>>(scratch, q, dk, T, nh, nkv, hd, 1);
    return done("forge_train_attn_bwd");
}
}  // extern "C"
