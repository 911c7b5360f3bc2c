// sample.cu — token sampling on the device: temperature, softmax, top-k,
// top-p and the multinomial draw of self/ml/gpu_sampler.hexa:89-277, for a
// batch of sequences, one CTA per sequence.
//
// The reference copies the logits to the host and runs every step there in
// f64 with f32 storage. Here the logits stay in HBM and only the token (and
// the RNG state) leave the device. Arithmetic follows the reference's
// roundings — f64 products and exponentials, each stored value rounded to
// f32, f64 sums — but sums are reduced in parallel, so a sum can differ from
// the reference's left-to-right sum in its last f64 bit; a token differs only
// when the draw lands within that distance of a cumulative boundary.
//
// Each thread owns a contiguous slice of the vocabulary, so "first index"
// rules (argmax ties, the first running sum above the draw) and index-order
// tie ranks are block scans over thread slices.
//
//   top-k   the k-th largest probability by a 4-pass radix select on the f32
//           bit pattern (8 bits a pass); entries below it are zeroed, ties
//           with it kept, as the reference's partial selection sort does.
//   top-p   the boundary probability by the same radix descent with a count
//           and a sum per bucket: the largest value t such that the
//           entries above t sum to less than p and those at or above t reach
//           it. Entries equal to t are kept in index order until the running
//           sum reaches p (the reference orders equal entries by the swaps
//           of its selection sort; the two differ only when several entries
//           share the boundary value and not all of them are kept). The
//           bucket sums are accumulated as 64-bit fixed-point integers (each
//           probability times 2^62, rounded): integer additions commute, so
//           the boundary is the same on every run for the same logits,
//           whatever order the threads' atomic additions land in.
//   draw    the reference's Xorshift-style RNG (gpu_sampler.hexa:57-65) on
//           a 64-bit state per sequence, in device memory.
#include <climits>
#include <cmath>
#include "common.cuh"
#include "forge_internal.h"
#include "../../include/forge_b200.h"

namespace {
constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

struct SampleArgs {
    const float* logits;
    int64_t ld;        // logits row stride (floats)
    int V;
    double temperature, top_p;
    int top_k;
    int64_t* rng;      // [B] states
    float* probs;      // [B][pld] working / final distribution
    int64_t pld;
    int32_t* out;      // [B] tokens
};

__device__ __forceinline__ double sampler_rand(int64_t* state) {
    int64_t x = *state;
    x = x ^ (int64_t)((uint64_t)x * 8192u);
    x = x ^ (x / 131072);
    x = x ^ (int64_t)((uint64_t)x * 32u);
    if (x < 0) x = (int64_t)(0u - (uint64_t)x);
    *state = x;
    return (double)(x % 1000000) / 1000000.0;
}

struct Shared {
    double red_d[kWarps];
    float red_f[kWarps];
    long long red_l[kWarps];
    int hist[256];
    unsigned long long hsum[256];  // fixed point, 2^-62 units
    double bcast_d[2];
    int bcast_i[4];
};

// Probability (0 <= v <= 1, sums to ~1) in 64-bit fixed point, 2^-62 units.
__device__ __forceinline__ unsigned long long fx62(float v) {
    return (unsigned long long)llrint((double)v * 0x1p62);
}
__device__ __forceinline__ double fx62_to_f64(unsigned long long x) { return (double)x * 0x1p-62; }

__device__ double block_sum(double v, Shared& sh) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh.red_d[w] = v;
    __syncthreads();
    double t = 0.0;
    if (w == 0) {
        t = l < kWarps ? sh.red_d[l] : 0.0;
        for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (l == 0) sh.bcast_d[0] = t;
    }
    __syncthreads();
    return sh.bcast_d[0];
}

// max over non-NaN values (-inf when none)
__device__ float block_max(float v, Shared& sh) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh.red_f[w] = v;
    __syncthreads();
    if (w == 0) {
        float t = l < kWarps ? sh.red_f[l] : -INFINITY;
        for (int o = 16; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
        if (l == 0) sh.bcast_d[1] = t;
    }
    __syncthreads();
    return (float)sh.bcast_d[1];
}

__device__ long long block_min_ll(long long v, Shared& sh) {
    for (int o = 16; o; o >>= 1) {
        const long long u = __shfl_xor_sync(0xffffffffu, v, o);
        v = u < v ? u : v;
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh.red_l[w] = v;
    __syncthreads();
    if (w == 0) {
        long long t = l < kWarps ? sh.red_l[l] : LLONG_MAX;
        for (int o = 16; o; o >>= 1) {
            const long long u = __shfl_xor_sync(0xffffffffu, t, o);
            t = u < t ? u : t;
        }
        if (l == 0) sh.red_l[0] = t;
    }
    __syncthreads();
    const long long r = sh.red_l[0];
    __syncthreads();
    return r;
}

// exclusive prefix over threads in index order (f64); total in *tot
__device__ double block_exclusive_scan(double v, Shared& sh, double* tot) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    double inc = v;
    for (int o = 1; o < 32; o <<= 1) {
        const double u = __shfl_up_sync(0xffffffffu, inc, o);
        if (l >= o) inc += u;
    }
    __syncthreads();
    if (l == 31) sh.red_d[w] = inc;
    __syncthreads();
    if (w == 0) {
        double t = l < kWarps ? sh.red_d[l] : 0.0, ti = t;
        for (int o = 1; o < 32; o <<= 1) {
            const double u = __shfl_up_sync(0xffffffffu, ti, o);
            if (l >= o) ti += u;
        }
        if (l < kWarps) sh.red_d[l] = ti - t;  // exclusive warp offsets
        if (l == kWarps - 1) sh.bcast_d[0] = ti;
    }
    __syncthreads();
    const double r = sh.red_d[w] + inc - v;
    if (tot) *tot = sh.bcast_d[0];
    __syncthreads();
    return r;
}

// 4-pass radix select over the f32 bit patterns of the non-negative values
// p[i0..i1) of every thread: the k-th largest (1-based), with multiplicity.
__device__ uint32_t radix_kth_largest(const float* p, int i0, int i1, int k, Shared& sh) {
    uint32_t prefix = 0, mask = 0;
    int kk = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int j = threadIdx.x; j < 256; j += kThreads) sh.hist[j] = 0;
        __syncthreads();
        for (int i = i0; i < i1; ++i) {
            const uint32_t u = __float_as_uint(p[i]);
            if ((u & mask) == prefix) atomicAdd(&sh.hist[(u >> shift) & 255u], 1);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int j = 255;
            for (; j > 0; --j) {
                if (kk <= sh.hist[j]) break;
                kk -= sh.hist[j];
            }
            sh.bcast_i[0] = j;
            sh.bcast_i[1] = kk;
        }
        __syncthreads();
        prefix |= (uint32_t)sh.bcast_i[0] << shift;
        kk = sh.bcast_i[1];
        mask |= 255u << shift;
        __syncthreads();
    }
    return prefix;
}

__global__ void __launch_bounds__(kThreads, 1) k_sample(const SampleArgs a) {
    __shared__ Shared sh;
    const int b = blockIdx.x;
    const float* lg = a.logits + (int64_t)b * a.ld;
    float* p = a.probs + (int64_t)b * a.pld;
    const int V = a.V;
    const int chunk = (V + kThreads - 1) / kThreads;
    const int i0 = min(V, (int)threadIdx.x * chunk), i1 = min(V, i0 + chunk);

    if (a.temperature <= 0.0) {
        // first maximum (gpu_sampler.hexa:70-85); a NaN first entry wins
        long long key = LLONG_MAX;
        if (!isnan(lg[0])) {
            float bv = -INFINITY;
            int bi = V;
            for (int i = i0; i < i1; ++i)
                if (lg[i] > bv) { bv = lg[i]; bi = i; }
            const float m = block_max(bv, sh);
            key = (bi < V && bv == m) ? bi : LLONG_MAX;
        }
        key = block_min_ll(key, sh);
        if (threadIdx.x == 0) a.out[b] = key == LLONG_MAX ? 0 : (int32_t)key;
        return;
    }

    // temperature, max, exp, normalise
    const double inv_t = 1.0 / a.temperature;
    float lm = -INFINITY;
    for (int i = i0; i < i1; ++i) {
        const float s = (float)((double)lg[i] * inv_t);
        p[i] = s;
        lm = fmaxf(lm, s);
    }
    float mxf = block_max(lm, sh);
    if (isnan((float)((double)lg[0] * inv_t))) mxf = NAN;  // the reference starts from entry 0
    const double mx = mxf;
    double ls = 0.0;
    for (int i = i0; i < i1; ++i) {
        const double e = exp((double)p[i] - mx);
        p[i] = (float)e;
        ls += e;
    }
    const double inv_sum = 1.0 / block_sum(ls, sh);
    for (int i = i0; i < i1; ++i) p[i] = (float)((double)p[i] * inv_sum);
    __syncthreads();

    if (a.top_k > 0 && a.top_k < V) {
        const float thr = __uint_as_float(radix_kth_largest(p, i0, i1, a.top_k, sh));
        double lk = 0.0;
        for (int i = i0; i < i1; ++i) {
            if (p[i] < thr) p[i] = 0.0f;
            else lk += (double)p[i];
        }
        const double sum_k = block_sum(lk, sh);
        if (sum_k > 0.0) {
            const double inv_k = 1.0 / sum_k;
            for (int i = i0; i < i1; ++i) p[i] = (float)((double)p[i] * inv_k);
        }
        __syncthreads();
    }

    if (a.top_p < 1.0 && a.top_p > 0.0) {
        // radix descent for the boundary value t (see the file comment)
        uint32_t prefix = 0, mask = 0;
        double above = 0.0;
        bool all = false;
        int cnt_t = 0;
        for (int shift = 24; shift >= 0 && !all; shift -= 8) {
            for (int j = threadIdx.x; j < 256; j += kThreads) {
                sh.hist[j] = 0;
                sh.hsum[j] = 0ull;
            }
            __syncthreads();
            for (int i = i0; i < i1; ++i) {
                const float v = p[i];
                const uint32_t u = __float_as_uint(v);
                if (v > 0.0f && (u & mask) == prefix) {
                    atomicAdd(&sh.hist[(u >> shift) & 255u], 1);
                    atomicAdd(&sh.hsum[(u >> shift) & 255u], fx62(v));
                }
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                int pick = -1, lowest = -1;
                double acc = above;
                for (int j = 255; j >= 0; --j) {
                    if (!sh.hist[j]) continue;
                    lowest = j;
                    const double hs = fx62_to_f64(sh.hsum[j]);
                    if (acc + hs >= a.top_p) { pick = j; break; }
                    acc += hs;
                }
                int allf = 0;
                if (pick < 0) {
                    if (shift == 24 || lowest < 0) {
                        allf = 1;  // the nonzero entries never reach p: keep them all
                    } else {       // rounding between levels: the smallest nonempty bucket
                        pick = lowest;
                        acc -= fx62_to_f64(sh.hsum[lowest]);
                    }
                }
                sh.bcast_i[0] = pick;
                sh.bcast_i[1] = allf;
                sh.bcast_i[2] = pick >= 0 ? sh.hist[pick] : 0;
                sh.bcast_d[0] = acc;
            }
            __syncthreads();
            all = sh.bcast_i[1] != 0;
            if (!all) {
                prefix |= (uint32_t)sh.bcast_i[0] << shift;
                mask |= 255u << shift;
                above = sh.bcast_d[0];
                cnt_t = sh.bcast_i[2];
            }
            __syncthreads();
        }
        if (!all) {
            const float t = __uint_as_float(prefix);
            // entries equal to t kept, in index order, until the sum reaches p
            int m = 0;
            double cum = above;
            while (m < cnt_t) {
                cum += (double)t;
                ++m;
                if (cum >= a.top_p) break;
            }
            int mine = 0;
            for (int i = i0; i < i1; ++i) mine += p[i] == t;
            int rank = (int)block_exclusive_scan((double)mine, sh, nullptr);
            double lp = 0.0;
            for (int i = i0; i < i1; ++i) {
                const float v = p[i];
                bool keep = v > t;
                if (v == t) keep = rank++ < m;
                if (keep) lp += (double)v;
                else p[i] = 0.0f;
            }
            const double sum_p = block_sum(lp, sh);
            if (sum_p > 0.0) {
                const double inv_p = 1.0 / sum_p;
                for (int i = i0; i < i1; ++i) p[i] = (float)((double)p[i] * inv_p);
            }
        } else {
            double lp = 0.0;
            for (int i = i0; i < i1; ++i) lp += p[i] > 0.0f ? (double)p[i] : 0.0;
            const double sum_p = block_sum(lp, sh);
            if (sum_p > 0.0) {
                const double inv_p = 1.0 / sum_p;
                for (int i = i0; i < i1; ++i) p[i] = (float)((double)p[i] * inv_p);
            }
        }
        __syncthreads();
    }

    // multinomial draw: first index whose running sum exceeds r
    if (threadIdx.x == 0) {
        int64_t st = a.rng[b];
        sh.bcast_d[1] = sampler_rand(&st);
        a.rng[b] = st;
    }
    __syncthreads();
    const double r = sh.bcast_d[1];
    double mine = 0.0;
    for (int i = i0; i < i1; ++i) mine += (double)p[i];
    double c = block_exclusive_scan(mine, sh, nullptr);
    long long cand = LLONG_MAX;
    for (int i = i0; i < i1; ++i) {
        c += (double)p[i];
        if (c > r) {
            cand = i;
            break;
        }
    }
    cand = block_min_ll(cand, sh);
    if (threadIdx.x == 0) a.out[b] = cand == LLONG_MAX ? V - 1 : (int32_t)cand;
}
}  // namespace

int forge_sample_launch(const float* logits, int64_t ld, int batch, int vocab, double temperature, int top_k,
                        double top_p, int64_t* rng_state, float* probs, int64_t pld, int32_t* tokens,
                        cudaStream_t stream) {
    if (!logits || !probs || !tokens || batch <= 0 || vocab <= 0 || ld < vocab || pld < vocab ||
        (temperature > 0.0 && !rng_state))
        return forge_fail(FORGE_INVALID_ARGS, "forge_sample: bad arguments (batch %d vocab %d)", batch, vocab);
    SampleArgs a{logits, ld, vocab, temperature, top_p, top_k, rng_state, probs, pld, tokens};
    k_sample<<<batch, kThreads, 0, stream>>>(a);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : forge_fail(-1, "forge_sample: launch failed: %s", cudaGetErrorString(e));
}

extern "C" FORGE_API int forge_sample(const float* logits, int64_t ld, int batch, int vocab, double temperature,
                                      int top_k, double top_p, int64_t* rng_state, float* probs, int32_t* tokens,
                                      void* stream) {
    return forge_sample_launch(logits, ld, batch, vocab, temperature, top_k, top_p, rng_state, probs, vocab, tokens,
                               (cudaStream_t)stream);
}
