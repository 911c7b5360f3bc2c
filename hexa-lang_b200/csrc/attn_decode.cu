// attn_decode.cu — split-K flash-decode over a contiguous bf16 KV cache.
//
// Single-query causal GQA attention for every sequence of the decode batch
// (nn_attn_core_fwd, nn_lib.hexa:221-278, row i = current position), split
// along the KV axis with per-split (m, l, O) partials and a log-sum-exp merge
// (self/ml/flash_decode.hexa:14-27). Replaces the reference's one-thread-per-
// (head, query) _hx_cuda_kern_attn_dt_fwd (runtime_cuda_emit.hexa:2819-2895)
// for decode.
//
// Cache layout per layer: [B][Hkv][lmax][hd] bf16, so one (b, kv head) is a
// contiguous [pos][hd] slab: keys are streamed with fully coalesced 16-byte
// loads (4 lanes per key row), values one 256-byte row per warp instruction.
// Grid (nsplit, Hkv, B), 128 threads; every CTA serves all G = H/Hkv query
// heads of its KV head, so each K/V byte is read once per step. The last CTA
// of a (b, kv head) to finish (atomic ticket) merges the splits — no extra
// launch. Scores and probabilities stay fp32; K/V are widened from bf16.
#include <cmath>
#include "common.cuh"
#include "forge_internal.h"

namespace {
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;

template <int HD, int G>
__global__ void __launch_bounds__(kThreads) k_flash_decode(const ForgeAttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    float* qs = sm;                 // [G][HD]
    float* red = qs + G * HD;       // [kWarps][G][HD]
    float* stat = red + kWarps * G * HD;  // [2 * G + 4]
    float* sc = stat + 2 * G + 4;   // [G][chunk_max]

    const int sp = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int nsplit = gridDim.x;
    pdl_trigger();
    pdl_wait();

    const int P = a.pos[b];
    if (P < 0 || P >= a.lmax) {
        if (tid == 0) atomicOr(a.err, FORGE_DEVERR_BAD_INDEX);
        return;
    }
    const int Lc = P + 1;
    const int chunk = (Lc + nsplit - 1) / nsplit;
    const int j0 = sp * chunk;
    const int j1 = min(Lc, j0 + chunk);
    const int n = max(0, j1 - j0);
    const int chunk_max = (a.lmax + nsplit - 1) / nsplit;
    const float scale = 1.0f / sqrtf((float)HD);

    for (int i = tid; i < G * HD; i += kThreads)
        qs[i] = a.q[(size_t)b * a.H * HD + (size_t)(kvh * G) * HD + i];
    __syncthreads();

    const size_t slab = ((size_t)b * a.Hkv + kvh) * a.lmax * HD;
    const uint16_t* K = a.kc + slab;
    const uint16_t* V = a.vc + slab;

    // ---- scores: 4 lanes per key; lane part qp reads 16 B at qp*16 + 64*m
    const int qp = lane & 3;
    constexpr int M = HD / 32;  // 16-byte pieces per lane per key
    for (int base = warp * 8; base < n; base += kWarps * 8) {
        const int jj = base + (lane >> 2);
        float dot[G];
#pragma unroll
        for (int gi = 0; gi < G; ++gi) dot[gi] = 0.f;
        if (jj < n) {
            const uint16_t* kr = K + (size_t)(j0 + jj) * HD;
            uint4 kv[M];
#pragma unroll
            for (int m = 0; m < M; ++m) kv[m] = *reinterpret_cast<const uint4*>(kr + m * 32 + qp * 8);
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const uint32_t w4[4] = {kv[m].x, kv[m].y, kv[m].z, kv[m].w};
#pragma unroll
                for (int gi = 0; gi < G; ++gi) {
                    const float* qv = qs + gi * HD + m * 32 + qp * 8;
                    const float4 q0 = *reinterpret_cast<const float4*>(qv);
                    const float4 q1 = *reinterpret_cast<const float4*>(qv + 4);
                    float d = dot[gi];
                    d = fmaf(q0.x, bf16_lo_f32(w4[0]), d); d = fmaf(q0.y, bf16_hi_f32(w4[0]), d);
                    d = fmaf(q0.z, bf16_lo_f32(w4[1]), d); d = fmaf(q0.w, bf16_hi_f32(w4[1]), d);
                    d = fmaf(q1.x, bf16_lo_f32(w4[2]), d); d = fmaf(q1.y, bf16_hi_f32(w4[2]), d);
                    d = fmaf(q1.z, bf16_lo_f32(w4[3]), d); d = fmaf(q1.w, bf16_hi_f32(w4[3]), d);
                    dot[gi] = d;
                }
            }
        }
#pragma unroll
        for (int gi = 0; gi < G; ++gi) {
            float d = dot[gi];
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            d += __shfl_xor_sync(0xffffffffu, d, 2);
            if (qp == 0 && jj < n) sc[gi * chunk_max + jj] = d * scale;
        }
    }
    __syncthreads();

    // ---- split-local softmax statistics per query head (warp gi % kWarps)
    for (int gi = warp; gi < G; gi += kWarps) {
        float mx = -INFINITY;
        for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[gi * chunk_max + j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float l = 0.f;
        for (int j = lane; j < n; j += 32) {
            const float p = expf(sc[gi * chunk_max + j] - mx);
            sc[gi * chunk_max + j] = p;
            l += p;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) { stat[2 * gi] = mx; stat[2 * gi + 1] = l; }
    }
    __syncthreads();

    // ---- P·V: each warp takes keys j = warp, warp + 4, ...; lane owns HD/32 dims
    constexpr int E = HD / 32;
    float acc[G][E];
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
#pragma unroll
        for (int e = 0; e < E; ++e) acc[gi][e] = 0.f;
    int j = warp;
    for (; j + 3 * kWarps < n; j += 4 * kWarps) {
        uint32_t vv[4][E / 2];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint16_t* vr = V + (size_t)(j0 + j + u * kWarps) * HD + lane * E;
            if (E == 4) { uint2 t2 = *reinterpret_cast<const uint2*>(vr); vv[u][0] = t2.x; vv[u][E / 2 - 1] = t2.y; }
            else vv[u][0] = *reinterpret_cast<const uint32_t*>(vr);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int gi = 0; gi < G; ++gi) {
                const float p = sc[gi * chunk_max + j + u * kWarps];
#pragma unroll
                for (int e2 = 0; e2 < E / 2; ++e2) {
                    acc[gi][2 * e2] = fmaf(p, bf16_lo_f32(vv[u][e2]), acc[gi][2 * e2]);
                    acc[gi][2 * e2 + 1] = fmaf(p, bf16_hi_f32(vv[u][e2]), acc[gi][2 * e2 + 1]);
                }
            }
    }
    for (; j < n; j += kWarps) {
        const uint16_t* vr = V + (size_t)(j0 + j) * HD + lane * E;
        uint32_t vv[E / 2];
        if (E == 4) { uint2 t2 = *reinterpret_cast<const uint2*>(vr); vv[0] = t2.x; vv[E / 2 - 1] = t2.y; }
        else vv[0] = *reinterpret_cast<const uint32_t*>(vr);
#pragma unroll
        for (int gi = 0; gi < G; ++gi) {
            const float p = sc[gi * chunk_max + j];
#pragma unroll
            for (int e2 = 0; e2 < E / 2; ++e2) {
                acc[gi][2 * e2] = fmaf(p, bf16_lo_f32(vv[e2]), acc[gi][2 * e2]);
                acc[gi][2 * e2 + 1] = fmaf(p, bf16_hi_f32(vv[e2]), acc[gi][2 * e2 + 1]);
            }
        }
    }
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
#pragma unroll
        for (int e = 0; e < E; ++e) red[(warp * G + gi) * HD + lane * E + e] = acc[gi][e];
    __syncthreads();

    // ---- write this split's partial (unnormalised O, m, l)
    const int stride = HD + 2;
    for (int i = tid; i < G * HD; i += kThreads) {
        const int gi = i / HD, e = i % HD;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += red[(w * G + gi) * HD + e];
        const int h = kvh * G + gi;
        a.partial[(((size_t)b * a.H + h) * nsplit + sp) * stride + e] = s;
    }
    if (tid < G) {
        const int h = kvh * G + tid;
        float* pm = a.partial + (((size_t)b * a.H + h) * nsplit + sp) * stride + HD;
        pm[0] = n > 0 ? stat[2 * tid] : -INFINITY;
        pm[1] = n > 0 ? stat[2 * tid + 1] : 0.f;
    }
    __threadfence();
    __syncthreads();
    __shared__ int is_last;
    if (tid == 0) {
        const uint32_t old = atomicAdd(a.counters + (size_t)b * a.Hkv + kvh, 1u);
        is_last = (old == (uint32_t)(nsplit - 1));
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();

    // ---- merge all splits (log-sum-exp), write fp32 context
    for (int i = tid; i < G * HD; i += kThreads) {
        const int gi = i / HD, e = i % HD;
        const int h = kvh * G + gi;
        const float* pb = a.partial + ((size_t)b * a.H + h) * nsplit * stride;
        float mg = -INFINITY;
        for (int s2 = 0; s2 < nsplit; ++s2) mg = fmaxf(mg, __ldcg(pb + s2 * stride + HD));
        float lsum = 0.f, o = 0.f;
        for (int s2 = 0; s2 < nsplit; ++s2) {
            const float ms = __ldcg(pb + s2 * stride + HD);
            const float w = ms == -INFINITY ? 0.f : expf(ms - mg);
            lsum = fmaf(w, __ldcg(pb + s2 * stride + HD + 1), lsum);
            o = fmaf(w, __ldcg(pb + s2 * stride + e), o);
        }
        a.out[(size_t)b * a.H * HD + (size_t)h * HD + e] = o / lsum;
    }
    if (tid == 0) a.counters[(size_t)b * a.Hkv + kvh] = 0u;
}

template <int HD, int G>
int launch(const ForgeAttnArgs& a, cudaStream_t stream, bool pdl) {
    const int chunk_max = (a.lmax + a.nsplit - 1) / a.nsplit;
    const size_t smem = sizeof(float) * ((size_t)G * HD + (size_t)kWarps * G * HD + 2 * G + 4 +
                                         (size_t)G * chunk_max);
    if (smem > 200 * 1024) return forge_fail(-1, "flash-decode: chunk too long (%d) — raise nsplit", chunk_max);
    auto kern = k_flash_decode<HD, G>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nsplit, a.Hkv, a.B);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return forge_fail(-1, "flash-decode launch: %s", cudaGetErrorString(e));
    return 0;
}

template <int HD>
int launch_g(const ForgeAttnArgs& a, cudaStream_t s, bool pdl) {
    switch (a.H / a.Hkv) {
    case 1: return launch<HD, 1>(a, s, pdl);
    case 2: return launch<HD, 2>(a, s, pdl);
    case 4: return launch<HD, 4>(a, s, pdl);
    case 8: return launch<HD, 8>(a, s, pdl);
    default: return forge_fail(-1, "flash-decode: query heads per KV head must be 1, 2, 4 or 8");
    }
}

template <int HD, int G>
int configure_one() {
    cudaError_t e = cudaFuncSetAttribute(k_flash_decode<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    return e == cudaSuccess ? 0 : forge_fail(-1, "flash-decode attr: %s", cudaGetErrorString(e));
}
}  // namespace

// One-time (per device) shared-memory opt-in of every flash-decode
// instantiation; must run outside stream capture.
int forge_attn_configure() {
    static bool done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return forge_fail(-1, "flash-decode: no device");
    if (done[dev]) return 0;
    int rc = configure_one<64, 1>() | configure_one<64, 2>() | configure_one<64, 4>() | configure_one<64, 8>() |
             configure_one<128, 1>() | configure_one<128, 2>() | configure_one<128, 4>() | configure_one<128, 8>();
    if (!rc) done[dev] = true;
    return rc ? -1 : 0;
}

int forge_attn_pick_splits(int B, int Hkv, int lmax) {
    // ~4 CTAs per SM of a 148-SM B200; fixed so workspace sizes do not depend
    // on which device is current.
    const int target = 4 * 148;
    int ns = (target + B * Hkv - 1) / (B * Hkv);
    const int cap = (lmax + 63) / 64;  // at least ~64 keys per split at full context
    if (ns > cap) ns = cap;
    if (ns < 1) ns = 1;
    // keep the score buffer within shared memory for long contexts
    while ((lmax + ns - 1) / ns > 8192) ++ns;
    return ns;
}
int64_t forge_attn_partial_floats(int B, int H, int hd, int nsplit) {
    return (int64_t)B * H * nsplit * (hd + 2);
}

int forge_attn_launch(const ForgeAttnArgs& a, cudaStream_t stream, bool pdl) {
    if (!a.q || !a.kc || !a.vc || !a.pos || !a.partial || !a.counters || !a.out || a.B <= 0 ||
        a.Hkv <= 0 || a.H % a.Hkv || a.nsplit <= 0 || a.lmax <= 0)
        return forge_fail(-1, "flash-decode: bad args");
    if (a.hd == 128) return launch_g<128>(a, stream, pdl);
    if (a.hd == 64) return launch_g<64>(a, stream, pdl);
    return forge_fail(-1, "flash-decode: head_dim must be 64 or 128 (got %d)", a.hd);
}
