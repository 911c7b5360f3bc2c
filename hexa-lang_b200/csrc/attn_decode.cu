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
//
// Paged mode (the page pool of self/alloc/paged_kv.hexa): K/V rows come from
// pages of page_tokens rows through a per-sequence page table; a key tile
// is gathered with one bulk copy per page segment into the same shared
// layout, so the arithmetic — and the result, bit for bit — is that of the
// contiguous cache. Page ids are checked against the pool before any copy.
#include <cmath>
#include "common.cuh"
#include "forge_internal.h"
#include "gemv_core.cuh"

namespace {
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 64;    // keys per shared-memory tile
constexpr int kStages = 2;   // K+V tiles in flight per CTA
constexpr int kFastMerge = 16;  // splits merged with all loads in one round trip

template <int HD>
constexpr int stage_bytes() { return 2 * kTile * HD * 2; }  // K tile + V tile, bf16

// Shared memory: [kStages][K tile | V tile] bf16, q [G][HD] f32, scores
// [G][kTile] f32, per-head running (m, l, alpha), mbarriers.
template <int HD, int G>
constexpr int smem_bytes() {
    return kStages * stage_bytes<HD>() + G * HD * 4 + G * kTile * 4 + 3 * G * 4 + kStages * 8 + 16;
}

template <int HD, int G, bool PAGED>
__global__ void __launch_bounds__(kThreads) k_flash_decode(const ForgeAttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint16_t* kv = reinterpret_cast<uint16_t*>(smem);
    float* qs = reinterpret_cast<float*>(smem + kStages * stage_bytes<HD>());
    float* sc = qs + G * HD;
    float* st_m = sc + G * kTile;
    float* st_l = st_m + G;
    float* st_a = st_l + G;
    uint64_t* full = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(st_a + G) + 7) & ~static_cast<uintptr_t>(7));

    const int sp = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int nsplit = gridDim.x;
    const int lin = sp + nsplit * (kvh + gridDim.y * b);
    unsigned long long* trace = (a.trace && lin < a.trace_ctas) ? a.trace + (size_t)lin * 4 : nullptr;
    if (trace && tid == 0) trace[0] = globaltimer_ns();

    // Positions only change between steps, so the split range and every
    // cached row below P can be fetched before the dependency wait; row P
    // (appended by the QKV kernel just before) is read after it.
    const int P = a.pos[b];
    const bool bad = (P < 0 || P >= a.lmax);
    const int Lc = bad ? 1 : P + 1;
    const int chunk = (Lc + nsplit - 1) / nsplit;
    const int j0 = sp * chunk;
    const int j1 = min(Lc, j0 + chunk);
    const int n = max(0, j1 - j0);
    const int ntiles = (n + kTile - 1) / kTile;
    const int sq = a.seq_of ? a.seq_of[b] : b;  // cache sequence of query row b
    const size_t slab = ((size_t)sq * a.Hkv + kvh) * a.lmax * HD;
    constexpr bool paged = PAGED;
    const int32_t* ptab = paged ? a.table + (size_t)b * a.max_pages : nullptr;
    // row r of this (sequence, kv head)
    auto row = [&](const uint16_t* base, int r) -> const uint16_t* {
        if (!paged) return base + slab + (size_t)r * HD;
        return base + (((size_t)ptab[r / a.page_tokens] * a.Hkv + kvh) * a.page_tokens + r % a.page_tokens) * HD;
    };

    auto issue = [&](int i) {
        const int s = i % kStages;
        const int t0 = j0 + i * kTile;
        const int rows = min(min(j1, t0 + kTile), P) - t0;  // row P excluded
        uint16_t* dst = kv + (size_t)s * (stage_bytes<HD>() / 2);
        if (rows > 0) {
            const uint32_t bytes = (uint32_t)rows * HD * 2;
            mbar_arrive_expect_tx(&full[s], 2 * bytes);
            if (!paged) {
                bulk_g2s_stream(dst, row(a.kc, t0), bytes, &full[s], l2_evict_first());
                bulk_g2s_stream(dst + kTile * HD, row(a.vc, t0), bytes, &full[s], l2_evict_first());
            } else {
                for (int r = t0; r < t0 + rows;) {  // one copy per page segment
                    const int seg = min(t0 + rows - r, a.page_tokens - r % a.page_tokens);
                    bulk_g2s(dst + (size_t)(r - t0) * HD, row(a.kc, r), (uint32_t)seg * HD * 2, &full[s]);
                    bulk_g2s(dst + (size_t)(kTile + r - t0) * HD, row(a.vc, r), (uint32_t)seg * HD * 2, &full[s]);
                    r += seg;
                }
            }
        } else {
            mbar_arrive(&full[s]);
        }
    };
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    // every page this sequence reads must be a page of the pool
    if (paged) {
        bool bad_page = false;
        if (!bad)
            for (int pg = tid; pg <= P / a.page_tokens; pg += kThreads)
                bad_page |= (unsigned)ptab[pg] >= (unsigned)a.num_pages;
        if (__syncthreads_or(bad_page)) {
            if (tid == 0) atomicOr(a.err, FORGE_DEVERR_BAD_INDEX);
            return;
        }
    } else {
        __syncthreads();
    }
    if (tid == 0 && !bad)
        for (int i = 0; i < kStages && i < ntiles; ++i) issue(i);
    pdl_trigger();
    pdl_wait();
    if (trace && tid == 0) trace[1] = globaltimer_ns();
    if (bad) {  // no copies were issued
        if (tid == 0) atomicOr(a.err, FORGE_DEVERR_BAD_INDEX);
        return;
    }
    for (int i = tid; i < G * HD; i += kThreads) qs[i] = a.q[(size_t)b * a.H * HD + (size_t)(kvh * G) * HD + i];
    if (tid < G) { st_m[tid] = -INFINITY; st_l[tid] = 0.f; }
    const float scale = 1.0f / sqrtf((float)HD);

    constexpr int E = HD / 32;            // value dims per lane
    constexpr int NCH = HD / 16;          // 16-byte chunks per half key row (HD/2 dims)
    float acc[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < E; ++e) acc[g][e] = 0.f;

    bool ok = true;
    for (int i = 0; i < ntiles && ok; ++i) {
        const int s = i % kStages;
        if (!mbar_wait(&full[s], (i / kStages) & 1, a.err)) { ok = false; break; }
        const uint16_t* Ks = kv + (size_t)s * (stage_bytes<HD>() / 2);
        const uint16_t* Vs = Ks + kTile * HD;
        const int t0 = j0 + i * kTile;
        const int nt = min(kTile, j1 - t0);
        if (t0 + nt == Lc) {
            // the newest row comes straight from global memory
            uint16_t* kd = const_cast<uint16_t*>(Ks) + (size_t)(nt - 1) * HD;
            uint16_t* vd = const_cast<uint16_t*>(Vs) + (size_t)(nt - 1) * HD;
            if (tid < HD / 8) reinterpret_cast<uint4*>(kd)[tid] = reinterpret_cast<const uint4*>(row(a.kc, P))[tid];
            else if (tid < HD / 4) reinterpret_cast<uint4*>(vd)[tid - HD / 8] = reinterpret_cast<const uint4*>(row(a.vc, P))[tid - HD / 8];
        }
        __syncthreads();
        // ---- scores: two threads per key, each half a row; chunk order rotated by
        // thread so the 8 threads of a shared-memory phase hit distinct banks
        {
            // rows past nt hold stale data: computed but never stored, so the
            // warp stays converged for the shuffle
            const int k = tid >> 1, h = tid & 1;
            float dot[G];
#pragma unroll
            for (int g = 0; g < G; ++g) dot[g] = 0.f;
            const uint16_t* kr = Ks + (size_t)k * HD + h * (HD / 2);
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                const int c = (j + tid) & (NCH - 1);
                const uint4 kw = *reinterpret_cast<const uint4*>(kr + c * 8);
                const uint32_t w4[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float* qv = qs + g * HD + h * (HD / 2) + c * 8;
                    const float4 q0 = *reinterpret_cast<const float4*>(qv);
                    const float4 q1 = *reinterpret_cast<const float4*>(qv + 4);
                    float d = dot[g];
                    d = fmaf(q0.x, bf16_lo_f32(w4[0]), d); d = fmaf(q0.y, bf16_hi_f32(w4[0]), d);
                    d = fmaf(q0.z, bf16_lo_f32(w4[1]), d); d = fmaf(q0.w, bf16_hi_f32(w4[1]), d);
                    d = fmaf(q1.x, bf16_lo_f32(w4[2]), d); d = fmaf(q1.y, bf16_hi_f32(w4[2]), d);
                    d = fmaf(q1.z, bf16_lo_f32(w4[3]), d); d = fmaf(q1.w, bf16_hi_f32(w4[3]), d);
                    dot[g] = d;
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float d = dot[g] + __shfl_xor_sync(0xffffffffu, dot[g], 1);
                if (h == 0 && k < nt) sc[g * kTile + k] = d * scale;
            }
        }
        __syncthreads();
        // ---- online softmax statistics (one warp per head)
        for (int g = warp; g < G; g += kWarps) {
            float mt = -INFINITY;
            for (int j = lane; j < nt; j += 32) mt = fmaxf(mt, sc[g * kTile + j]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
            const float mo = st_m[g];
            const float mn = fmaxf(mo, mt);
            float ls = 0.f;
            for (int j = lane; j < nt; j += 32) {
                const float p = expf(sc[g * kTile + j] - mn);
                sc[g * kTile + j] = p;
                ls += p;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
            if (lane == 0) {
                const float al = (mo == -INFINITY) ? 0.f : expf(mo - mn);
                st_a[g] = al;
                st_l[g] = st_l[g] * al + ls;
                st_m[g] = mn;
            }
        }
        __syncthreads();
        // ---- P·V: warp w takes keys w, w+4, ...; lane owns dims lane*E..+E
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float al = st_a[g];
#pragma unroll
            for (int e = 0; e < E; ++e) acc[g][e] *= al;
        }
        for (int j = warp; j < nt; j += kWarps) {
            uint32_t vv[E / 2];
            if (E == 4) {
                const uint2 t2 = *reinterpret_cast<const uint2*>(Vs + (size_t)j * HD + lane * E);
                vv[0] = t2.x; vv[E / 2 - 1] = t2.y;
            } else {
                vv[0] = *reinterpret_cast<const uint32_t*>(Vs + (size_t)j * HD + lane * E);
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float p = sc[g * kTile + j];
#pragma unroll
                for (int e2 = 0; e2 < E / 2; ++e2) {
                    acc[g][2 * e2] = fmaf(p, bf16_lo_f32(vv[e2]), acc[g][2 * e2]);
                    acc[g][2 * e2 + 1] = fmaf(p, bf16_hi_f32(vv[e2]), acc[g][2 * e2 + 1]);
                }
            }
        }
        __syncthreads();  // stage s and the scores are free again
        if (tid == 0 && i + kStages < ntiles) issue(i + kStages);
    }
    if (!ok) return;

    // ---- combine the four warps' partial O (reusing the tile buffers)
    float* red = reinterpret_cast<float*>(smem);  // [kWarps][G][HD]
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < E; ++e) red[(warp * G + g) * HD + lane * E + e] = acc[g][e];
    __syncthreads();
    const int stride = HD + 2;
    for (int idx = tid; idx < G * HD; idx += kThreads) {
        const int g = idx / HD, e = idx % HD;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) sum += red[(w * G + g) * HD + e];
        const int h = kvh * G + g;
        a.partial[(((size_t)b * a.H + h) * nsplit + sp) * stride + e] = sum;
    }
    if (tid < G) {
        const int h = kvh * G + tid;
        float* pm = a.partial + (((size_t)b * a.H + h) * nsplit + sp) * stride + HD;
        pm[0] = n > 0 ? st_m[tid] : -INFINITY;
        pm[1] = n > 0 ? st_l[tid] : 0.f;
    }
    // ticket: the block barrier orders every thread's partial stores before
    // thread 0's release; the last CTA's acquire orders its loads after all
    // the other CTAs' stores (the barrier hands the acquire to every thread)
    __syncthreads();
    if (trace && tid == 0) trace[2] = globaltimer_ns();
    __shared__ int is_last;
    if (tid == 0) {
        uint32_t old;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                     : "=r"(old) : "l"(a.counters + (size_t)b * a.Hkv + kvh) : "memory");
        is_last = (old == (uint32_t)(nsplit - 1));
    }
    __syncthreads();
    if (!is_last) return;

    // ---- merge all splits (log-sum-exp), write the fp32 context: per head,
    // mg = max m_s, w_s = exp(m_s - mg), o = sum_s w_s O_s / sum_s w_s l_s,
    // both sums in split order.
    float* mw = reinterpret_cast<float*>(smem);  // [G][nsplit] m, then the weight
    float* lw = mw + G * nsplit;                 // [G][nsplit] l
    float* ls = lw + G * nsplit;                 // [G] normaliser
    float* vals = mw + ((2 * G * nsplit + G + 3) & ~3);  // [G][HD] merged context (handoff), 16-byte aligned
    if (nsplit <= kFastMerge) {
        // every thread loads all splits' (m, l) and partials of its elements
        // at once (one L2 round trip) and forms its head's weights itself
        for (int idx = tid; idx < G * HD; idx += kThreads) {
            const int g = idx / HD, e = idx % HD;
            const int h = kvh * G + g;
            const float* pb = a.partial + ((size_t)b * a.H + h) * nsplit * stride;
            float2 ml[kFastMerge];
            float v[kFastMerge];
#pragma unroll
            for (int s2 = 0; s2 < kFastMerge; ++s2) {
                if (s2 < nsplit) {
                    ml[s2].x = __ldcg(pb + (size_t)s2 * stride + HD);
                    ml[s2].y = __ldcg(pb + (size_t)s2 * stride + HD + 1);
                    v[s2] = __ldcg(pb + (size_t)s2 * stride + e);
                }
            }
            float mg = -INFINITY;
#pragma unroll
            for (int s2 = 0; s2 < kFastMerge; ++s2)
                if (s2 < nsplit) mg = fmaxf(mg, ml[s2].x);
            float lsum = 0.f, o = 0.f;
#pragma unroll
            for (int s2 = 0; s2 < kFastMerge; ++s2) {
                if (s2 < nsplit) {
                    const float w = ml[s2].x == -INFINITY ? 0.f : expf(ml[s2].x - mg);
                    lsum = fmaf(w, ml[s2].y, lsum);
                    o = fmaf(w, v[s2], o);
                }
            }
            const float val = o / lsum;
            a.out[(size_t)b * a.H * HD + (size_t)h * HD + e] = val;
            if (HD == 128 && a.pq_out) vals[idx] = val;
        }
    } else {
        // many splits: every split's (m, l) once into shared memory, one
        // thread per head forms the weights and the normaliser, then every
        // output element sums its splits with its loads issued in batches
        for (int idx = tid; idx < G * nsplit; idx += kThreads) {
            const int g = idx / nsplit, s2 = idx % nsplit;
            const float* pm = a.partial + (((size_t)b * a.H + kvh * G + g) * nsplit + s2) * stride + HD;
            mw[idx] = __ldcg(pm);
            lw[idx] = __ldcg(pm + 1);
        }
        __syncthreads();
        if (tid < G) {
            float mg = -INFINITY;
            for (int s2 = 0; s2 < nsplit; ++s2) mg = fmaxf(mg, mw[tid * nsplit + s2]);
            float lsum = 0.f;
            for (int s2 = 0; s2 < nsplit; ++s2) {
                const float ms = mw[tid * nsplit + s2];
                const float w = ms == -INFINITY ? 0.f : expf(ms - mg);
                mw[tid * nsplit + s2] = w;
                lsum = fmaf(w, lw[tid * nsplit + s2], lsum);
            }
            ls[tid] = lsum;
        }
        __syncthreads();
        for (int idx = tid; idx < G * HD; idx += kThreads) {
            const int g = idx / HD, e = idx % HD;
            const int h = kvh * G + g;
            const float* pb = a.partial + ((size_t)b * a.H + h) * nsplit * stride + e;
            const float* wg = mw + g * nsplit;
            float o = 0.f;
            int s2 = 0;
            for (; s2 + 8 <= nsplit; s2 += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __ldcg(pb + (size_t)(s2 + j) * stride);
#pragma unroll
                for (int j = 0; j < 8; ++j) o = fmaf(wg[s2 + j], v[j], o);
            }
            for (; s2 < nsplit; ++s2) o = fmaf(wg[s2], __ldcg(pb + (size_t)s2 * stride), o);
            const float val = o / ls[g];
            a.out[(size_t)b * a.H * HD + (size_t)h * HD + e] = val;
            if (HD == 128 && a.pq_out) vals[idx] = val;
        }
    }
    if (HD == 128 && a.pq_out) {
        // each head's context is one 128-group of the O projection's input:
        // hand it over staged (one warp per head)
        __syncthreads();
        for (int g = warp; g < G; g += kWarps) {
            const float4 v = reinterpret_cast<const float4*>(vals + g * HD)[lane];
            pq_group_warp(v, kvh * G + g, b, 2 * a.B, a.H, a.pq_out);
        }
    }
    if (tid == 0) a.counters[(size_t)b * a.Hkv + kvh] = 0u;
    if (trace && tid == 0) trace[3] = globaltimer_ns();
}

template <int HD, int G>
int launch(const ForgeAttnArgs& a, cudaStream_t stream, bool pdl) {
    constexpr int smem = smem_bytes<HD, G>();
    static_assert(kWarps * G * HD * 4 <= kStages * stage_bytes<HD>(), "partial-O reduction must fit the tile buffers");
    auto kern = a.table ? k_flash_decode<HD, G, true> : k_flash_decode<HD, G, false>;
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
    cudaError_t e = cudaFuncSetAttribute(k_flash_decode<HD, G, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_flash_decode<HD, G, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    for (auto f : {k_flash_decode<HD, G, false>, k_flash_decode<HD, G, true>})
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
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
    // Splits per (sequence, kv head) minimising waves x (fixed cost + key
    // tiles per split): every CTA of a wave of the resident slots (3 per SM
    // of a 148-SM B200 at ~65 KB of shared memory each) runs about as long
    // as its tile count plus a fixed ~2 tiles (ramp, partial write and
    // merge), so a partly filled last wave costs as much as a full one.
    // Fixed so workspace sizes do not depend on which device is current.
    const int resident = 3 * 148;
    const int pairs = B * Hkv;
    const int cap = (lmax + 127) / 128;  // at least ~128 keys per split at full context
    int best = 1;
    long long best_cost = -1;
    for (int ns = 1; ns <= cap; ++ns) {
        const long long items = (long long)pairs * ns;
        const long long waves = (items + resident - 1) / resident;
        const int tiles = ((lmax + ns - 1) / ns + kTile - 1) / kTile;
        const long long cost = waves * (2 + tiles);
        if (best_cost < 0 || cost <= best_cost) { best_cost = cost; best = ns; }  // ties: more splits
    }
    return best;
}
int64_t forge_attn_partial_floats(int B, int H, int hd, int nsplit) {
    return (int64_t)B * H * nsplit * (hd + 2);
}

int forge_attn_launch(const ForgeAttnArgs& a, cudaStream_t stream, bool pdl) {
    if (!a.q || !a.kc || !a.vc || !a.pos || !a.partial || !a.counters || !a.out || a.B <= 0 ||
        a.Hkv <= 0 || a.H % a.Hkv || a.nsplit <= 0 || a.lmax <= 0)
        return forge_fail(-1, "flash-decode: bad args");
    if (a.table && (a.page_tokens <= 0 || a.max_pages <= 0 || a.num_pages <= 0 ||
                    (int64_t)a.max_pages * a.page_tokens != a.lmax))
        return forge_fail(-1, "flash-decode: bad page geometry");
    // the merge keeps (m, l) of every split of the CTA's heads in the tile buffers
    if (a.hd == 128 || a.hd == 64) {
        const long long merge_bytes = 4LL * (2LL * (a.H / a.Hkv) * a.nsplit + a.H / a.Hkv + 3 +
                                             (a.pq_out ? (long long)(a.H / a.Hkv) * a.hd : 0));
        const long long tile_bytes = a.hd == 128 ? kStages * stage_bytes<128>() : kStages * stage_bytes<64>();
        if (merge_bytes > tile_bytes) return forge_fail(-1, "flash-decode: %d splits are too many to merge", a.nsplit);
    }
    if (a.pq_out && (a.hd != 128 || a.B > 4 || a.table || a.seq_of))
        return forge_fail(-1, "flash-decode: the staged handoff needs head_dim 128, batch <= 4, contiguous decode");
    if (a.hd == 128) return launch_g<128>(a, stream, pdl);
    if (a.hd == 64) return launch_g<64>(a, stream, pdl);
    return forge_fail(-1, "flash-decode: head_dim must be 64 or 128 (got %d)", a.hd);
}
