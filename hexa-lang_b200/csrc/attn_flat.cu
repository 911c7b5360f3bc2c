// attn_flat.cu — flash-decode for small decode batches over the contiguous
// bf16 KV cache: the same single-query causal GQA attention as attn_decode.cu
// (nn_attn_core_fwd, nn_lib.hexa:221-278, row i = current position; split
// partials merged by log-sum-exp as self/ml/flash_decode.hexa:14-27), laid
// out for a batch of one to a few sequences.
//
// At batch 1 the per-(sequence, head, split) grid of attn_decode.cu gives
// every CTA three 64-key tiles: most of its time goes to the first copy's
// latency, one more round trip for the third tile, and the split merge.
// Here the key tiles of all (sequence, KV head) pairs are laid end to end
// and cut into one contiguous range per CTA (one CTA per SM), so every SM
// streams the same number of bytes:
//   warp 8 (producer)  walks the CTA's tiles and streams each one — K rows
//                      and V rows of 32 (head_dim 128) or 64 (head_dim 64)
//                      keys, 16 KB — into an 8-stage (6 for 4 or more query
//                      heads per KV head) mbarrier ring with cp.async.bulk.
//                      Cached rows never change during a step, so it starts
//                      before the dependency wait; only the row appended
//                      this step (position P, written by the QKV kernel) is
//                      read after it, from global memory.
//   warps 0-7          tile i of the range belongs to warp i % 8, which runs
//                      the whole tile on its own online-softmax state: scores
//                      (4 lanes per key, staged in shared memory), the tile
//                      maximum and probabilities (one lane per key), then
//                      P.V (one lane per 4 or 2 value dims). Eight tiles are
//                      in work at once, so one tile's dependent steps
//                      (shuffles, exponentials) overlap the others'. Where
//                      the range crosses from one pair to the next (and at
//                      its end) the eight warp states are merged into one
//                      partial per (pair, CTA).
//   The last CTA to finish a pair (atomic ticket) merges that pair's
//   partials (at most one per CTA it spans) and writes the fp32 context.
// The kernel is held to 72 registers per thread and at most ~135 KB of
// shared memory, so a CTA fits on an SM beside one CTA of the decode GEMV:
// under programmatic dependent launch the KV stream starts while the QKV
// projection is still running.
#include <cmath>
#include "common.cuh"
#include "forge_internal.h"

namespace {
constexpr int kCW = 8;                 // consumer warps
constexpr int kNT = kCW * 32;          // consumer threads
constexpr int kThreads = kNT + 32;     // + one producer warp
constexpr int kTileBytes = 16384;      // K tile + V tile
constexpr int kMaxB = 32;              // sequences per launch

template <int HD, int G>
struct Geo {
    static constexpr int TK = kTileBytes / (4 * HD);  // keys per tile: 32 (hd 128) or 64 (hd 64)
    static constexpr int NSB = TK / 8;                 // 8-key blocks of the score step (4 lanes per key)
    static constexpr int NCH = HD / 8;                 // 16-byte chunks per key row
    static constexpr int CPL = NCH / 4;                // chunks per lane in the score step
    static constexpr int KPL = TK / 32;                // keys per lane in the softmax step
    static constexpr int E = HD / 32;                  // value dims per lane in the P.V step
    static constexpr int S = G <= 2 ? 8 : 6;           // ring stages
    static constexpr int SW = HD + 2;                  // floats per (warp or partial, head) state: O[HD], m, l
};

template <int HD, int G>
constexpr int smem_bytes() {
    using Gm = Geo<HD, G>;
    return Gm::S * kTileBytes + 4 * (G * HD + kCW * G * Gm::TK + kCW * G * Gm::SW) + 8 * (kMaxB + 1) +
           4 * 2 * kMaxB + 16 * Gm::S + 16;
}

// (sequence, kv head, tile within the pair) of flat tile t.
__device__ __forceinline__ void tile_at(long long t, const long long* tstart, const int* tcount, int B, int& b,
                                        int& kvh, int& j) {
    b = 0;
    while (b + 1 < B && tstart[b + 1] <= t) ++b;
    const int r = (int)(t - tstart[b]);
    kvh = r / tcount[b];
    j = r - kvh * tcount[b];
}
// CTA whose range [NT*c/grid, NT*(c+1)/grid) holds tile t.
__device__ __forceinline__ int cta_of(long long t, long long NT, int grid) {
    return (int)(((t + 1) * grid - 1) / NT);
}

template <int HD, int G>
__global__ void __maxnreg__(72) k_attn_flat(const ForgeAttnArgs a) {
    using Gm = Geo<HD, G>;
    constexpr int TK = Gm::TK, NSB = Gm::NSB, NCH = Gm::NCH, CPL = Gm::CPL, KPL = Gm::KPL, E = Gm::E, S = Gm::S,
                  SW = Gm::SW;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    float* qs = reinterpret_cast<float*>(smem + S * kTileBytes);   // [G][HD] query of the current pair
    float* sc = qs + G * HD;                                        // [kCW][G][TK] scores, then probabilities
    float* wst = sc + kCW * G * TK;                                 // [kCW][G][SW] warp states at a flush
    long long* tstart = reinterpret_cast<long long*>(wst + kCW * G * SW);  // [B+1] first flat tile of sequence b
    int* tcount = reinterpret_cast<int*>(tstart + kMaxB + 1);      // [B] tiles per pair of sequence b
    int* spos = tcount + kMaxB;                                     // [B] position P
    uint64_t* full = reinterpret_cast<uint64_t*>(spos + kMaxB);
    uint64_t* empty = full + S;
    // [0] abort, [1] last CTA of a pair, [2] tiles the producer has issued
    volatile int* flags = reinterpret_cast<volatile int*>(empty + S);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int B = a.B;
    if (a.trace && tid == 0) a.trace[blockIdx.x * 4 + 0] = globaltimer_ns();
    if (tid == 0) {
        // Positions change only between steps, so the tile plan (and every
        // cached row below P) is known before the dependency wait.
        long long acc = 0;
        bool bad = false;
        for (int b = 0; b < B; ++b) {
            const int P = a.pos[b];
            const bool ok = P >= 0 && P < a.lmax;
            bad |= !ok;
            const int T = ok ? (P + TK) / TK : 0;  // ceil((P + 1) / TK)
            spos[b] = ok ? P : -1;
            tcount[b] = T;
            tstart[b] = acc;
            acc += (long long)T * a.Hkv;
        }
        tstart[B] = acc;
        flags[0] = 0;
        flags[1] = 0;
        flags[2] = 0;
        if (bad && blockIdx.x == 0) atomicOr(a.err, FORGE_DEVERR_BAD_INDEX);
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);  // released by the one warp that used the tile
        }
        fence_mbar_init();
    }
    __syncthreads();
    const long long NT = tstart[B];
    const int grid = gridDim.x;
    const long long t_begin = NT * blockIdx.x / grid, t_end = NT * (blockIdx.x + 1) / grid;
    pdl_trigger();

    if (warp == kCW) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t it = 0;
            for (long long t = t_begin; t < t_end; ++t) {
                int b, kvh, j;
                tile_at(t, tstart, tcount, B, b, kvh, j);
                const int s = it % S;
                if (flags[0] || !mbar_wait(&empty[s], ((it / S) & 1u) ^ 1u, a.err)) {
                    flags[0] = 1;
                    break;
                }
                const int r0 = j * TK;
                const int rows = min(r0 + TK, spos[b]) - r0;  // row P is read after the dependency wait
                uint8_t* dst = ring + (size_t)s * kTileBytes;
                __threadfence_block();
                flags[2] = (int)(it + 1);  // slot s's previous tile has been released
                if (rows > 0) {
                    const uint32_t bytes = (uint32_t)rows * HD * 2;
                    const size_t base = (((size_t)b * a.Hkv + kvh) * a.lmax + r0) * HD;
                    mbar_arrive_expect_tx(&full[s], 2 * bytes);
                    bulk_g2s(dst, a.kc + base, bytes, &full[s]);
                    bulk_g2s(dst + TK * HD * 2, a.vc + base, bytes, &full[s]);
                } else {
                    mbar_arrive(&full[s]);
                }
                ++it;
            }
            // every copy issued lands before the CTA exits (bounded)
            for (uint32_t k = 0; k < (uint32_t)S && k < it; ++k) {
                const uint32_t idx = it - 1 - k;
                mbar_wait(&full[idx % S], (idx / S) & 1u, a.err);
            }
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    // Tile i of the CTA's range goes to warp i % 8, which runs the whole
    // tile (scores, online softmax, P.V) on its own state, so eight tiles are
    // in work at once and a tile's dependent steps overlap other tiles'.
    pdl_wait();
    if (a.trace && tid == 0) a.trace[blockIdx.x * 4 + 1] = globaltimer_ns();
    const float scale = 1.0f / sqrtf((float)HD);
    const int kl = lane >> 2, qp = lane & 3;  // score step: key kl of an 8-key block, quarter qp of its row
    float* scw = sc + warp * G * TK;
    uint32_t it = 0;

    for (long long t = t_begin; t < t_end;) {
        int b, kvh, j0;
        tile_at(t, tstart, tcount, B, b, kvh, j0);
        const long long pair_end = tstart[b] + (long long)(kvh + 1) * tcount[b];
        const long long seg_end = pair_end < t_end ? pair_end : t_end;
        const int P = spos[b];
        const size_t slab = ((size_t)b * a.Hkv + kvh) * a.lmax * HD;
        for (int i = tid; i < G * HD; i += kNT) qs[i] = __ldcg(a.q + (size_t)b * a.H * HD + (size_t)kvh * G * HD + i);
        named_bar_sync(1, kNT);
        if (t == t_begin && a.trace && tid == 0) a.trace[blockIdx.x * 4 + 2] = globaltimer_ns();
        float m[G], l[G], acc[G][E];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            m[g] = -INFINITY;
            l[g] = 0.f;
#pragma unroll
            for (int e = 0; e < E; ++e) acc[g][e] = 0.f;
        }
        for (long long u = t; u < seg_end; ++u, ++it) {
            if ((int)(it % kCW) != warp) continue;
            const int s = it % S;
            // With fewer ring slots than warps (S = 6), a warp can reach tile
            // `it` before the producer has refilled slot s for tile it - S;
            // the slot's phase parity would then read as already complete.
            // Wait (bounded) until tile `it` has been issued: from then on
            // the slot's phase is that of tile it or the one after.
            if (S != kCW && !flags[0] && flags[2] <= (int)it) {
                const uint64_t t0 = globaltimer_ns();
                uint32_t spins = 0;
                while (flags[2] <= (int)it && !flags[0]) {
                    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > FORGE_WAIT_NS) {
                        if (lane == 0) atomicOr(a.err, FORGE_DEVERR_MBAR_TIMEOUT);
                        flags[0] = 1;
                    }
                }
                __threadfence_block();
            }
            if (!flags[0] && !mbar_wait(&full[s], (it / S) & 1u, a.err)) flags[0] = 1;
            if (!flags[0]) {
                const int r0 = (j0 + (int)(u - t)) * TK;
                const int nv = min(TK, P - r0 + 1);  // valid keys of the tile (row P is key P - r0)
                const uint16_t* Ks = reinterpret_cast<const uint16_t*>(ring + (size_t)s * kTileBytes);
                const uint16_t* Vs = Ks + TK * HD;
                // ---- scores: lanes (kl, qp) of block sb take key sb*8+kl,
                // chunks qp, qp+4, ... rotated by 4 on odd keys (no bank conflicts)
#pragma unroll
                for (int sb = 0; sb < NSB; ++sb) {
                    const int key = sb * 8 + kl;
                    float dot[G];
#pragma unroll
                    for (int g = 0; g < G; ++g) dot[g] = 0.f;
#pragma unroll
                    for (int c = 0; c < CPL; ++c) {
                        const int ch = (qp + 4 * c + 4 * (kl & 1)) & (NCH - 1);
                        uint4 kw = make_uint4(0u, 0u, 0u, 0u);
                        if (key == P - r0) kw = __ldcg(reinterpret_cast<const uint4*>(a.kc + slab + (size_t)P * HD + ch * 8));
                        else if (key < nv) kw = *reinterpret_cast<const uint4*>(Ks + key * HD + ch * 8);
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            const float4 q0 = *reinterpret_cast<const float4*>(qs + g * HD + ch * 8);
                            const float4 q1 = *reinterpret_cast<const float4*>(qs + g * HD + ch * 8 + 4);
                            float d = dot[g];
                            d = fmaf(q0.x, bf16_lo_f32(kw.x), d); d = fmaf(q0.y, bf16_hi_f32(kw.x), d);
                            d = fmaf(q0.z, bf16_lo_f32(kw.y), d); d = fmaf(q0.w, bf16_hi_f32(kw.y), d);
                            d = fmaf(q1.x, bf16_lo_f32(kw.z), d); d = fmaf(q1.y, bf16_hi_f32(kw.z), d);
                            d = fmaf(q1.z, bf16_lo_f32(kw.w), d); d = fmaf(q1.w, bf16_hi_f32(kw.w), d);
                            dot[g] = d;
                        }
                    }
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        float d = dot[g];
                        d += __shfl_xor_sync(0xffffffffu, d, 1);
                        d += __shfl_xor_sync(0xffffffffu, d, 2);
                        if (qp == 0) scw[g * TK + key] = key < nv ? d * scale : -INFINITY;
                    }
                }
                __syncwarp();
                // ---- online softmax over the tile (lane owns keys lane + 32i)
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float sv[KPL];
                    float tm = -INFINITY;
#pragma unroll
                    for (int i = 0; i < KPL; ++i) {
                        sv[i] = scw[g * TK + lane + 32 * i];
                        tm = fmaxf(tm, sv[i]);
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o));
                    const float mn = fmaxf(m[g], tm);  // finite: every tile has a valid key
                    const float al = m[g] == -INFINITY ? 0.f : expf(m[g] - mn);
                    float ps = 0.f;
#pragma unroll
                    for (int i = 0; i < KPL; ++i) {
                        const float p = sv[i] == -INFINITY ? 0.f : expf(sv[i] - mn);
                        scw[g * TK + lane + 32 * i] = p;
                        ps += p;
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
                    l[g] = l[g] * al + ps;
                    m[g] = mn;
#pragma unroll
                    for (int e = 0; e < E; ++e) acc[g][e] *= al;
                }
                __syncwarp();
                // ---- P.V: lane owns value dims lane*E .. lane*E+E-1
                for (int k = 0; k < nv; ++k) {
                    float v[E];
                    if constexpr (E == 4) {
                        const uint2 w2 = k == P - r0
                                             ? __ldcg(reinterpret_cast<const uint2*>(a.vc + slab + (size_t)P * HD + lane * 4))
                                             : *reinterpret_cast<const uint2*>(Vs + k * HD + lane * 4);
                        v[0] = bf16_lo_f32(w2.x); v[1] = bf16_hi_f32(w2.x);
                        v[E - 2] = bf16_lo_f32(w2.y); v[E - 1] = bf16_hi_f32(w2.y);
                    } else {
                        const uint32_t w1 = k == P - r0
                                                ? __ldcg(reinterpret_cast<const unsigned int*>(a.vc + slab + (size_t)P * HD + lane * 2))
                                                : *reinterpret_cast<const uint32_t*>(Vs + k * HD + lane * 2);
                        v[0] = bf16_lo_f32(w1); v[E - 1] = bf16_hi_f32(w1);
                    }
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float p = scw[g * TK + k];
#pragma unroll
                        for (int e = 0; e < E; ++e) acc[g][e] = fmaf(p, v[e], acc[g][e]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }

        // ---- flush: the eight warp states of this pair into the CTA's partial;
        // the last CTA of the pair merges all partials into the context
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float* w = wst + (warp * G + g) * SW;
#pragma unroll
            for (int e = 0; e < E; ++e) w[lane * E + e] = acc[g][e];
            if (lane == 0) {
                w[HD] = m[g];
                w[HD + 1] = l[g];
            }
        }
        named_bar_sync(1, kNT);
        // Partials of this pair: with at least one tile per CTA (NT >= grid)
        // the pair's tiles sit in the consecutive CTAs c0..c1, slot c - c0;
        // with fewer tiles than CTAs every CTA holds at most one tile and
        // CTAs without tiles can fall between them, so the slot is the tile's
        // index in the pair. Either way at most tcount slots.
        const long long ts = pair_end - tcount[b];
        int np, slot;
        if (NT >= grid) {
            const int c0 = cta_of(ts, NT, grid), c1 = cta_of(pair_end - 1, NT, grid);
            np = c1 - c0 + 1;
            slot = blockIdx.x - c0;
        } else {
            np = tcount[b];
            slot = (int)(t_begin - ts);
        }
        const int pair = b * a.Hkv + kvh;
        float* pp = a.partial + (size_t)pair * a.flat_slots * G * SW;
        for (int idx = tid; idx < G * HD; idx += kNT) {
            const int g = idx / HD, e = idx - g * HD;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kCW; ++w) M = fmaxf(M, wst[(w * G + g) * SW + HD]);
            float O = 0.f, L = 0.f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) {
                const float mw = wst[(w * G + g) * SW + HD];
                const float f = mw == -INFINITY ? 0.f : expf(mw - M);
                O = fmaf(f, wst[(w * G + g) * SW + e], O);
                L = fmaf(f, wst[(w * G + g) * SW + HD + 1], L);
            }
            float* dst = pp + ((size_t)slot * G + g) * SW;
            dst[e] = O;
            if (e == 0) {
                dst[HD] = M;
                dst[HD + 1] = L;
            }
        }
        __threadfence();
        named_bar_sync(1, kNT);
        if (tid == 0) {
            const uint32_t old = atomicAdd(a.counters + pair, 1u);
            flags[1] = old == (uint32_t)(np - 1);
        }
        named_bar_sync(1, kNT);
        if (flags[1]) {
            __threadfence();
            for (int idx = tid; idx < G * HD; idx += kNT) {
                const int g = idx / HD, e = idx - g * HD;
                float M = -INFINITY;
                for (int k = 0; k < np; ++k) M = fmaxf(M, __ldcg(pp + ((size_t)k * G + g) * SW + HD));
                float O = 0.f, L = 0.f;
                for (int k = 0; k < np; ++k) {
                    const float* src = pp + ((size_t)k * G + g) * SW;
                    const float mk = __ldcg(src + HD);
                    const float f = mk == -INFINITY ? 0.f : expf(mk - M);
                    O = fmaf(f, __ldcg(src + e), O);
                    L = fmaf(f, __ldcg(src + HD + 1), L);
                }
                a.out[(size_t)b * a.H * HD + (size_t)(kvh * G + g) * HD + e] = O / L;
            }
            if (tid == 0) a.counters[pair] = 0u;
        }
        t = seg_end;
    }
    if (a.trace && tid == 0) a.trace[blockIdx.x * 4 + 3] = globaltimer_ns();
}

template <int HD, int G>
int launch(const ForgeAttnArgs& a, cudaStream_t stream, bool pdl) {
    auto kern = k_attn_flat<HD, G>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(forge_sm_count());
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes<HD, G>();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return forge_fail(-1, "flat flash-decode launch: %s", cudaGetErrorString(e));
    return 0;
}

template <int HD, int G>
int configure_one() {
    cudaError_t e = cudaFuncSetAttribute(k_attn_flat<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_bytes<HD, G>());
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_attn_flat<HD, G>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
    return e == cudaSuccess ? 0 : forge_fail(-1, "flat flash-decode attr: %s", cudaGetErrorString(e));
}
}  // namespace

// Shapes the flat kernel serves: batch <= 32, head_dim 64 or 128, and the
// per-warp states of all query heads of a KV head within 2048 floats.
bool forge_attn_flat_supported(int B, int H, int Hkv, int hd) {
    if (B < 1 || B > kMaxB || Hkv <= 0 || H % Hkv) return false;
    const int G = H / Hkv;
    if (hd == 128) return G == 1 || G == 2 || G == 4;
    if (hd == 64) return G == 1 || G == 2 || G == 4 || G == 8;
    return false;
}
// Partial slots per pair (flat_slots) and the partial floats a launch needs.
int forge_attn_flat_slots(int hd, int lmax) {
    const int TK = kTileBytes / (4 * hd);
    return (lmax + TK - 1) / TK;
}
int64_t forge_attn_flat_partial_floats(int B, int H, int hd, int lmax) {
    return (int64_t)B * H * forge_attn_flat_slots(hd, lmax) * (hd + 2);
}

int forge_attn_flat_configure() {
    static bool done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return forge_fail(-1, "flat flash-decode: no device");
    if (done[dev]) return 0;
    int rc = configure_one<128, 1>() | configure_one<128, 2>() | configure_one<128, 4>() | configure_one<64, 1>() |
             configure_one<64, 2>() | configure_one<64, 4>() | configure_one<64, 8>();
    if (!rc) done[dev] = true;
    return rc ? -1 : 0;
}

int forge_attn_flat_launch(const ForgeAttnArgs& a, cudaStream_t stream, bool pdl) {
    if (!a.q || !a.kc || !a.vc || !a.pos || !a.partial || !a.counters || !a.out || a.table ||
        !forge_attn_flat_supported(a.B, a.H, a.Hkv, a.hd) || a.lmax <= 0 ||
        a.flat_slots < forge_attn_flat_slots(a.hd, a.lmax))
        return forge_fail(-1, "flat flash-decode: bad args");
    const int G = a.H / a.Hkv;
    if (a.hd == 128) {
        if (G == 1) return launch<128, 1>(a, stream, pdl);
        if (G == 2) return launch<128, 2>(a, stream, pdl);
        return launch<128, 4>(a, stream, pdl);
    }
    if (G == 1) return launch<64, 1>(a, stream, pdl);
    if (G == 2) return launch<64, 2>(a, stream, pdl);
    if (G == 4) return launch<64, 4>(a, stream, pdl);
    return launch<64, 8>(a, stream, pdl);
}
