// gemv_batched.cu — int4 decode GEMV for larger batches: the weights are
// streamed once per launch for up to 32 sequences.
//
// The small-batch kernel (gemv.cu) keeps every sequence's int8 activations
// in shared memory, which limits one launch to 4 sequences; a batch of 32
// would stream the weights 8 times. Here the activations are quantised once
// per sequence by k_quant_x into a global scratch (the same int8 hi/lo
// fragment order, per-group scales and column sums; the bytes are exactly
// those the small-batch staging produces), and k_gemv_b reads them from L2
// while each 16 KB weight piece in the TMA ring serves every column block of
// 4 sequences. Per-group arithmetic and the order of every sum match
// k_gemv, so results are bit-identical to the small-batch path.
#include <algorithm>
#include <cstdlib>
#include "common.cuh"
#include "layout.cuh"
#include "forge_internal.h"
#include "gemv_core.cuh"


namespace {
constexpr int kCW = 8;                      // consumer warps
constexpr int kThreads = (kCW + 1) * 32;    // + producer warp
constexpr int kStages = 4;
constexpr int kStageW = 16384, kStageS = 512, kStageBytes = kStageW + kStageS;
constexpr int kMaxSeq = 32;                 // sequences per launch (8 column blocks of 4)
constexpr int kRedFloats = 2 * kCW * 16 * kMaxSeq;

// One CTA per sequence: the staging of the small-batch kernel into shared
// memory (batch 1), then copied out to the batched global layout.
template <int PRO>
__global__ void __launch_bounds__(256) k_quant_x(const ForgeGemvArgs a, int nseq, uint8_t* xq_g, float* sx_g,
                                                 int* ss_g) {
    extern __shared__ __align__(16) uint8_t smem[];
    float* red = reinterpret_cast<float*>(smem);
    const int G = a.K / 128;
    float* sxf = red + 16;
    int* ssum = reinterpret_cast<int*>(sxf + G * 4);
    uint8_t* xq = reinterpret_cast<uint8_t*>(ssum + G * 8);
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x;
    ForgeGemvArgs s = a;
    s.batch = 1;
    s.b0 = a.b0 + b;
    s.x = a.x + (size_t)b * a.x_stride;
    stage_x_q8<PRO, 256>(s, xq, sxf, ssum, red);
    __syncthreads();
    const int ncols = 2 * nseq;
    for (int i = threadIdx.x; i < a.K / 2; i += 256) {  // words of 4 k, hi and lo columns
        const int k = (i >> 1) * 4, col = i & 1;
        *reinterpret_cast<uint32_t*>(xq_g + xq_index(k, 2 * b + col, ncols)) =
            *reinterpret_cast<const uint32_t*>(xq + xq_index(k, col, 2));
    }
    for (int g = threadIdx.x; g < G; g += 256) {
        sx_g[g * nseq + b] = sxf[g * 4];
        ss_g[g * 2 * nseq + 2 * b] = ssum[g * 8];
        ss_g[g * 2 * nseq + 2 * b + 1] = ssum[g * 8 + 1];
    }
}

// NCB: column blocks of 4 sequences per launch (2, 4 or 8), so the B-fragment
// loads of a group are all issued before its MMAs.
template <int EPI, int NCB>
__global__ void __launch_bounds__(kThreads, 1) k_gemv_b(const ForgeGemvArgs a, const uint8_t* __restrict__ xq_g,
                                                        const float* __restrict__ sx_g,
                                                        const int* __restrict__ ss_g) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    float* red = reinterpret_cast<float*>(empty + kStages);
    const int B = a.batch, G = a.K / 128;
    float* sxs = red + kRedFloats;              // [G][B]
    int* sss = reinterpret_cast<int*>(sxs + G * B);  // [G][2B]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KT = a.K >> 4;
    constexpr int kItemKT = 128;
    const int nitems = (KT + kItemKT - 1) / kItemKT;
    const int units = a.N >> 4;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == kCW) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            const uint8_t* wbase = static_cast<const uint8_t*>(a.w);
            const uint8_t* sbase = static_cast<const uint8_t*>(a.s);
            const int G4 = (KT / 8 + 3) / 4;
            uint32_t it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                for (int i = 0; i < nitems; ++i) {
                    const int s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, a.err)) { ok = false; break; }
                    const int kt0 = i * kItemKT, nkt = min(kItemKT, KT - kt0);
                    const uint32_t wb = (uint32_t)nkt * 128;
                    const uint32_t sb = (uint32_t)(((nkt / 8) + 3) / 4) * 128u;
                    mbar_arrive_expect_tx(&full[s], wb + sb);
                    bulk_g2s_stream(stages + s * kStageBytes, wbase + ((int64_t)u * KT + kt0) * 128, wb, &full[s], l2_evict_first());
                    bulk_g2s_stream(stages + s * kStageBytes + kStageW, sbase + ((int64_t)u * G4 + kt0 / 32) * 128, sb,
                                    &full[s], l2_evict_first());
                    ++it;
                }
            }
            for (uint32_t j = 0; j < (uint32_t)kStages && j < it; ++j) {
                const uint32_t idx = it - 1 - j;
                mbar_wait(&full[idx % kStages], (idx / kStages) & 1u, a.err);
            }
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    pdl_wait();
    for (int i = threadIdx.x; i < G * B; i += kCW * 32) sxs[i] = sx_g[i];
    for (int i = threadIdx.x; i < G * 2 * B; i += kCW * 32) sss[i] = ss_g[i];
    named_bar_sync(1, kCW * 32);

    const int g = lane >> 2, t = lane & 3;
    const int ncols = 2 * B;
    unsigned long long best = 0ull;
    uint32_t it = 0;
    int slot = 0;
    bool ok = true;
    // B fragments of this warp's two groups of piece i (they depend only on
    // the group, so every unit walks the same pieces). Up to 8 sequences
    // the next piece's are loaded from L2 before the current piece is
    // waited for and computed, hiding the L2 latency that bound this loop.
    auto load_b = [&](int i, uint4 (&bb)[2][NCB][2]) {
        const int kt0 = i * kItemKT, ngl = min(kItemKT, KT - kt0) / 8;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int gl = 2 * warp + h;
            if (gl < ngl) {
                const uint4* xg = reinterpret_cast<const uint4*>(xq_g) + (size_t)(2 * (kt0 / 8 + gl)) * ncols * 4;
#pragma unroll
                for (int cb = 0; cb < NCB; ++cb) {
                    const int col = min(cb * 8 + g, ncols - 1);
                    bb[h][cb][0] = __ldg(xg + (size_t)col * 4 + t);
                    bb[h][cb][1] = __ldg(xg + (size_t)(ncols + col) * 4 + t);
                }
            }
        }
    };
    constexpr bool kPrefetch = NCB <= 2;
    uint4 bcur[2][NCB][2], bnext[2][NCB][2];
    if (kPrefetch) load_b(0, bcur);
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, slot ^= 1) {
        float totA[NCB][2], totB[NCB][2];
#pragma unroll
        for (int c = 0; c < NCB; ++c) totA[c][0] = totA[c][1] = totB[c][0] = totB[c][1] = 0.f;
        for (int i = 0; i < nitems; ++i) {
            if (kPrefetch) load_b(i + 1 < nitems ? i + 1 : 0, bnext);
            const int s = it % kStages;
            const uint32_t ph = (it / kStages) & 1u;
            if (!mbar_wait(&full[s], ph, a.err)) { ok = false; break; }
            const int kt0 = i * kItemKT, nkt = min(kItemKT, KT - kt0);
            const uint8_t* st = stages + s * kStageBytes;
            const uint16_t* sst = reinterpret_cast<const uint16_t*>(st + kStageW);
            const int ng = nkt / 8;
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // this warp's groups 2w and 2w+1 of the piece
                const int gl = 2 * warp + h;
                if (gl < ng) {
                const int gg = kt0 / 8 + gl;
                const uint4 w0 = *reinterpret_cast<const uint4*>(st + (4 * warp + 2 * h) * 512 + lane * 16);
                const uint4 w1 = *reinterpret_cast<const uint4*>(st + (4 * warp + 2 * h + 1) * 512 + lane * 16);
                const uint32_t sc = *reinterpret_cast<const uint32_t*>(sst + (gl >> 2) * 64 + g * 8 + (gl & 3) * 2);
                uint32_t af[4][4];
                dequant_q4_u8(w0.x, w0.y, af[0]);
                dequant_q4_u8(w0.z, w0.w, af[1]);
                dequant_q4_u8(w1.x, w1.y, af[2]);
                dequant_q4_u8(w1.z, w1.w, af[3]);
                uint4 bf[NCB][2];
                if (kPrefetch) {
#pragma unroll
                    for (int cb = 0; cb < NCB; ++cb) {
                        bf[cb][0] = bcur[h][cb][0];
                        bf[cb][1] = bcur[h][cb][1];
                    }
                } else {
                    const uint4* xg = reinterpret_cast<const uint4*>(xq_g) + (size_t)(2 * gg) * ncols * 4;
#pragma unroll
                    for (int cb = 0; cb < NCB; ++cb) {
                        const int col = min(cb * 8 + g, ncols - 1);
                        bf[cb][0] = __ldg(xg + (size_t)col * 4 + t);
                        bf[cb][1] = __ldg(xg + (size_t)(ncols + col) * 4 + t);
                    }
                }
#pragma unroll
                for (int cb = 0; cb < NCB; ++cb) {
                    int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
                    mma_u8s8_16832(c0, af[0], bf[cb][0].x, bf[cb][0].y);
                    mma_u8s8_16832(c1, af[1], bf[cb][0].z, bf[cb][0].w);
                    mma_u8s8_16832(c0, af[2], bf[cb][1].x, bf[cb][1].y);
                    mma_u8s8_16832(c1, af[3], bf[cb][1].z, bf[cb][1].w);
                    const int sq = min(cb * 4 + t, B - 1);
                    const int shi = sss[gg * 2 * B + 2 * sq], slo = sss[gg * 2 * B + 2 * sq + 1];
                    const float sx = sxs[gg * B + sq];
                    // exact int -> float through the bits of 1.5 * 2^23 (|n| < 2^22), as in q4_group
                    auto i2f = [](int n) { return __fsub_rn(__int_as_float(n + 0x4B400000), 12582912.0f); };
                    const float v0 = i2f(c0[0] + c1[0] - 7 * shi) + i2f(c0[1] + c1[1] - 7 * slo) * (1.0f / 256.0f);
                    const float v1 = i2f(c0[2] + c1[2] - 7 * shi) + i2f(c0[3] + c1[3] - 7 * slo) * (1.0f / 256.0f);
                    const float y0 = bf16_lo_f32(sc) * sx * v0;
                    const float y1 = bf16_hi_f32(sc) * sx * v1;
                    if (h == 0) { totA[cb][0] += y0; totA[cb][1] += y1; }
                    else { totB[cb][0] += y0; totB[cb][1] += y1; }
                }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            ++it;
            if (kPrefetch) {
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int cb = 0; cb < NCB; ++cb) {
                        bcur[h][cb][0] = bnext[h][cb][0];
                        bcur[h][cb][1] = bnext[h][cb][1];
                    }
            }
        }
        if (!ok) break;
        // cross-warp reduction: lane (g, t) holds rows g / g+8 of sequences 4cb + t
        float* rw = red + (slot * kCW + warp) * 16 * kMaxSeq;
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) {
            const int sq = cb * 4 + t;
            if (sq < B) {
                rw[g * kMaxSeq + sq] = totA[cb][0] + totB[cb][0];
                rw[(g + 8) * kMaxSeq + sq] = totA[cb][1] + totB[cb][1];
            }
        }
        named_bar_sync(1, kCW * 32);
        const int tid = threadIdx.x;
        if (tid < 8 * B) {
            const int p = tid & 7, b = tid >> 3;
            const float* rs = red + slot * kCW * 16 * kMaxSeq;
            float ylo = 0.f, yhi = 0.f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) {
                ylo += rs[(w * 16 + p) * kMaxSeq + b];
                yhi += rs[(w * 16 + p + 8) * kMaxSeq + b];
            }
            epilogue<EPI>(a, u, p, b, ylo, yhi, best);
        }
    }
}

// bf16 weights: the activations as bf16 (no hi/lo split) in the mma.m16n8k16
// B-fragment order of the small-batch kernel, all sequences of the launch
// side by side (column = sequence).
template <int PRO>
__global__ void __launch_bounds__(256) k_conv_x(const ForgeGemvArgs a, int nseq, uint16_t* xf_g) {
    extern __shared__ __align__(16) uint8_t smem[];
    float* red = reinterpret_cast<float*>(smem);
    uint16_t* xf = reinterpret_cast<uint16_t*>(red + 16);
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x;
    ForgeGemvArgs s = a;
    s.batch = 1;
    s.split = 0;
    s.b0 = a.b0 + b;
    s.x = a.x + (size_t)b * a.x_stride;
    stage_x<PRO, 256>(s, xf, red);
    zero_x_pad<256>(s, xf);
    __syncthreads();
    const int kpad = (a.K + 31) / 32 * 32;
    for (int k = threadIdx.x; k < kpad; k += 256) xf_g[xf_index(k, b, nseq)] = xf[xf_index(k, 0, 1)];
}

template <int EPI, int NCB>  // NCB column blocks of 8 sequences
__global__ void __launch_bounds__(kThreads, 1) k_gemv_bf16_b(const ForgeGemvArgs a, const uint16_t* __restrict__ xf_g) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    float* red = reinterpret_cast<float*>(empty + kStages);
    const int B = a.batch;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KT = a.K >> 4;
    constexpr int kItemKT = 32;  // 16 KB pieces of 16x16 bf16 tiles
    const int nitems = (KT + kItemKT - 1) / kItemKT;
    const int units = a.N >> 4;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();
    if (warp == kCW) {
        if (lane == 0) {
            const uint8_t* wbase = static_cast<const uint8_t*>(a.w);
            uint32_t it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                for (int i = 0; i < nitems; ++i) {
                    const int s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, a.err)) { ok = false; break; }
                    const int kt0 = i * kItemKT, nkt = min(kItemKT, KT - kt0);
                    const uint32_t wb = (uint32_t)nkt * 512;
                    mbar_arrive_expect_tx(&full[s], wb);
                    bulk_g2s_stream(stages + s * kStageBytes, wbase + ((int64_t)u * KT + kt0) * 512, wb, &full[s], l2_evict_first());
                    ++it;
                }
            }
            for (uint32_t j = 0; j < (uint32_t)kStages && j < it; ++j) {
                const uint32_t idx = it - 1 - j;
                mbar_wait(&full[idx % kStages], (idx / kStages) & 1u, a.err);
            }
        }
        return;
    }
    pdl_wait();
    const int g = lane >> 2, t = lane & 3;
    const int ncols = B;
    unsigned long long best = 0ull;
    uint32_t it = 0;
    int slot = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, slot ^= 1) {
        float tot[NCB][4], tot2[NCB][4];
#pragma unroll
        for (int c = 0; c < NCB; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) tot[c][e] = tot2[c][e] = 0.f;
        for (int i = 0; i < nitems; ++i) {
            const int s = it % kStages;
            const uint32_t ph = (it / kStages) & 1u;
            if (!mbar_wait(&full[s], ph, a.err)) { ok = false; break; }
            const int kt0 = i * kItemKT, nkt = min(kItemKT, KT - kt0);
            const uint8_t* st = stages + s * kStageBytes;
            const int ktw = 4 * warp;  // warp w: k-tiles 4w .. 4w+3 (two pairs)
            if (ktw < nkt) {
                const int kp = (kt0 + ktw) >> 1;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    if (ktw + 2 * j < nkt) {
                        const uint4 a0 = *reinterpret_cast<const uint4*>(st + (ktw + 2 * j) * 512 + lane * 16);
                        const uint4 a1 = (ktw + 2 * j + 1 < nkt)
                            ? *reinterpret_cast<const uint4*>(st + (ktw + 2 * j + 1) * 512 + lane * 16)
                            : make_uint4(0, 0, 0, 0);
                        const uint32_t f0[4] = {a0.x, a0.y, a0.z, a0.w};
                        const uint32_t f1[4] = {a1.x, a1.y, a1.z, a1.w};
                        const uint4* xg = reinterpret_cast<const uint4*>(xf_g) + (size_t)(kp + j) * ncols * 4;
                        uint4 bb[NCB];
#pragma unroll
                        for (int cb = 0; cb < NCB; ++cb) bb[cb] = __ldg(xg + (size_t)min(cb * 8 + g, ncols - 1) * 4 + t);
#pragma unroll
                        for (int cb = 0; cb < NCB; ++cb) {
                            mma_bf16_16816(tot[cb], f0, bb[cb].x, bb[cb].y, tot[cb]);
                            mma_bf16_16816(tot2[cb], f1, bb[cb].z, bb[cb].w, tot2[cb]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            ++it;
        }
        if (!ok) break;
        // lane (g, t) holds rows g / g+8 of sequences 8cb + 2t and 8cb + 2t + 1
        float* rw = red + (slot * kCW + warp) * 16 * kMaxSeq;
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) {
            const int sq = cb * 8 + 2 * t;
            if (sq < B) {
                rw[g * kMaxSeq + sq] = tot[cb][0] + tot2[cb][0];
                rw[(g + 8) * kMaxSeq + sq] = tot[cb][2] + tot2[cb][2];
            }
            if (sq + 1 < B) {
                rw[g * kMaxSeq + sq + 1] = tot[cb][1] + tot2[cb][1];
                rw[(g + 8) * kMaxSeq + sq + 1] = tot[cb][3] + tot2[cb][3];
            }
        }
        named_bar_sync(1, kCW * 32);
        const int tid = threadIdx.x;
        if (tid < 8 * B) {
            const int p = tid & 7, b = tid >> 3;
            const float* rs = red + slot * kCW * 16 * kMaxSeq;
            float ylo = 0.f, yhi = 0.f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) {
                ylo += rs[(w * 16 + p) * kMaxSeq + b];
                yhi += rs[(w * 16 + p + 8) * kMaxSeq + b];
            }
            epilogue<EPI>(a, u, p, b, ylo, yhi, best);
        }
    }
    if (EPI == FORGE_EPI_LOGITS) {
        // thread (p, b) = (tid & 7, tid >> 3): reduce over the 8 row pairs
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
            best = v > best ? v : best;
        }
        const int tid = threadIdx.x;
        if ((tid & 7) == 0 && (tid >> 3) < B && best != 0ull) atomicMax(a.argmax_key + a.b0 + (tid >> 3), best);
    }
}

template <int EPI, int NCB>
int launch_bf(const ForgeGemvArgs& a, const uint16_t* xf, cudaStream_t stream, int smem) {
    const int units = a.N / 16;
    int grid = forge_sm_count();
    if (grid > units) grid = units;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemv_bf16_b<EPI, NCB>, a, xf);
    return e == cudaSuccess ? 0 : forge_fail(-1, "batched bf16 gemv launch: %s", cudaGetErrorString(e));
}

template <int EPI>
int launch_bfn(const ForgeGemvArgs& a, const uint16_t* xf, cudaStream_t stream, int smem) {
    if (a.batch <= 8) return launch_bf<EPI, 1>(a, xf, stream, smem);
    if (a.batch <= 16) return launch_bf<EPI, 2>(a, xf, stream, smem);
    return launch_bf<EPI, 4>(a, xf, stream, smem);
}

template <int EPI, int NCB>
int launch_b(const ForgeGemvArgs& a, const uint8_t* xq, const float* sx, const int* ss, cudaStream_t stream, bool pdl,
             int smem) {
    const int units = a.N / 16;
    int grid = forge_sm_count();
    if (grid > units) grid = units;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemv_b<EPI, NCB>, a, xq, sx, ss);
    return e == cudaSuccess ? 0 : forge_fail(-1, "batched gemv launch: %s", cudaGetErrorString(e));
}

template <int EPI>
int launch_bn(const ForgeGemvArgs& a, const uint8_t* xq, const float* sx, const int* ss, cudaStream_t stream,
              bool pdl, int smem) {
    if (a.batch <= 8) return launch_b<EPI, 2>(a, xq, sx, ss, stream, pdl, smem);
    if (a.batch <= 16) return launch_b<EPI, 4>(a, xq, sx, ss, stream, pdl, smem);
    return launch_b<EPI, 8>(a, xq, sx, ss, stream, pdl, smem);
}

template <int PRO>
int launch_q(const ForgeGemvArgs& a, int nseq, uint8_t* xq, float* sx, int* ss, cudaStream_t stream, bool pdl) {
    const int smem = 16 * 4 + (a.K / 128) * 12 * 4 + a.K * 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nseq);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_quant_x<PRO>, a, nseq, xq, sx, ss);
    return e == cudaSuccess ? 0 : forge_fail(-1, "activation quantise launch: %s", cudaGetErrorString(e));
}

constexpr int smem_b(int K, int B) {
    return kStages * kStageBytes + 2 * kStages * 8 + kRedFloats * 4 + (K / 128) * B * 12;
}
}  // namespace

int forge_gemv_b_max_seq() { return kMaxSeq; }

// int4 chunks of at least this many sequences run on the tensor cores
// (gemv_tc.cu); smaller ones on the register-fragment kernel above. Measured
// on the 7B decode step: 32 sequences 2944 vs 2915 tok/s, 16 sequences 2022
// vs 2408, 8 sequences 1338 vs 1700. FORGE_GEMV_TC_MIN_SEQ overrides (1 runs
// every chunk on the tensor cores).
static int tc_min_seq() {
    static int v = [] {
        const char* e = getenv("FORGE_GEMV_TC_MIN_SEQ");
        const int x = e ? atoi(e) : 0;
        return x > 0 ? x : 24;
    }();
    return v;
}

int64_t forge_gemv_b_scratch_bytes(int K) {
    // int4: int8 hi/lo [K][2 x 32] + scales and sums; bf16: [K padded to 32][32] bf16
    const int64_t q4 = (int64_t)K * 2 * kMaxSeq + (int64_t)(K / 128) * kMaxSeq * 12 + 256;
    const int64_t bf = (int64_t)((K + 31) / 32 * 32) * 2 * kMaxSeq + 256;
    const int64_t tc = forge_gemv_tc_scratch_bytes(K);
    return std::max({q4 + forge_gemv_scratch_header(), bf + forge_gemv_scratch_header(), tc});
}

int forge_gemv_b_configure() {
    static bool done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return forge_fail(-1, "batched gemv: no device");
    if (done[dev]) return 0;
    const int mx = 227 * 1024;
    cudaError_t e = cudaSuccess;
    auto set = [&](const void* f) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    };
#define FORGE_SET_B(E) \
    set((const void*)k_gemv_b<E, 2>); set((const void*)k_gemv_b<E, 4>); set((const void*)k_gemv_b<E, 8>)
    FORGE_SET_B(FORGE_EPI_STORE);
    FORGE_SET_B(FORGE_EPI_RESID);
    FORGE_SET_B(FORGE_EPI_QKV);
    FORGE_SET_B(FORGE_EPI_SWIGLU);
#undef FORGE_SET_B
    set((const void*)k_quant_x<FORGE_PRO_PLAIN>);
    set((const void*)k_quant_x<FORGE_PRO_RMSNORM>);
    set((const void*)k_conv_x<FORGE_PRO_PLAIN>);
    set((const void*)k_conv_x<FORGE_PRO_RMSNORM>);
#define FORGE_SET_BF(E) \
    set((const void*)k_gemv_bf16_b<E, 1>); set((const void*)k_gemv_bf16_b<E, 2>); set((const void*)k_gemv_bf16_b<E, 4>)
    FORGE_SET_BF(FORGE_EPI_STORE);
    FORGE_SET_BF(FORGE_EPI_RESID);
    FORGE_SET_BF(FORGE_EPI_QKV);
    FORGE_SET_BF(FORGE_EPI_SWIGLU);
    FORGE_SET_BF(FORGE_EPI_LOGITS);
#undef FORGE_SET_BF
    if (e != cudaSuccess) return forge_fail(-1, "batched gemv: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    if (forge_gemv_tc_configure()) return -1;
    done[dev] = true;
    return 0;
}

// One chunk of up to kMaxSeq sequences: quantise, then one weight stream.
// scratch: forge_gemv_b_scratch_bytes(K) bytes of device memory.
int forge_gemv_b_launch(const ForgeGemvArgs& a, void* scratch_all, cudaStream_t stream, bool pdl) {
    if (a.batch <= 0 || a.batch > kMaxSeq || !scratch_all)
        return forge_fail(-1, "batched gemv: 1..%d sequences and a scratch buffer", kMaxSeq);
    // the header of the scratch belongs to the tensor-core path
    void* scratch = static_cast<uint8_t*>(scratch_all) + forge_gemv_scratch_header();
    if (a.wkind == FORGE_W_BF16) {
        if (a.split || a.pro == FORGE_PRO_EMBED_RMSNORM)
            return forge_fail(-1, "batched bf16 gemv: bf16 activations and plain/RMSNorm prologue only");
        uint16_t* xf = static_cast<uint16_t*>(scratch);
        const int kpad = (a.K + 31) / 32 * 32;
        const int qsmem = 16 * 4 + kpad * 2;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(a.batch);
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = qsmem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        cudaError_t e = a.pro == FORGE_PRO_RMSNORM ? cudaLaunchKernelEx(&cfg, k_conv_x<FORGE_PRO_RMSNORM>, a, a.batch, xf)
                                                   : cudaLaunchKernelEx(&cfg, k_conv_x<FORGE_PRO_PLAIN>, a, a.batch, xf);
        if (e != cudaSuccess) return forge_fail(-1, "activation convert launch: %s", cudaGetErrorString(e));
        const int smem = kStages * kStageBytes + 2 * kStages * 8 + kRedFloats * 4;
        switch (a.epi) {
        case FORGE_EPI_STORE: return launch_bfn<FORGE_EPI_STORE>(a, xf, stream, smem);
        case FORGE_EPI_RESID: return launch_bfn<FORGE_EPI_RESID>(a, xf, stream, smem);
        case FORGE_EPI_QKV: return launch_bfn<FORGE_EPI_QKV>(a, xf, stream, smem);
        case FORGE_EPI_SWIGLU: return launch_bfn<FORGE_EPI_SWIGLU>(a, xf, stream, smem);
        case FORGE_EPI_LOGITS: return launch_bfn<FORGE_EPI_LOGITS>(a, xf, stream, smem);
        default: return forge_fail(-1, "batched bf16 gemv: unknown epilogue %d", a.epi);
        }
    }
    if (a.wkind != FORGE_W_Q4) return forge_fail(-1, "batched gemv: unknown weight kind");
    if (a.pro == FORGE_PRO_EMBED_RMSNORM || a.epi == FORGE_EPI_LOGITS)
        return forge_fail(-1, "batched gemv: prologue/epilogue not supported");
    if (a.batch >= tc_min_seq()) return forge_gemv_tc_launch(a, scratch_all, stream, pdl);
    const int smem = smem_b(a.K, a.batch);
    if (smem > 227 * 1024) return forge_fail(-1, "batched gemv: K=%d too large", a.K);
    uint8_t* xq = static_cast<uint8_t*>(scratch);
    float* sx = reinterpret_cast<float*>(xq + (size_t)a.K * 2 * kMaxSeq);
    int* ss = reinterpret_cast<int*>(sx + (size_t)(a.K / 128) * kMaxSeq);
    int rc = a.pro == FORGE_PRO_RMSNORM ? launch_q<FORGE_PRO_RMSNORM>(a, a.batch, xq, sx, ss, stream, pdl)
                                        : launch_q<FORGE_PRO_PLAIN>(a, a.batch, xq, sx, ss, stream, pdl);
    if (rc) return rc;
    switch (a.epi) {
    case FORGE_EPI_STORE: return launch_bn<FORGE_EPI_STORE>(a, xq, sx, ss, stream, true, smem);
    case FORGE_EPI_RESID: return launch_bn<FORGE_EPI_RESID>(a, xq, sx, ss, stream, true, smem);
    case FORGE_EPI_QKV: return launch_bn<FORGE_EPI_QKV>(a, xq, sx, ss, stream, true, smem);
    case FORGE_EPI_SWIGLU: return launch_bn<FORGE_EPI_SWIGLU>(a, xq, sx, ss, stream, true, smem);
    default: return forge_fail(-1, "batched gemv: unknown epilogue %d", a.epi);
    }
}
