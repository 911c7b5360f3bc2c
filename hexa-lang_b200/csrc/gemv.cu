// gemv.cu — decode GEMV for sm_100a: y = W x for a handful of sequences,
// W int4 (group-128, bf16 scales) or bf16, packed per layout.cuh.
//
// Replaces forge's _hx_k_packed_gemv_offset[_f32/_bf16]
// (self/cuda/runtime_cuda_emit.hexa:1245-1389, host :1858-1967) for every
// projection of the decode step, with the step's elementwise work fused in:
//   prologue  RMSNorm of the fp32 residual stream (nn_lib.hexa:150-171)
//   epilogue  QKV: RoPE (nn_lib.hexa:541-562) + KV-cache append + q out
//             SwiGLU: silu(gate) * up (nn_lib.hexa:385-412)
//             RESID: residual add (decoder_block_lib.hexa:431-440)
//             LOGITS: LM head logits + first-max argmax (decoder_lib.hexa:485-500)
//
// Structure (one CTA per SM, persistent over 16-row units):
//   warp 8 (producer)  streams each unit's weight tiles in 16 KB pieces (plus
//                      their 512 B of int4 scales) with cp.async.bulk into a
//                      4-stage mbarrier ring; it never waits on the previous
//                      kernel, so under programmatic dependent launch the next
//                      kernel's weights are in flight while the previous one
//                      drains.
//   warps 0-7          stage the activations once per CTA (RMSNorm in the same
//                      pass; int4: int8 hi/lo pairs per 128-group, bf16: hi/lo
//                      bf16) — or, for int4 when the kernel before has staged
//                      them into a block (ForgeGemvArgs::pq_in), copy that
//                      block with one bulk copy, folding the RMSNorm factor
//                      into the group scales — then for every piece take A
//                      fragments straight from the packed weights (int4: two
//                      LOP3 per register into mma.sync.m16n8k32 u8 x s8;
//                      bf16: mma.sync.m16n8k16) with the activations as B
//                      operand.
//   The eight warps split each piece along K (two 128-groups per warp for
//   int4); a shared-memory reduction and the fused epilogue finish each unit.
// Why mma.sync: at batch 1-4 the GEMV has 1-8 columns; a tcgen05 MMA needs
// M >= 64 rows of A in shared memory or TMEM, so the int4 codes would have to
// be expanded on chip before every MMA, while the register-fragment path
// consumes them as they land in the ring.
#include <cstdio>
#include <cstdlib>
#include "common.cuh"
#include "layout.cuh"
#include "forge_internal.h"
#include "gemv_core.cuh"

namespace {
#ifndef FORGE_GEMV_STAGES
#define FORGE_GEMV_STAGES 4
#endif
// Registers per thread: 112 (the compiler's free choice was 148-166). The
// register file is split over four sub-partitions of 16K registers and a
// 9-warp CTA puts three warps on one of them; at 112 a GEMV CTA and a
// flash-decode CTA (72) fit one SM together, so under programmatic dependent
// launch the attention kernel's KV stream starts while the QKV projection
// runs. Two GEMV CTAs would need 96 or fewer, which was measured slower
// (the weight stream of the next GEMV overlaps less than the lost registers
// cost in the MMA loop).
#ifndef FORGE_GEMV_MAXNREG
#define FORGE_GEMV_MAXNREG 112
#endif
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = FORGE_GEMV_STAGES;
constexpr int kStageW = 16384;                        // weight bytes per piece
constexpr int kStageS = 512;                          // q4 scale bytes per piece (16 groups)
constexpr int kStageBytes = kStageW + kStageS;
constexpr int kRedFloats = 2 * kConsumerWarps * 16 * 8;  // two unit slots
constexpr int kMaxG = 128;                            // K <= 16384 (staging keeps K/4/threads float4 in registers)
constexpr int kFixedSmem = kStages * kStageBytes + 2 * kStages * 8 + 16 + kRedFloats * 4;
constexpr int kMaxSmem = 227 * 1024;

__device__ __forceinline__ void sys_store_release(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t sys_load_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// FORGE_EPI_RESID_TP, run by warp 0 of a CTA (lane (p, b) for p < 8 and
// b < batch <= 4 holds rows p / p+8 of sequence b of 16-row tile u).
// tp_resid_post, when the CTA has reduced tile u: the tile's share goes into
// this rank's slot on every rank (rank 0's share carries the residual, the
// additions of its FORGE_EPI_RESID) with plain stores, no fence.
// tp_resid_flags, once the CTA has stored all its tiles: one system-scope
// fence for all of them, then a flag per (rank, tile) on every rank says
// they landed. tp_resid_finish: when every rank's flag for the tile is in,
// the slots are summed in rank order — the additions of the separate
// all-reduce, so the result is the same — into the residual. One fence per
// CTA instead of one per tile keeps the NVLink round trip of the fence off
// the CTA's remaining units. The per-tile call counter selects one of two
// buffer generations: a rank can be at most one call ahead of another on a
// tile, because its launch ends only after every rank's share of its tiles
// arrived. Waits are bounded (error word).
__device__ __noinline__ void tp_resid_post(const ForgeGemvArgs& a, int u, int p, int b, bool act, float ylo,
                                           float yhi) {
    const ForgeTpFusedDev& f = *a.tpf;
    const int lane = threadIdx.x & 31;
    const int T = f.T, rank = f.rank;
    uint32_t ep = 0;
    if (lane == 0) ep = ++f.tile_epoch[u];
    ep = __shfl_sync(0xffffffffu, ep, 0);
    const int gen = ep & 1;
    const size_t i0 = (size_t)b * a.y_stride + (size_t)u * 16 + p, i1 = i0 + 8;
    if (act) {
        float v0 = ylo, v1 = yhi;
        if (rank == 0) {
            v0 = a.y[i0] + ylo;
            v1 = a.y[i1] + yhi;
        }
        for (int r = 0; r < T; ++r) {
            float* dst = f.buf[r] + ((size_t)gen * T + rank) * f.cap;
            dst[i0] = v0;
            dst[i1] = v1;
        }
    }
}

__device__ __noinline__ void tp_resid_flags(const ForgeGemvArgs& a, int units) {
    const ForgeTpFusedDev& f = *a.tpf;
    const int lane = threadIdx.x & 31;
    const int T = f.T, rank = f.rank;
    __threadfence_system();  // every lane's remote stores of every tile of this CTA
    __syncwarp();
    if (lane < T)
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            const uint32_t ep = f.tile_epoch[u];
            sys_store_release(f.flag[lane] + ((size_t)(ep & 1) * T + rank) * f.max_tiles + u, ep);
        }
}

__device__ __noinline__ void tp_resid_finish(const ForgeGemvArgs& a, int u, int p, int b, bool act) {
    const ForgeTpFusedDev& f = *a.tpf;
    const int lane = threadIdx.x & 31;
    const int T = f.T, rank = f.rank;
    uint32_t ep = 0;
    if (lane == 0) ep = f.tile_epoch[u];  // this call's, set by tp_resid_post
    ep = __shfl_sync(0xffffffffu, ep, 0);
    const int gen = ep & 1;
    const size_t i0 = (size_t)b * a.y_stride + (size_t)u * 16 + p, i1 = i0 + 8;
    bool ok = true;
    if (lane < T) {
        const volatile uint32_t* fl = f.flag[rank] + ((size_t)gen * T + lane) * f.max_tiles + u;
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (*fl != ep) {
            if ((++spins & 1023u) == 0 && globaltimer_ns() - t0 > FORGE_WAIT_NS) {
                atomicOr(a.err, FORGE_DEVERR_COUNTER_TIMEOUT);
                ok = false;
                break;
            }
        }
        (void)sys_load_acquire(const_cast<const uint32_t*>(fl));
    }
    ok = __all_sync(0xffffffffu, ok);
    if (ok && act) {
        const float* base = f.buf[rank] + (size_t)gen * T * f.cap;
        float s0 = __ldcv(base + i0), s1 = __ldcv(base + i1);
        for (int r = 1; r < T; ++r) {
            s0 += __ldcv(base + (size_t)r * f.cap + i0);
            s1 += __ldcv(base + (size_t)r * f.cap + i1);
        }
        a.y[i0] = s0;
        a.y[i1] = s1;
    }
}

template <int WK, int PRO, int EPI>
__global__ void __maxnreg__(FORGE_GEMV_MAXNREG) k_gemv(const ForgeGemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* pq_bar = empty + kStages;  // the handoff copy (16 bytes with padding)
    float* red = reinterpret_cast<float*>(pq_bar + 2);
    // int4: per-group activation scales [G][4] and column sums [G][8], then
    // the int8 activations; bf16: the bf16 hi/lo activations
    float* sxf = red + kRedFloats;
    int* ssum = reinterpret_cast<int*>(sxf + (WK == FORGE_W_Q4 ? (a.K / 128) * 4 : 0));
    uint16_t* xf = reinterpret_cast<uint16_t*>(ssum + (WK == FORGE_W_Q4 ? (a.K / 128) * 8 : 0));
    uint8_t* xq = reinterpret_cast<uint8_t*>(xf);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KT = a.K >> 4;
    constexpr int kItemKT = (WK == FORGE_W_Q4) ? 128 : 32;
    constexpr int kTileBytes = (WK == FORGE_W_Q4) ? 128 : 512;  // per 16x16 tile
    const int nitems = (KT + kItemKT - 1) / kItemKT;
    const int units = a.N >> 4;

    if (threadIdx.x == 0) {
        if (a.trace) a.trace[blockIdx.x * 4 + 0] = globaltimer_ns();
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(pq_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = l2_evict_first();
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
                    const uint32_t wb = (uint32_t)nkt * kTileBytes;
                    uint32_t sb = 0;
                    if (WK == FORGE_W_Q4) sb = (uint32_t)(((nkt / 8) + 3) / 4) * 128u;
                    mbar_arrive_expect_tx(&full[s], wb + sb);
                    bulk_g2s_stream(stages + s * kStageBytes, wbase + ((int64_t)u * KT + kt0) * kTileBytes, wb,
                                    &full[s], pol);
                    if (WK == FORGE_W_Q4)
                        bulk_g2s_stream(stages + s * kStageBytes + kStageW,
                                        sbase + ((int64_t)u * G4 + kt0 / 32) * 128, sb, &full[s], pol);
                    ++it;
                }
            }
            // Drain: every copy issued must land before the CTA exits.
            for (uint32_t j = 0; j < (uint32_t)kStages && j < it; ++j) {
                const uint32_t idx = it - 1 - j;
                mbar_wait(&full[idx % kStages], (idx / kStages) & 1u, a.err);
            }
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    pdl_wait();
    if (a.trace && threadIdx.x == 0) a.trace[blockIdx.x * 4 + 1] = globaltimer_ns();
    if (WK == FORGE_W_Q4 && (PRO == FORGE_PRO_PLAIN || (PRO == FORGE_PRO_RMSNORM && a.pq_ssq)) && a.pq_in) {
        // the previous kernel staged the activations: one copy of its block
        if (threadIdx.x == 0) {
            const uint32_t bytes = (uint32_t)forge_pq_bytes(a.K, a.batch);
            mbar_arrive_expect_tx(pq_bar, bytes);
            bulk_g2s(sxf, a.pq_in, bytes, pq_bar);
        }
        if (PRO == FORGE_PRO_RMSNORM) {
            // RMSNorm factor of sequence b (warp b) from the groups' sums of
            // squares, in the same order in every CTA, folded into the
            // group scales
            float* invs = red + kRedFloats - 8;
            const int G = a.K >> 7;
            if (warp < a.batch) {
                float tot = 0.f;
                for (int g = lane; g < G; g += 32) tot += __ldcg(a.pq_ssq + warp * G + g);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
                if (lane == 0) invs[warp] = 1.0f / sqrtf(tot / (float)a.K + a.eps);
            }
            mbar_wait(pq_bar, 0, a.err);
            named_bar_sync(1, 256);
            for (int i = threadIdx.x; i < G * a.batch; i += 256) sxf[(i / a.batch) * 4 + i % a.batch] *= invs[i % a.batch];
        } else {
            mbar_wait(pq_bar, 0, a.err);
        }
    } else if (WK == FORGE_W_Q4) {
        stage_x_q8<PRO, 256>(a, xq, sxf, ssum, red);
    } else {
        stage_x<PRO, 256>(a, xf, red);
        zero_x_pad<256>(a, xf);
    }
    named_bar_sync(1, 256);
    if (a.trace && threadIdx.x == 0) a.trace[blockIdx.x * 4 + 2] = globaltimer_ns();

    const int g = lane >> 2, t = lane & 3;
    const int ncols = (WK == FORGE_W_Q4 || a.split) ? 2 * a.batch : a.batch;
    constexpr int RC = (WK == FORGE_W_Q4) ? 4 : 8;  // reduction columns per row
    const int col = g < ncols ? g : ncols - 1;  // unused columns re-read a valid one
    const int c0 = min(2 * t, ncols - 1), c1 = min(2 * t + 1, ncols - 1);
    unsigned long long best = 0ull;
    uint32_t it = 0;
    int slot = 0;
    bool ok = true;

    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, slot ^= 1) {
        float tot[4] = {0.f, 0.f, 0.f, 0.f};
        float tot2[4] = {0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < nitems; ++i) {
            const int s = it % kStages;
            const uint32_t ph = (it / kStages) & 1u;
            if (!mbar_wait(&full[s], ph, a.err)) { ok = false; break; }
            const int kt0 = i * kItemKT, nkt = min(kItemKT, KT - kt0);
            const uint8_t* st = stages + s * kStageBytes;
            if (WK == FORGE_W_Q4) {
                // warp w: groups 2w and 2w+1 of this piece (int8 tensor-core path)
                const int ng = nkt / 8;
                const int gA = 2 * warp;
                const uint16_t* sst = reinterpret_cast<const uint16_t*>(st + kStageW);
                const int ggA = kt0 / 8 + gA;
                if (gA + 1 < ng) {
                    // both groups in one block so their loads and MMAs interleave
                    const uint4 wA0 = *reinterpret_cast<const uint4*>(st + (4 * warp + 0) * 512 + lane * 16);
                    const uint4 wA1 = *reinterpret_cast<const uint4*>(st + (4 * warp + 1) * 512 + lane * 16);
                    const uint4 wB0 = *reinterpret_cast<const uint4*>(st + (4 * warp + 2) * 512 + lane * 16);
                    const uint4 wB1 = *reinterpret_cast<const uint4*>(st + (4 * warp + 3) * 512 + lane * 16);
                    const uint32_t scA = *reinterpret_cast<const uint32_t*>(sst + (gA >> 2) * 64 + g * 8 + (gA & 3) * 2);
                    const int gB = gA + 1;
                    const uint32_t scB = *reinterpret_cast<const uint32_t*>(sst + (gB >> 2) * 64 + g * 8 + (gB & 3) * 2);
                    float yA0, yA1, yB0, yB1;
                    q4_group(wA0, wA1, xq, ggA, ncols, col, t, scA, sxf, ssum, a.batch, yA0, yA1);
                    q4_group(wB0, wB1, xq, ggA + 1, ncols, col, t, scB, sxf, ssum, a.batch, yB0, yB1);
                    tot[0] += yA0;
                    tot[1] += yA1;
                    tot2[0] += yB0;
                    tot2[1] += yB1;
                } else if (gA < ng) {
                    const uint4 w0 = *reinterpret_cast<const uint4*>(st + (4 * warp + 0) * 512 + lane * 16);
                    const uint4 w1 = *reinterpret_cast<const uint4*>(st + (4 * warp + 1) * 512 + lane * 16);
                    const uint32_t sc = *reinterpret_cast<const uint32_t*>(sst + (gA >> 2) * 64 + g * 8 + (gA & 3) * 2);
                    float y0, y1;
                    q4_group(w0, w1, xq, ggA, ncols, col, t, sc, sxf, ssum, a.batch, y0, y1);
                    tot[0] += y0;
                    tot[1] += y1;
                }
            } else {
                // warp w: k-tiles 4w .. 4w+3 (two pairs), two accumulator chains
                const int ktw = 4 * warp;
                if (ktw < nkt) {
                    const int kp = (kt0 + ktw) >> 1;
                    const uint4* xa = reinterpret_cast<const uint4*>(xf) + (size_t)(kp * ncols + col) * 4 + t;
                    const size_t pstride = (size_t)ncols * 4;
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        if (ktw + 2 * j < nkt) {
                            const uint4 a0 = *reinterpret_cast<const uint4*>(st + (ktw + 2 * j) * 512 + lane * 16);
                            // the odd last k-tile of a K/16-odd matrix has no partner in the piece
                            const uint4 a1 = (ktw + 2 * j + 1 < nkt)
                                ? *reinterpret_cast<const uint4*>(st + (ktw + 2 * j + 1) * 512 + lane * 16)
                                : make_uint4(0, 0, 0, 0);
                            const uint4 bb = xa[j * pstride];
                            const uint32_t f0[4] = {a0.x, a0.y, a0.z, a0.w};
                            const uint32_t f1[4] = {a1.x, a1.y, a1.z, a1.w};
                            mma_bf16_16816(tot, f0, bb.x, bb.y, tot);
                            mma_bf16_16816(tot2, f1, bb.z, bb.w, tot2);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            ++it;
        }
        if (!ok) break;
        // cross-warp reduction through one of two slots: one barrier per unit;
        // warps 0-1 run the epilogue while the others start the next unit
        float* rw = red + (slot * kConsumerWarps + warp) * 16 * RC;
        if (WK == FORGE_W_Q4) {  // lane (g, t): rows g / g+8 of sequence t
            if (t < a.batch) {
                rw[g * RC + t] = tot[0] + tot2[0];
                rw[(g + 8) * RC + t] = tot[1] + tot2[1];
            }
        } else {
            rw[g * 8 + 2 * t] = tot[0] + tot2[0];
            rw[g * 8 + 2 * t + 1] = tot[1] + tot2[1];
            rw[(g + 8) * 8 + 2 * t] = tot[2] + tot2[2];
            rw[(g + 8) * 8 + 2 * t + 1] = tot[3] + tot2[3];
        }
        named_bar_sync(1, 256);
        const int tid = threadIdx.x;
        const bool act = tid < 8 * a.batch;
        // FORGE_EPI_RESID_TP (batch <= 4): all of warp 0 takes part
        if (act || (EPI == FORGE_EPI_RESID_TP && warp == 0)) {
            const int p = tid & 7, b = tid >> 3;
            const float* rs = red + slot * kConsumerWarps * 16 * RC;
            float ylo = 0.f, yhi = 0.f;
            if (!act) {
            } else if (WK == FORGE_W_Q4) {
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) {
                    ylo += rs[(w * 16 + p) * RC + b];
                    yhi += rs[(w * 16 + p + 8) * RC + b];
                }
            } else {
                const int c = a.split ? 2 * b : b;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) {
                    ylo += rs[(w * 16 + p) * 8 + c];
                    yhi += rs[(w * 16 + p + 8) * 8 + c];
                    if (a.split) {
                        ylo += rs[(w * 16 + p) * 8 + c + 1];
                        yhi += rs[(w * 16 + p + 8) * 8 + c + 1];
                    }
                }
            }
            if (EPI == FORGE_EPI_RESID_TP)
                tp_resid_post(a, u, p, b, act, ylo, yhi);
            else
                epilogue<EPI>(a, u, p, b, ylo, yhi, best);
        }
    }
    if (a.trace && threadIdx.x == 0) a.trace[blockIdx.x * 4 + 3] = globaltimer_ns();
    if (EPI == FORGE_EPI_RESID_TP && warp == 0) {
        const int tid = threadIdx.x;
        tp_resid_flags(a, units);  // also after a failed wait: the tiles that were posted
        if (__all_sync(0xffffffffu, ok))
            for (int u = blockIdx.x; u < units; u += gridDim.x)
                tp_resid_finish(a, u, tid & 7, tid >> 3, tid < 8 * a.batch);
    }

    if (EPI == FORGE_EPI_LOGITS && warp < 2) {
        // thread (p, b) = (tid & 7, tid >> 3): reduce over the 8 row pairs
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
            best = v > best ? v : best;
        }
        const int tid = threadIdx.x;
        if ((tid & 7) == 0 && (tid >> 3) < a.batch && best != 0ull)
            atomicMax(a.argmax_key + a.b0 + (tid >> 3), best);
    }
}

template <int WK, int PRO, int EPI>
int configure_one() {
    cudaError_t e = cudaFuncSetAttribute(k_gemv<WK, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    // every decode kernel asks for the largest shared-memory carveout, so an
    // SM never has to be reconfigured (which needs it idle) before the next
    // kernel's CTA can join the one still running there
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_gemv<WK, PRO, EPI>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
    return e == cudaSuccess ? 0 : forge_fail(-1, "gemv: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
}
template <int WK, int PRO>
int configure_epi() {
    return configure_one<WK, PRO, FORGE_EPI_STORE>() | configure_one<WK, PRO, FORGE_EPI_RESID>() |
           configure_one<WK, PRO, FORGE_EPI_QKV>() | configure_one<WK, PRO, FORGE_EPI_SWIGLU>() |
           configure_one<WK, PRO, FORGE_EPI_LOGITS>() | configure_one<WK, PRO, FORGE_EPI_RESID_TP>();
}

template <int WK, int PRO, int EPI>
int launch_one(const ForgeGemvArgs& a, cudaStream_t stream, bool pdl, int smem) {
    auto kern = k_gemv<WK, PRO, EPI>;
    const int units = a.N / 16;
    static int ctas_per_sm = 0;
    if (!ctas_per_sm) {
        const char* e = getenv("FORGE_GEMV_CTAS_PER_SM");
        ctas_per_sm = (e && atoi(e) > 0 && atoi(e) <= 4) ? atoi(e) : 1;
    }
    // the tensor-parallel epilogue waits for the peers' CTAs of the same
    // tile: one CTA per SM, so every CTA is resident
    int grid = forge_sm_count() * (EPI == FORGE_EPI_RESID_TP ? 1 : ctas_per_sm);
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
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return forge_fail(-1, "gemv launch: %s", cudaGetErrorString(e));
    return 0;
}

template <int WK, int PRO>
int dispatch_epi(const ForgeGemvArgs& a, cudaStream_t s, bool pdl, int smem) {
    switch (a.epi) {
    case FORGE_EPI_STORE: return launch_one<WK, PRO, FORGE_EPI_STORE>(a, s, pdl, smem);
    case FORGE_EPI_RESID: return launch_one<WK, PRO, FORGE_EPI_RESID>(a, s, pdl, smem);
    case FORGE_EPI_QKV: return launch_one<WK, PRO, FORGE_EPI_QKV>(a, s, pdl, smem);
    case FORGE_EPI_SWIGLU: return launch_one<WK, PRO, FORGE_EPI_SWIGLU>(a, s, pdl, smem);
    case FORGE_EPI_LOGITS: return launch_one<WK, PRO, FORGE_EPI_LOGITS>(a, s, pdl, smem);
    case FORGE_EPI_RESID_TP: return launch_one<WK, PRO, FORGE_EPI_RESID_TP>(a, s, pdl, smem);
    default: return forge_fail(-1, "gemv: unknown epilogue %d", a.epi);
    }
}
}  // namespace

// Raises the dynamic shared-memory limit of every GEMV instantiation once per
// device. Must run outside stream capture (forge_b200_create / first per-op call).
int forge_gemv_configure() {
    static bool done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return forge_fail(-1, "gemv: no device");
    if (done[dev]) return 0;
    int rc = configure_epi<FORGE_W_Q4, FORGE_PRO_RMSNORM>() | configure_epi<FORGE_W_Q4, FORGE_PRO_PLAIN>() |
             configure_epi<FORGE_W_BF16, FORGE_PRO_RMSNORM>() | configure_epi<FORGE_W_BF16, FORGE_PRO_PLAIN>();
    if (!rc) done[dev] = true;
    return rc ? -1 : 0;
}

namespace {
// One warp per (128-group, sequence) of x: the group staged in an int4
// GEMV's input block (ForgeGemvArgs::pq_in), the bytes of stage_x_q8. With
// a gain (the next GEMV's RMSNorm): the codes of gain * x, and the group's
// sum of squares of x in ssq [B][K / 128].
__global__ void __launch_bounds__(128) k_stage_groups(const float* x, int x_stride, int K, int B, uint8_t* blk,
                                                      const float* gain, float* ssq) {
    pdl_trigger();
    pdl_wait();
    const int G = K >> 7, lane = threadIdx.x & 31;
    const int item = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (item >= G * B) return;
    const int g = item % G, b = item / G;
    float4 v = __ldcg(reinterpret_cast<const float4*>(x + (size_t)b * x_stride + g * 128) + lane);
    if (gain) {
        float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) ssq[b * G + g] = ss;
        const float4 gv = __ldg(reinterpret_cast<const float4*>(gain + g * 128) + lane);
        v = make_float4(gv.x * v.x, gv.y * v.y, gv.z * v.z, gv.w * v.w);
    }
    pq_group_warp(v, g, b, 2 * B, G, blk);
}
}  // namespace

int forge_stage_groups_launch(const float* x, int x_stride, int K, int B, uint8_t* blk, const float* gain, float* ssq,
                              cudaStream_t stream, bool pdl) {
    if (!x || !blk || K <= 0 || (K % 128) || (x_stride % 4) || B <= 0 || B > 4 || (gain && !ssq))
        return forge_fail(-1, "stage groups: bad shape K=%d B=%d", K, B);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((K / 128 * B + 3) / 4));
    cfg.blockDim = dim3(128);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_stage_groups, x, x_stride, K, B, blk, gain, ssq);
    return e == cudaSuccess ? 0 : forge_fail(-1, "stage groups launch: %s", cudaGetErrorString(e));
}

// Number of launches forge_gemv_launch issues for one call (int4 with a
// batched scratch: two per forge_gemv_b_max_seq() sequences).
int forge_gemv_launch_count(int K, int batch, bool split, bool q4, bool batched) {
    const int row = q4 ? K : ((K + 31) / 32) * 64;
    int max_cols = (kMaxSmem - kFixedSmem - (q4 ? (K / 128) * 48 : 0)) / row;
    if (max_cols > 8) max_cols = 8;
    const int per = max_cols / ((split || q4) ? 2 : 1);
    if (batched && batch > 4 && (q4 || !split)) return 2 * ((batch + forge_gemv_b_max_seq() - 1) / forge_gemv_b_max_seq());
    return per > 0 ? (batch + per - 1) / per : 0;
}

int forge_gemv_launch(const ForgeGemvArgs& a0, cudaStream_t stream, bool pdl) {
    if (!a0.w || !a0.x || a0.N <= 0 || a0.K <= 0 || (a0.N % 16) || (a0.K % 16) || a0.batch <= 0)
        return forge_fail(-1, "gemv: bad shape N=%d K=%d batch=%d", a0.N, a0.K, a0.batch);
    if (a0.wkind == FORGE_W_Q4 && (!a0.s || (a0.K % 128)))
        return forge_fail(-1, "gemv: int4 weights need scales and K %% 128 == 0 (group 128)");
    if (a0.pro == FORGE_PRO_RMSNORM && !a0.gain) return forge_fail(-1, "gemv: RMSNorm prologue needs a gain");
    if ((a0.x_stride % 4) || (a0.K % 16)) return forge_fail(-1, "gemv: K %% 16 == 0 and 16-byte aligned x rows required");
    if (a0.epi == FORGE_EPI_SWIGLU && a0.N != 2 * a0.F) return forge_fail(-1, "gemv: SwiGLU needs N == 2F");
    if (a0.epi == FORGE_EPI_RESID_TP && (!a0.tpf || a0.batch > 4))
        return forge_fail(-1, "gemv: the tensor-parallel residual epilogue takes 1..4 sequences and exchange buffers");
    if (a0.epi == FORGE_EPI_QKV && (a0.hd % 16 || a0.N != (a0.H + 2 * a0.Hkv) * a0.hd))
        return forge_fail(-1, "gemv: QKV epilogue shape mismatch");
    const bool q4 = a0.wkind == FORGE_W_Q4;
    const int cols_per_seq = (q4 || a0.split) ? 2 : 1;
    if (a0.K / 128 > kMaxG) return forge_fail(-1, "gemv: K=%d above the supported maximum", a0.K);
    const int sx_bytes = q4 ? (a0.K / 128) * 12 * 4 : 0;
    // bf16: K padded to whole k-tile pairs, 2 bytes; int4: int8 activations
    const int xs_row = q4 ? a0.K : ((a0.K + 31) / 32) * 32 * 2;
    int max_cols = (kMaxSmem - kFixedSmem - sx_bytes) / xs_row;
    if (max_cols > 8) max_cols = 8;
    const int per_launch = max_cols / cols_per_seq;
    if (per_launch < 1) return forge_fail(-1, "gemv: K=%d too large for the staged activation", a0.K);
    if (a0.pq_in && (!q4 || a0.batch > 4 || a0.batch > per_launch || (a0.pro == FORGE_PRO_RMSNORM && !a0.pq_ssq)))
        return forge_fail(-1, "gemv: a staged input block takes int4 weights and 1..4 sequences in one launch");
    const bool batched_ok = q4 ? (a0.epi != FORGE_EPI_LOGITS) : !a0.split;
    // above 4 sequences (int4: more than one launch's worth; bf16: bf16
    // activations, where one CTA per sequence stages in parallel)
    if (a0.batch > 4 && a0.bscratch && a0.pro != FORGE_PRO_EMBED_RMSNORM && batched_ok) {
        // larger batches: one weight stream per forge_gemv_b_max_seq() sequences
        const int mx = forge_gemv_b_max_seq();
        for (int b0 = 0; b0 < a0.batch; b0 += mx) {
            ForgeGemvArgs a = a0;
            a.batch = a0.batch - b0 < mx ? a0.batch - b0 : mx;
            a.b0 = a0.b0 + b0;
            a.x = a0.x + (size_t)b0 * a0.x_stride;
            if (a.y) a.y = a0.y + (size_t)b0 * a0.y_stride;
            if (a.q_out) a.q_out = a0.q_out + (size_t)b0 * a0.H * a0.hd;
            if (a.s_out) a.s_out = a0.s_out + (size_t)b0 * a0.F;
            if (int rc = forge_gemv_b_launch(a, a0.bscratch, stream, pdl && b0 == 0)) return rc;
        }
        return 0;
    }
    for (int b0 = 0; b0 < a0.batch; b0 += per_launch) {
        ForgeGemvArgs a = a0;
        a.batch = a0.batch - b0 < per_launch ? a0.batch - b0 : per_launch;
        a.b0 = a0.b0 + b0;
        a.x = a0.x + (size_t)b0 * a0.x_stride;
        if (a.y) a.y = a0.y + (size_t)b0 * a0.y_stride;
        if (a.q_out) a.q_out = a0.q_out + (size_t)b0 * a0.H * a0.hd;
        if (a.s_out) a.s_out = a0.s_out + (size_t)b0 * a0.F;
        const int smem = kFixedSmem + sx_bytes + a.batch * cols_per_seq * xs_row;
        int rc;
        const bool p = pdl && b0 == 0;
        if (a.wkind == FORGE_W_Q4)
            rc = a.pro == FORGE_PRO_RMSNORM ? dispatch_epi<FORGE_W_Q4, FORGE_PRO_RMSNORM>(a, stream, p, smem)
                                            : dispatch_epi<FORGE_W_Q4, FORGE_PRO_PLAIN>(a, stream, p, smem);
        else
            rc = a.pro == FORGE_PRO_RMSNORM ? dispatch_epi<FORGE_W_BF16, FORGE_PRO_RMSNORM>(a, stream, p, smem)
                                            : dispatch_epi<FORGE_W_BF16, FORGE_PRO_PLAIN>(a, stream, p, smem);
        if (rc) return rc;
    }
    return 0;
}
