// decode_step.cu — one greedy decode step for the whole model as a single
// persistent cooperative kernel (one CTA per SM).
//
// The step (embed -> L x [QKV+RoPE+KV append, flash-decode, O+residual,
// gate/up+SwiGLU, down+residual] -> LM head+argmax -> next token; the same
// math as model.cu's multi-kernel path, decoder_lib.hexa:93-208 with a KV
// cache) is a list of phases. Inside the kernel:
//   * one producer thread walks every phase's work list for its CTA and
//     streams the weight pieces (and the cached K/V rows of attention,
//     except the row appended this step) into a shared-memory ring with
//     cp.async.bulk. Weights and old cache rows never change during a step,
//     so the producer runs ahead across phase boundaries: HBM keeps
//     streaming while the consumers wait at a grid barrier.
//   * sixteen consumer warps run each phase (activation staging, mma.sync
//     fragment GEMV or split-K attention, fused epilogue) and meet the other
//     CTAs at a grid barrier only where a phase reads the previous phase's
//     output.
// Activations crossing CTAs are read with ld.global.cg (no stale L1 lines).
// Every wait is bounded: a timeout raises the device error word and turns
// all later waits of the CTA into no-ops, so a fault ends the step quickly
// instead of hanging; the producer still waits (bounded) for its own copies
// before exiting.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include "common.cuh"
#include "layout.cuh"
#include "forge_internal.h"
#include "gemv_core.cuh"

namespace {
constexpr int kCW = 8;                // consumer warps
constexpr int kNT = kCW * 32;         // consumer threads
#ifndef FORGE_STEP_PRODUCER_WARP_DEF
#define FORGE_STEP_PRODUCER_WARP_DEF 1
#endif
constexpr int kThreadsMK = kNT + (FORGE_STEP_PRODUCER_WARP_DEF ? 32 : 0);
constexpr int kPiece = 16384;         // weight bytes per ring stage
constexpr int kPieceS = 512;          // int4 scale bytes per ring stage
constexpr int kStage = kPiece + kPieceS;
constexpr int kRedSlot = kCW * 16 * 8;
constexpr int kMaxGroups = 128;       // K <= 16384 for int4 phases
constexpr int kSxFloats = kMaxGroups * 12;  // [G][4] scales + [G][8] column sums
constexpr int kProdBytes = 128;
constexpr int kPhaseBytes = (int)((sizeof(ForgePhase) + 15) / 16 * 16);

template <int HD> constexpr int attn_tile() { return kPiece / (4 * HD); }  // keys per K+V stage
template <int HD, int G> constexpr int red_floats() {
    return (4096 > kCW * G * (HD + 2)) ? 4096 : kCW * G * (HD + 2);
}
template <int HD, int G> constexpr int attn_floats() {
    return G * HD + 2 * G * attn_tile<HD>() + 4 * G + 8;
}

struct Prod;
struct Smem {
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    float* red;
    float* sx;
    float* qs;
    float* sc;
    float* st;
    int* flags;  // [0] abort, [1] is_last
    uint16_t* xf;
    struct Prod* prod;
    ForgePhase* ph;  // shared copy of the current phase's descriptor
    unsigned long long* tr;  // this CTA's trace row for the current phase (or null)
};

// Producer cursor (touched by thread 0 only): next item to issue.
struct Prod {
    int p, u, i, done;
    uint32_t issued;
    // production parameters of phase p (cached so the producer never reads
    // the descriptor array in global memory while streaming)
    const uint8_t* w;
    const uint8_t* s;
    int KT, item_kt, tb, nitems, units, G4, q4;
};

__device__ __forceinline__ bool aborted(const Smem& m) { return *(volatile int*)&m.flags[0] != 0; }

#define FORGE_STEP_PRODUCER_WARP FORGE_STEP_PRODUCER_WARP_DEF

__device__ bool mk_wait_plain(const Smem& m, uint64_t* bar, uint32_t parity, uint32_t* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u) {
            if (*(volatile int*)&m.flags[0]) return false;
            if (globaltimer_ns() - t0 > FORGE_WAIT_NS || i > FORGE_SPIN_LIMIT) {
                atomicOr(err, FORGE_DEVERR_MBAR_TIMEOUT);
                *(volatile int*)&m.flags[0] = 1;
                return false;
            }
        }
    }
}

// Moves the cursor to the next GEMV piece this CTA owns (or marks done).
__device__ void cursor_normalize(Prod& c, const ForgeStepArgs& sa) {
    while (c.p < sa.nphases) {
        const ForgePhase& ph = sa.phases[c.p];
        if (ph.type == FORGE_PH_GEMV && c.u < (ph.g.N >> 4)) {
            c.w = static_cast<const uint8_t*>(ph.g.w);
            c.s = static_cast<const uint8_t*>(ph.g.s);
            c.q4 = ph.g.wkind == FORGE_W_Q4;
            c.KT = ph.g.K >> 4;
            c.item_kt = c.q4 ? 128 : 32;
            c.tb = c.q4 ? 128 : 512;
            c.nitems = (c.KT + c.item_kt - 1) / c.item_kt;
            c.units = ph.g.N >> 4;
            c.G4 = (c.KT / 8 + 3) / 4;
            return;
        }
        ++c.p;
        c.u = blockIdx.x;
        c.i = 0;
    }
    c.done = 1;
}

// Issues the cursor's next piece into stage (issued % S) and advances.
__device__ __forceinline__ void issue_one(const Smem& m, const ForgeStepArgs& sa, int S) {
    Prod& c = *m.prod;
    const int s = c.issued % S;
    const int kt0 = c.i * c.item_kt, nkt = min(c.item_kt, c.KT - kt0);
    const uint32_t wb = (uint32_t)nkt * c.tb;
    const uint32_t sb = c.q4 ? (uint32_t)(((nkt / 8) + 3) / 4) * 128u : 0u;
    uint8_t* dst = m.ring + (size_t)s * kStage;
    mbar_arrive_expect_tx(&m.full[s], wb + sb);
    bulk_g2s(dst, c.w + ((int64_t)c.u * c.KT + kt0) * c.tb, wb, &m.full[s]);
    if (c.q4) bulk_g2s(dst + kPiece, c.s + ((int64_t)c.u * c.G4 + kt0 / 32) * 128, sb, &m.full[s]);
    ++c.issued;
    if (++c.i == c.nitems) {
        c.i = 0;
        c.u += gridDim.x;
        cursor_normalize(c, sa);
    }
}

#if FORGE_STEP_PRODUCER_WARP
// Dedicated producer (one lane of the last warp): blocks on each stage's
// release, then refills it; runs ahead across phases up to the ring depth.
__device__ void produce_all(const Smem& m, const ForgeStepArgs& sa, int S) {
    Prod& c = *m.prod;
    while (!c.done && !aborted(m)) {
        const int s = c.issued % S;
        if (!mk_wait_plain(m, &m.empty[s], ((c.issued / S) & 1u) ^ 1u, sa.err)) break;
        issue_one(m, sa, S);
    }
}
__device__ __forceinline__ void pump(const Smem&, const ForgeStepArgs&, int, uint32_t) {}
#else
// Issues ring pieces while stages are free and the ring is less than S
// pieces ahead of `consumed` (thread 0 only; never blocks).
__device__ void pump(const Smem& m, const ForgeStepArgs& sa, int S, uint32_t consumed) {
    Prod& c = *m.prod;
    while (!c.done && c.issued < consumed + (uint32_t)S && !aborted(m)) {
        const int s = c.issued % S;
        if (!mbar_test_wait(&m.empty[s], ((c.issued / S) & 1u) ^ 1u)) break;
        issue_one(m, sa, S);
    }
}
#endif

// Bounded, abort-aware mbarrier wait. Thread 0 keeps pumping the ring
// while it waits (it is the only producer).
__device__ bool mk_wait(const Smem& m, uint64_t* bar, uint32_t parity, uint32_t* err,
                        const ForgeStepArgs& sa, int S, uint32_t consumed) {
    const bool producer = !FORGE_STEP_PRODUCER_WARP && threadIdx.x == 0;
    if (producer) pump(m, sa, S, consumed);
    if (producer ? mbar_test_wait(bar, parity) : mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0;; ++i) {
        if (producer) pump(m, sa, S, consumed);
        // the producer thread polls without suspending so it keeps refilling
        if (producer ? mbar_test_wait(bar, parity) : mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u) {
            if (aborted(m)) return false;
            if (globaltimer_ns() - t0 > FORGE_WAIT_NS || i > FORGE_SPIN_LIMIT) {
                atomicOr(err, FORGE_DEVERR_MBAR_TIMEOUT);
                *(volatile int*)&m.flags[0] = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier on a monotonic counter: every CTA adds 1 per phase.
__device__ void grid_wait(const Smem& m, const ForgeStepArgs& sa, unsigned long long target, int S,
                          uint32_t consumed) {
    if (threadIdx.x == 0 && !aborted(m)) {
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t i = 0;; ++i) {
            pump(m, sa, S, consumed);
            if (ld_acquire_u64(sa.bar) >= target) break;
            if ((i & 63u) == 63u) {
                if (*(volatile uint32_t*)sa.err & (FORGE_DEVERR_MBAR_TIMEOUT | FORGE_DEVERR_COUNTER_TIMEOUT)) {
                    *(volatile int*)&m.flags[0] = 1;
                    break;
                }
                if (globaltimer_ns() - t0 > FORGE_WAIT_NS || i > FORGE_SPIN_LIMIT) {
                    atomicOr(sa.err, FORGE_DEVERR_COUNTER_TIMEOUT);
                    *(volatile int*)&m.flags[0] = 1;
                    break;
                }
            }
        }
        __threadfence();
    }
    named_bar_sync(1, kNT);
}

__device__ void grid_arrive(const ForgeStepArgs& sa) {
    named_bar_sync(1, kNT);
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(sa.bar, 1ull);
    }
}

// The staging routines are inlined into the standalone GEMV; in this kernel
// (one CTA per SM, many phase types) they stay out of line so their
// registers do not add to every phase's.
template <int PRO, int NT>
__device__ __noinline__ void stage_q8_call(const ForgeGemvArgs& a, uint8_t* xq, float* sxf, int* ssum, float* red) {
    stage_x_q8<PRO, NT>(a, xq, sxf, ssum, red);
}
template <int PRO, int NT>
__device__ __noinline__ void stage_bf16_call(const ForgeGemvArgs& a, uint16_t* xf, float* red) {
    stage_x<PRO, NT>(a, xf, red);
}

// ------------------------------------------------------------------ GEMV
template <int WK, int PRO, int EPI>
__device__ void gemv_phase(const Smem& m, const ForgeStepArgs& sa, const ForgeGemvArgs& a, uint32_t& it, int S) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KT = a.K >> 4;
    constexpr int kItemKT = (WK == FORGE_W_Q4) ? 128 : 32;
    const int nitems = (KT + kItemKT - 1) / kItemKT;
    const int units = a.N >> 4;

    float* sxf = m.sx;
    int* ssum = reinterpret_cast<int*>(m.sx + kMaxGroups * 4);
    uint8_t* xq = reinterpret_cast<uint8_t*>(m.xf);
    if (WK == FORGE_W_Q4) {
        stage_q8_call<PRO, kNT>(a, xq, sxf, ssum, m.red);
    } else {
        stage_bf16_call<PRO, kNT>(a, m.xf, m.red);
        zero_x_pad<kNT>(a, m.xf);
    }
    if (PRO == FORGE_PRO_EMBED_RMSNORM && blockIdx.x == 0) {
        // the residual stream starts as the embedding row (written once)
        for (int b = 0; b < a.batch; ++b)
            for (int k = threadIdx.x * 2; k < a.K; k += kNT * 2) {
                const uint32_t v = *reinterpret_cast<const uint32_t*>(a.emb + (size_t)a.emb_tok[a.b0 + b] * a.K + k);
                a.y[(size_t)b * a.y_stride + k] = bf16_lo_f32(v);
                a.y[(size_t)b * a.y_stride + k + 1] = bf16_hi_f32(v);
            }
    }
    named_bar_sync(1, kNT);
    if (m.tr && threadIdx.x == 0) m.tr[2] = globaltimer_ns();

    const int g = lane >> 2, t = lane & 3;
    const int ncols = (WK == FORGE_W_Q4 || a.split) ? 2 * a.batch : a.batch;
    const int col = g < ncols ? g : ncols - 1;
    const int rc = (WK == FORGE_W_Q4) ? a.batch : ncols;  // reduction columns per row
    unsigned long long best = 0ull;
    const int slot_floats = kCW * 16 * rc;
    int R = 4096 / (2 * slot_floats);
    R = R < 1 ? 1 : (R > 8 ? 8 : R);
    int ui = 0;

    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        float tot[4] = {0.f, 0.f, 0.f, 0.f}, tot2[4] = {0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < nitems; ++i) {
            const int s = it % S;
            mk_wait(m, &m.full[s], (it / S) & 1u, a.err, sa, S, it);
            const int kt0 = i * kItemKT, nkt = min(kItemKT, KT - kt0);
            const uint8_t* st = m.ring + (size_t)s * kStage;
            if (WK == FORGE_W_Q4) {
                // warp w: groups 2w and 2w+1 of the piece (int8 tensor-core path)
                const int ng = nkt / 8;
                const int gA = 2 * warp;
                const uint16_t* sst = reinterpret_cast<const uint16_t*>(st + kPiece);
                if (gA + 1 < ng) {
                    // both groups in one block so their loads and MMAs interleave
                    const uint4 wA0 = *reinterpret_cast<const uint4*>(st + (4 * warp) * 512 + lane * 16);
                    const uint4 wA1 = *reinterpret_cast<const uint4*>(st + (4 * warp + 1) * 512 + lane * 16);
                    const uint4 wB0 = *reinterpret_cast<const uint4*>(st + (4 * warp + 2) * 512 + lane * 16);
                    const uint4 wB1 = *reinterpret_cast<const uint4*>(st + (4 * warp + 3) * 512 + lane * 16);
                    const uint32_t scA = *reinterpret_cast<const uint32_t*>(sst + (gA >> 2) * 64 + g * 8 + (gA & 3) * 2);
                    const int gB = gA + 1;
                    const uint32_t scB = *reinterpret_cast<const uint32_t*>(sst + (gB >> 2) * 64 + g * 8 + (gB & 3) * 2);
                    float yA0, yA1, yB0, yB1;
                    q4_group(wA0, wA1, xq, kt0 / 8 + gA, ncols, col, t, scA, sxf, ssum, a.batch, yA0, yA1);
                    q4_group(wB0, wB1, xq, kt0 / 8 + gB, ncols, col, t, scB, sxf, ssum, a.batch, yB0, yB1);
                    tot[0] += yA0;
                    tot[1] += yA1;
                    tot2[0] += yB0;
                    tot2[1] += yB1;
                } else if (gA < ng) {
                    const uint4 w0 = *reinterpret_cast<const uint4*>(st + (4 * warp) * 512 + lane * 16);
                    const uint4 w1 = *reinterpret_cast<const uint4*>(st + (4 * warp + 1) * 512 + lane * 16);
                    const uint32_t sc = *reinterpret_cast<const uint32_t*>(sst + (gA >> 2) * 64 + g * 8 + (gA & 3) * 2);
                    float y0, y1;
                    q4_group(w0, w1, xq, kt0 / 8 + gA, ncols, col, t, sc, sxf, ssum, a.batch, y0, y1);
                    tot[0] += y0;
                    tot[1] += y1;
                }
            } else {
                const int ktw = 4 * warp;  // warp w: k-tiles 4w .. 4w+3 (two pairs)
#pragma unroll
                for (int jp = 0; jp < 2; ++jp) {
                    const int kt = ktw + 2 * jp;
                    if (kt < nkt) {
                        const uint4 w0 = *reinterpret_cast<const uint4*>(st + kt * 512 + lane * 16);
                        const uint4 w1 = (kt + 1 < nkt) ? *reinterpret_cast<const uint4*>(st + (kt + 1) * 512 + lane * 16)
                                                        : make_uint4(0, 0, 0, 0);
                        const int kp = (kt0 + kt) >> 1;
                        const uint4 bb = *(reinterpret_cast<const uint4*>(m.xf) + (size_t)(kp * ncols + col) * 4 + t);
                        const uint32_t f0[4] = {w0.x, w0.y, w0.z, w0.w};
                        const uint32_t f1[4] = {w1.x, w1.y, w1.z, w1.w};
                        mma_bf16_16816(tot, f0, bb.x, bb.y, tot);
                        mma_bf16_16816(tot2, f1, bb.z, bb.w, tot2);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&m.empty[s]);
            ++it;
        }
        // defer the cross-warp reduction: partials of up to R units collect in
        // one of two slot groups; one barrier per R units, then the epilogue
        // threads finish those units while the other warps continue
        const int grp = (ui / R) & 1, si = ui % R;
        float* rw = m.red + ((size_t)(grp * R + si) * kCW + warp) * 16 * rc;
        if (WK == FORGE_W_Q4) {
            if (t < a.batch) {
                rw[g * rc + t] = tot[0] + tot2[0];
                rw[(g + 8) * rc + t] = tot[1] + tot2[1];
            }
        } else {
            if (2 * t < ncols) {
                rw[g * rc + 2 * t] = tot[0] + tot2[0];
                rw[(g + 8) * rc + 2 * t] = tot[2] + tot2[2];
            }
            if (2 * t + 1 < ncols) {
                rw[g * rc + 2 * t + 1] = tot[1] + tot2[1];
                rw[(g + 8) * rc + 2 * t + 1] = tot[3] + tot2[3];
            }
        }
        if (si == R - 1 || u + (int)gridDim.x >= units) {
            named_bar_sync(1, kNT);
            // epilogue threads sit in the last warps so warp 0 (the producer)
            // keeps pumping the ring meanwhile
            const int et = kNT - 1 - (int)threadIdx.x;
            if (et < 8 * a.batch) {
                const int p = et & 7, b = et >> 3;
                const int c = (WK == FORGE_W_Q4) ? b : (a.split ? 2 * b : b);
                const bool two = WK != FORGE_W_Q4 && a.split;
                for (int k = 0; k <= si; ++k) {
                    const int uk = blockIdx.x + (ui - si + k) * (int)gridDim.x;
                    const float* rs = m.red + (size_t)(grp * R + k) * kCW * 16 * rc;
                    float ylo = 0.f, yhi = 0.f;
#pragma unroll
                    for (int w = 0; w < kCW; ++w) {
                        ylo += rs[(w * 16 + p) * rc + c];
                        yhi += rs[(w * 16 + p + 8) * rc + c];
                        if (two) {
                            ylo += rs[(w * 16 + p) * rc + c + 1];
                            yhi += rs[(w * 16 + p + 8) * rc + c + 1];
                        }
                    }
                    epilogue<EPI>(a, uk, p, b, ylo, yhi, best);
                }
            }
        }
        ++ui;
    }
    if (EPI == FORGE_EPI_LOGITS && warp >= kCW - 2) {
        // thread (p, b) = (et & 7, et >> 3): reduce over the 8 row pairs
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
            best = v > best ? v : best;
        }
        const int et = kNT - 1 - (int)threadIdx.x;
        if ((et & 7) == 0 && (et >> 3) < a.batch && best != 0ull)
            atomicMax(a.argmax_key + a.b0 + (et >> 3), best);
    }
}

__device__ void gemv_dispatch(const Smem& m, const ForgeStepArgs& sa, const ForgeGemvArgs& a, uint32_t& it, int S) {
#define FORGE_GEMV_CASE(WK, PRO, EPI) \
    if (a.wkind == WK && a.pro == PRO && a.epi == EPI) { gemv_phase<WK, PRO, EPI>(m, sa, a, it, S); return; }
    FORGE_GEMV_CASE(FORGE_W_Q4, FORGE_PRO_RMSNORM, FORGE_EPI_QKV)
    FORGE_GEMV_CASE(FORGE_W_Q4, FORGE_PRO_EMBED_RMSNORM, FORGE_EPI_QKV)
    FORGE_GEMV_CASE(FORGE_W_Q4, FORGE_PRO_PLAIN, FORGE_EPI_RESID)
    FORGE_GEMV_CASE(FORGE_W_Q4, FORGE_PRO_RMSNORM, FORGE_EPI_SWIGLU)
    FORGE_GEMV_CASE(FORGE_W_BF16, FORGE_PRO_RMSNORM, FORGE_EPI_QKV)
    FORGE_GEMV_CASE(FORGE_W_BF16, FORGE_PRO_EMBED_RMSNORM, FORGE_EPI_QKV)
    FORGE_GEMV_CASE(FORGE_W_BF16, FORGE_PRO_PLAIN, FORGE_EPI_RESID)
    FORGE_GEMV_CASE(FORGE_W_BF16, FORGE_PRO_RMSNORM, FORGE_EPI_SWIGLU)
    FORGE_GEMV_CASE(FORGE_W_BF16, FORGE_PRO_RMSNORM, FORGE_EPI_LOGITS)
#undef FORGE_GEMV_CASE
    atomicOr(a.err, FORGE_DEVERR_BAD_INDEX);
}

// ------------------------------------------------------------- attention
// CTA work item = (sequence b, KV head, split of the context). Inside the
// item every warp owns a contiguous run of keys and keeps its own online
// softmax (lane = key for the scores, lanes = dims for P·V), so the only
// CTA-wide synchronisation is the final 16-way merge. K/V rows come straight
// from HBM (streaming loads; the row appended this step was written by the
// QKV phase and is visible after the grid barrier), leaving the producer's
// ring free to prefetch the next phases' weights meanwhile.
struct AttnItem {
    int b, kvh, sp, P, Lc, j0, j1, n;
    bool bad;
};
__device__ __forceinline__ AttnItem attn_item(const ForgeStepArgs& sa, int item) {
    AttnItem r;
    r.sp = item % sa.nsplit;
    r.kvh = (item / sa.nsplit) % sa.Hkv;
    r.b = item / (sa.nsplit * sa.Hkv);
    r.P = __ldcg(sa.pos + r.b);
    r.bad = r.P < 0 || r.P >= sa.lmax;
    r.Lc = r.bad ? 0 : r.P + 1;
    const int chunk = (r.Lc + sa.nsplit - 1) / sa.nsplit;
    r.j0 = r.sp * chunk;
    r.j1 = min(r.Lc, r.j0 + chunk);
    r.n = max(0, r.j1 - r.j0);
    return r;
}

template <int HD, int G>
__device__ void attn_phase(const Smem& m, const ForgeStepArgs& sa, const ForgePhase& ph, int S, uint32_t consumed) {
    constexpr int E = HD / 32;          // value dims per lane
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const float scale = 1.0f / sqrtf((float)HD);
    const int nitem = sa.B * sa.Hkv * sa.nsplit;
    const int stride = HD + 2;
    float* wm = m.red;                          // [kCW][G] warp running max
    float* wl = m.red + kCW * G;                // [kCW][G] warp running sum
    float* wo = m.red + 2 * kCW * G;            // [kCW][G][HD] warp partial O

    for (int item = blockIdx.x; item < nitem; item += gridDim.x) {
        const AttnItem r = attn_item(sa, item);
        if (r.bad) {
            if (tid == 0) atomicOr(sa.err, FORGE_DEVERR_BAD_INDEX);
            continue;
        }
        const size_t slab = ((size_t)r.b * sa.Hkv + r.kvh) * sa.lmax * HD;
        const uint16_t* Kg = ph.g.kc + slab;
        const uint16_t* Vg = ph.g.vc + slab;
        for (int i = tid; i < G * HD / 4; i += kNT)
            reinterpret_cast<float4*>(m.qs)[i] =
                __ldcg(reinterpret_cast<const float4*>(sa.q + (size_t)r.b * sa.H * HD + (size_t)(r.kvh * G) * HD) + i);
        named_bar_sync(1, kNT);
        // this warp's keys: [k0, k1)
        const int per = (r.n + kCW - 1) / kCW;
        const int k0 = r.j0 + warp * per, k1 = min(r.j1, k0 + per);
        float mx[G], ls[G], acc[G][E];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            mx[g] = -INFINITY; ls[g] = 0.f;
#pragma unroll
            for (int e = 0; e < E; ++e) acc[g][e] = 0.f;
        }
        // blocks of 8 keys: 4 lanes per key for the scores (lane part qp reads
        // dims qp*8 + 32m), lane-owned dims for P·V; the K and V loads of a
        // block are issued together, one memory round trip per block
        const int kj = lane >> 2, qp = lane & 3;
        constexpr int M = HD / 32;
        for (int base = k0; base < k1; base += 8) {
#if !FORGE_STEP_PRODUCER_WARP
            if (tid == 0) pump(m, sa, S, consumed);  // keep prefetching the next weights
#endif
            const int j = base + kj;
            const bool valid = j < k1;
            const int jc = valid ? j : k0;
            uint4 kw[M];
#pragma unroll
            for (int mm = 0; mm < M; ++mm)
                kw[mm] = __ldcs(reinterpret_cast<const uint4*>(Kg + (size_t)jc * HD + mm * 32 + qp * 8));
            uint32_t vv[8][E / 2];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int jv = min(base + u, k1 - 1);
                const uint16_t* vr = Vg + (size_t)jv * HD + lane * E;
                if (E == 4) {
                    const uint2 t2 = __ldcs(reinterpret_cast<const uint2*>(vr));
                    vv[u][0] = t2.x; vv[u][E / 2 - 1] = t2.y;
                } else {
                    vv[u][0] = __ldcs(reinterpret_cast<const unsigned int*>(vr));
                }
            }
            float pk[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float d = 0.f;
#pragma unroll
                for (int mm = 0; mm < M; ++mm) {
                    const float4 q0 = *reinterpret_cast<const float4*>(m.qs + g * HD + mm * 32 + qp * 8);
                    const float4 q1 = *reinterpret_cast<const float4*>(m.qs + g * HD + mm * 32 + qp * 8 + 4);
                    d = fmaf(q0.x, bf16_lo_f32(kw[mm].x), d); d = fmaf(q0.y, bf16_hi_f32(kw[mm].x), d);
                    d = fmaf(q0.z, bf16_lo_f32(kw[mm].y), d); d = fmaf(q0.w, bf16_hi_f32(kw[mm].y), d);
                    d = fmaf(q1.x, bf16_lo_f32(kw[mm].z), d); d = fmaf(q1.y, bf16_hi_f32(kw[mm].z), d);
                    d = fmaf(q1.z, bf16_lo_f32(kw[mm].w), d); d = fmaf(q1.w, bf16_hi_f32(kw[mm].w), d);
                }
                d += __shfl_xor_sync(0xffffffffu, d, 1);
                d += __shfl_xor_sync(0xffffffffu, d, 2);
                const float sv = valid ? d * scale : -INFINITY;
                float t = sv;
                t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, 4));
                t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, 8));
                t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, 16));
                const float mn = fmaxf(mx[g], t);
                const float al = (mx[g] == -INFINITY) ? 0.f : expf(mx[g] - mn);
                const float p = valid ? expf(sv - mn) : 0.f;
                float ps = qp == 0 ? p : 0.f;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
                ls[g] = ls[g] * al + ps;
                mx[g] = mn;
#pragma unroll
                for (int e = 0; e < E; ++e) acc[g][e] *= al;
                pk[g] = p;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float p = __shfl_sync(0xffffffffu, pk[g], 4 * u);
#pragma unroll
                    for (int e2 = 0; e2 < E / 2; ++e2) {
                        acc[g][2 * e2] = fmaf(p, bf16_lo_f32(vv[u][e2]), acc[g][2 * e2]);
                        acc[g][2 * e2 + 1] = fmaf(p, bf16_hi_f32(vv[u][e2]), acc[g][2 * e2 + 1]);
                    }
                }
            }
        }
        // ---- merge the 16 warps (log-sum-exp) into this item's partial
        if (lane == 0)
#pragma unroll
            for (int g = 0; g < G; ++g) { wm[warp * G + g] = mx[g]; wl[warp * G + g] = ls[g]; }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < E; ++e) wo[(warp * G + g) * HD + lane * E + e] = acc[g][e];
        named_bar_sync(1, kNT);
        for (int idx = tid; idx < G * HD; idx += kNT) {
            const int g = idx / HD, e = idx % HD;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kCW; ++w) M = fmaxf(M, wm[w * G + g]);
            float L = 0.f, O = 0.f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) {
                const float mw = wm[w * G + g];
                const float f = (mw == -INFINITY) ? 0.f : expf(mw - M);
                L = fmaf(f, wl[w * G + g], L);
                O = fmaf(f, wo[(w * G + g) * HD + e], O);
            }
            const int h = r.kvh * G + g;
            float* pp = sa.partial + (((size_t)r.b * sa.H + h) * sa.nsplit + r.sp) * stride;
            pp[e] = O;
            if (e == 0) { pp[HD] = M; pp[HD + 1] = L; }
        }
        __threadfence();
        named_bar_sync(1, kNT);
        if (tid == 0) {
            const uint32_t old = atomicAdd(sa.counters + (size_t)r.b * sa.Hkv + r.kvh, 1u);
            m.flags[1] = (old == (uint32_t)(sa.nsplit - 1));
        }
        named_bar_sync(1, kNT);
        if (m.flags[1]) {
            __threadfence();
            for (int idx = tid; idx < G * HD; idx += kNT) {
                const int g = idx / HD, e = idx % HD;
                const int h = r.kvh * G + g;
                const float* pb = sa.partial + ((size_t)r.b * sa.H + h) * sa.nsplit * stride;
                float mg = -INFINITY;
                for (int s2 = 0; s2 < sa.nsplit; ++s2) mg = fmaxf(mg, __ldcg(pb + s2 * stride + HD));
                float lsum = 0.f, o = 0.f;
                for (int s2 = 0; s2 < sa.nsplit; ++s2) {
                    const float ms = __ldcg(pb + s2 * stride + HD);
                    const float w = ms == -INFINITY ? 0.f : expf(ms - mg);
                    lsum = fmaf(w, __ldcg(pb + s2 * stride + HD + 1), lsum);
                    o = fmaf(w, __ldcg(pb + s2 * stride + e), o);
                }
                sa.ctx[(size_t)r.b * sa.H * HD + (size_t)h * HD + e] = o / lsum;
            }
            if (tid == 0) sa.counters[(size_t)r.b * sa.Hkv + r.kvh] = 0u;
        }
        named_bar_sync(1, kNT);
    }
}

template <int HD, int G>
__global__ void __launch_bounds__(kThreadsMK, 1) k_decode_step(const ForgeStepArgs sa) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int S = sa.stages;
    Smem m;
    m.ring = smem_raw;
    m.full = reinterpret_cast<uint64_t*>(smem_raw + (size_t)S * kStage);
    m.empty = m.full + S;
    m.red = reinterpret_cast<float*>(m.empty + S);
    m.sx = m.red + red_floats<HD, G>();
    m.qs = m.sx + kSxFloats;
    m.sc = m.qs + G * HD;
    m.st = m.sc + 2 * G * attn_tile<HD>();
    m.flags = reinterpret_cast<int*>(m.st + 4 * G);
    m.prod = reinterpret_cast<Prod*>(m.qs + attn_floats<HD, G>());
    m.ph = reinterpret_cast<ForgePhase*>(reinterpret_cast<uint8_t*>(m.prod) + kProdBytes);
    m.xf = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(m.ph) + kPhaseBytes);

    const unsigned long long epoch = *reinterpret_cast<volatile const uint32_t*>(sa.epoch);
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&m.full[s], 1);
            mbar_init(&m.empty[s], kCW);
        }
        m.flags[0] = 0;
        m.flags[1] = 0;
        m.prod->p = 0; m.prod->u = blockIdx.x; m.prod->i = 0; m.prod->done = 0; m.prod->issued = 0;
        cursor_normalize(*m.prod, sa);
        fence_mbar_init();
    }
    __syncthreads();

#if FORGE_STEP_PRODUCER_WARP
    if ((threadIdx.x >> 5) == kCW) {
        if ((threadIdx.x & 31) == 0) {
            produce_all(m, sa, S);
            const uint32_t issued = m.prod->issued;
            for (uint32_t j = 0; j < (uint32_t)S && j < issued; ++j) {
                const uint32_t idx = issued - 1 - j;
                mbar_wait(&m.full[idx % S], (idx / S) & 1u, sa.err);
            }
        }
        return;
    }
#endif
    const unsigned long long nbar = (unsigned long long)(sa.nphases - 1);
    uint32_t it = 0;
    unsigned long long* tr = sa.trace ? sa.trace + (size_t)blockIdx.x * sa.nphases * 4 : nullptr;
    for (int p = 0; p < sa.nphases; ++p) {
        if (tr && threadIdx.x == 0) tr[p * 4 + 0] = globaltimer_ns();
        // the descriptor copy rides on the barrier below (or the one after
        // the previous phase's copy for p == 0)
        for (int i = threadIdx.x; i < (int)(sizeof(ForgePhase) / 4); i += kNT)
            reinterpret_cast<uint32_t*>(m.ph)[i] = reinterpret_cast<const uint32_t*>(sa.phases + p)[i];
        if (p > 0) grid_wait(m, sa, (epoch * nbar + (unsigned long long)p) * gridDim.x, S, it);
        else named_bar_sync(1, kNT);
        const ForgePhase& ph = *m.ph;
        m.tr = tr ? tr + p * 4 : nullptr;
        if (tr && threadIdx.x == 0) tr[p * 4 + 1] = globaltimer_ns();
        if (ph.type == FORGE_PH_GEMV) {
            gemv_dispatch(m, sa, ph.g, it, S);
        } else if (ph.type == FORGE_PH_ATTN) {
            attn_phase<HD, G>(m, sa, ph, S, it);
        } else if (ph.type == FORGE_PH_FIN) {
            if (blockIdx.x == 0) {
                const int b = threadIdx.x;
                const int s = *sa.step;
                if (b < sa.B) {
                    const unsigned long long k = __ldcg(sa.amax + b);
                    const int32_t tk = k ? (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0;
                    sa.tok[b] = tk;
                    if (s < sa.hist_cap) sa.hist[(size_t)s * sa.B + b] = tk;
                    sa.amax[b] = 0ull;
                    sa.pos[b] += 1;
                }
                named_bar_sync(1, kNT);
                if (threadIdx.x == 0) {
                    *sa.step = s + 1;
                    *sa.epoch = (uint32_t)(epoch + 1);
                    __threadfence();
                }
            }
        }
        if (tr && threadIdx.x == 0) tr[p * 4 + 3] = globaltimer_ns();
        if (p < sa.nphases - 1) grid_arrive(sa);  // its CTA barrier also retires readers of m.ph
    }
    // Every issued piece was waited for by its consumers unless the step
    // aborted; either way no bulk copy may outlive the CTA (bounded wait).
    if (!FORGE_STEP_PRODUCER_WARP && threadIdx.x == 0) {
        const uint32_t issued = m.prod->issued;
        for (uint32_t j = 0; j < (uint32_t)S && j < issued; ++j) {
            const uint32_t idx = issued - 1 - j;
            mbar_wait(&m.full[idx % S], (idx / S) & 1u, sa.err);
        }
    }
}

template <int HD, int G>
size_t smem_for(const ForgeStepArgs& sa, int xf_bytes, int S) {
    return (size_t)S * kStage + 16 * (size_t)S + 4 * (size_t)red_floats<HD, G>() + 4 * (size_t)kSxFloats +
           4 * (size_t)attn_floats<HD, G>() + kProdBytes + kPhaseBytes + (size_t)xf_bytes + 64;
}

template <int HD, int G>
int launch_mk(const ForgeStepArgs& sa0, int xf_bytes, cudaStream_t stream, bool probe_only) {
    auto kern = k_decode_step<HD, G>;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return forge_fail(-1, "decode step attr: %s", cudaGetErrorString(e));
        configured[dev] = true;
    }
    ForgeStepArgs sa = sa0;
    int S = 12;
    while (S >= 4 && smem_for<HD, G>(sa, xf_bytes, S) > 227 * 1024) --S;
    const bool verbose = getenv("FORGE_VERBOSE") != nullptr;
    if (S < 4) {  // does not fit: caller uses the multi-kernel path
        if (verbose) fprintf(stderr, "[forge_b200] fused step: shared memory for %d activation bytes does not fit\n", xf_bytes);
        return 1;
    }
    sa.stages = S;
    const size_t smem = smem_for<HD, G>(sa, xf_bytes, S);
    int nb = 0;
    cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kThreadsMK, smem);
    if (oe != cudaSuccess || nb < 1) {
        if (verbose) {
            cudaFuncAttributes fa{};
            cudaFuncGetAttributes(&fa, kern);
            fprintf(stderr, "[forge_b200] fused step: occupancy %d (%s), smem %zu, stages %d, regs %d, static smem %zu, max threads %d\n",
                    nb, cudaGetErrorString(oe), smem, S, fa.numRegs, fa.sharedSizeBytes, fa.maxThreadsPerBlock);
        }
        cudaGetLastError();
        return 1;
    }
    if (probe_only) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sa.grid);
    cfg.blockDim = dim3(kThreadsMK);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, sa);
    if (e != cudaSuccess) return forge_fail(-1, "decode step launch: %s", cudaGetErrorString(e));
    return 0;
}
}  // namespace

// Returns 0 when launched (or, with probe_only, when the configuration fits),
// 1 when the configuration does not fit one CTA per SM, -1 on error.
int forge_step_attn_tile(int hd) { return hd == 128 ? attn_tile<128>() : attn_tile<64>(); }

int forge_step_launch(const ForgeStepArgs& sa, int xf_bytes, cudaStream_t stream, bool probe_only) {
    const int G = sa.H / sa.Hkv;
    if (sa.hd == 128) {
        switch (G) {
        case 1: return launch_mk<128, 1>(sa, xf_bytes, stream, probe_only);
        case 2: return launch_mk<128, 2>(sa, xf_bytes, stream, probe_only);
        case 4: return launch_mk<128, 4>(sa, xf_bytes, stream, probe_only);
        default: return 1;
        }
    }
    if (sa.hd == 64) {
        switch (G) {
        case 1: return launch_mk<64, 1>(sa, xf_bytes, stream, probe_only);
        case 2: return launch_mk<64, 2>(sa, xf_bytes, stream, probe_only);
        case 4: return launch_mk<64, 4>(sa, xf_bytes, stream, probe_only);
        case 8: return launch_mk<64, 8>(sa, xf_bytes, stream, probe_only);
        default: return 1;
        }
    }
    return 1;
}
