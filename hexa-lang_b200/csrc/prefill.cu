// prefill.cu — causal flash-attention prefill on the 5th-generation tensor
// cores (tcgen05 + TMEM, TMA-fed), head_dim 128 or 64, bf16 in / bf16 out,
// fp32 accumulation.
//
// Semantics follow nn_attn_core_fwd (stdlib/flame/nn_lib.hexa:221-278):
// O = softmax(Q K^T / sqrt(hd) + causal mask) V per (batch, head), the mask
// hiding keys after the query. The reference's own fused prefill kernel
// (tool/r14_walls/flash_attn_bm32_bk32_v0.cu:75) is fp16 wmma at d = 64
// and non-causal only; this is a new kernel for hd = 128 with the mask.
//
// One CTA owns two tiles of 128 query rows of one (batch, head) and walks the
// key blocks of 128 up to the diagonal (k_flash_prefill_pp below):
//   warp 8             TMA: Q of both tiles once, then K and V of every key
//                      block through a 4-slot ring (128-byte swizzled 64 x
//                      128 boxes);
//   warp 9 (one lane)  tensor-core issue: S = Q K^T and O += P V per tile
//                      (tcgen05.mma kind::f16, M 128, N 128, 8 x K16 steps),
//                      alternating tiles so one tile's MMAs overlap the other
//                      tile's softmax;
//   warps 0-3 / 4-7    softmax of tile A / B, one thread per query row: S out
//                      of TMEM (tcgen05.ld), online max / sum in fp32 with
//                      exp2 (the scale folded in), O rescaled in TMEM only
//                      when the row max grows by more than 2^8, P written as
//                      bf16 pairs into TMEM over S (the A operand of O += P V),
//                      and finally O / l to global memory.
// Every wait is bounded (error word, then the CTA drains its copies and
// tensor-core work and frees its TMEM).
#include <cmath>
#include <cstring>
#include <mutex>
#include "tcgen05.cuh"
#include "forge_internal.h"
#include "../../include/forge_b200.h"
#include "../../include/forge_farr.h"

namespace {
constexpr int kBM = 128;                  // query rows per CTA
constexpr int kBN = 128;                  // keys per block
constexpr int kHalf = 128 * 64 * 2;       // 16 KB: 64 columns x 128 rows, swizzled
// one Q / K / V tile: HD / 64 such halves (32 KB at head dim 128, 16 KB at 64)
template <int HD> constexpr int tile_bytes() { return kBM * HD * 2; }
constexpr uint32_t kIdescS = umma_idesc_bf16_f32(kBM, kBN, false);  // B = K rows, K-major

struct PrefillArgs {
    uint16_t* o;
    int B, H, S, causal;
    float scale_log2;  // log2(e) / sqrt(hd)
    uint32_t* err;
    // K/V rows: (b * Hkv + h / (H / Hkv)) * kv_ld + position, so K and V can
    // be a decode KV cache ([B][Hkv][kv_ld][hd], GQA) rather than [B][H][S][hd]
    int Hkv, kv_ld;
};

// 2^x with the hardware approximation (ex2.approx, relative error ~2^-22;
// 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// Packed fp32 pairs (low = first) and the sm_100 two-lane fp32 instructions.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// Two floats to packed bf16x2 (round to nearest even), first in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// ---- two query tiles per CTA -------------------------------------------------------
// Tiles A (rows 256p .. +127) and B (rows 256p+128 .. +255) share every K/V
// block (loaded once) and alternate on the tensor core: while the softmax
// warpgroup of one tile works on its S, the MMA warp runs the other tile's
// S = QK^T or O += PV. TMEM holds S_A, O_A, S_B, O_B (512 columns); the softmax
// reads each S row twice (max, then exp) so no thread holds a whole row, and
// writes P as packed bf16 over the S columns it has read (P of a tile takes
// 64 columns), where the PV MMA takes it as its A operand. S of the next
// block overwrites P only after that MMA: tcgen05 MMAs of one thread run in
// issue order.
// Shared memory: Q_A Q_B | a ring of kPStages 32 KB slots carrying K0 V0 K1
// V1 ... in the order the MMAs use them, so the next block's V and K load
// while the current block is in flight.
constexpr int kPThreads = 320;            // warps 0-3 softmax A, 4-7 softmax B, 8 TMA, 9 MMA
#ifndef FORGE_PREFILL_STAGES
#define FORGE_PREFILL_STAGES 4
#endif
constexpr int kPStages = FORGE_PREFILL_STAGES;  // K/V ring slots (4 or 5 fit)
constexpr int kPOffQ = 0;
template <int HD> constexpr int off_kv() { return 2 * tile_bytes<HD>(); }
template <int HD> constexpr int off_bar() { return (2 + kPStages) * tile_bytes<HD>(); }
template <int HD> constexpr int psmem() { return off_bar<HD>() + 256 + 1024; }
constexpr uint32_t kPTmemCols = 512;

template <int HD>
__global__ void __launch_bounds__(kPThreads, 1)
    k_flash_prefill_pp(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const PrefillArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const uint32_t sbase = smem_u32(base);
    constexpr int kTile = tile_bytes<HD>();
    constexpr int kNH = HD / 64;  // 64-column halves of a tile
    constexpr int kPOffKV = off_kv<HD>();
    constexpr uint32_t kIdescO = umma_idesc_bf16_f32(kBM, HD, true);  // B = V rows, MN-major
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + off_bar<HD>());
    uint64_t* q_full = bars + 0;
    uint64_t* s_full = bars + 1;    // [2] per tile
    uint64_t* p_full = bars + 3;    // [2]
    uint64_t* o_done = bars + 5;    // [2]
    uint64_t* drain = bars + 7;
    uint64_t* kv_full = bars + 8;   // [kPStages]
    uint64_t* kv_empty = bars + 8 + kPStages;
    uint64_t* done = bars + 8 + 2 * kPStages;   // every warp finished (one arrival per warp)
    uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);

    __shared__ uint32_t s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile uint32_t*>(a.err);
    __syncthreads();
    if (s_abort) return;

    const int ntile = a.S / kBM;
    const int npair = (ntile + 1) / 2;
    const int qp = npair - 1 - (int)blockIdx.x;  // longest causal rows first
    const int h = blockIdx.y, b = blockIdx.z;
    const int tA = 2 * qp, tB = 2 * qp + 1;      // query tile indices
    const bool hasB = tB < ntile;
    // key blocks each tile needs (causal: up to its diagonal)
    const int nA = a.causal ? tA + 1 : ntile;
    const int nB = hasB ? (a.causal ? tB + 1 : ntile) : 0;
    const int nblk = nA > nB ? nA : nB;
    const int row0 = (b * a.H + h) * a.S;
    const int row0kv = (b * a.Hkv + h / (a.H / a.Hkv)) * a.kv_ld;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 128);
            mbar_init(&o_done[i], 1);
        }
        for (int i = 0; i < kPStages; ++i) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
        }
        mbar_init(drain, 1);
        mbar_init(done, kPThreads / 32);
        fence_mbar_init();
    }
    if (warp == 9) tmem_alloc(tslot, kPTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    // TMEM columns: S_A 0-127, O_A 128-255, S_B 256-383, O_B 384-511
    const uint32_t tS[2] = {tmem, tmem + 256}, tO[2] = {tmem + 128, tmem + 384};

    if (warp == 8) {
        // --------------------------------------------------------------- TMA
        if (lane == 0) {
            // Q of both tiles, then the K ring
            mbar_arrive_expect_tx(q_full, hasB ? 2 * kTile : kTile);
#pragma unroll
            for (int h2 = 0; h2 < kNH; ++h2) {
                tma_load_2d(base + kPOffQ + h2 * kHalf, &tq, 64 * h2, row0 + tA * kBM, q_full);
                if (hasB) tma_load_2d(base + kPOffQ + kTile + h2 * kHalf, &tq, 64 * h2, row0 + tB * kBM, q_full);
            }
            // item i of the ring: block i / 2, K when i is even, V when odd
            const int nitem = 2 * nblk;
            int issued = 0;
            for (int it = 0; it < nitem; ++it) {
                const int st = it % kPStages;
                if (!mbar_wait(&kv_empty[st], ((it / kPStages) & 1) ^ 1, a.err)) break;
                uint8_t* dst = base + kPOffKV + st * kTile;
                const CUtensorMap* map = (it & 1) ? &tv : &tk;
                const int y = row0kv + (it >> 1) * kBN;
                mbar_arrive_expect_tx(&kv_full[st], kTile);
#pragma unroll
                for (int h2 = 0; h2 < kNH; ++h2) tma_load_2d(dst + h2 * kHalf, map, 64 * h2, y, &kv_full[st]);
                issued = it + 1;
            }
            // every copy issued has landed before the CTA may exit
            mbar_wait(q_full, 0, a.err);
            for (int it = issued > kPStages ? issued - kPStages : 0; it < issued; ++it)
                mbar_wait(&kv_full[it % kPStages], (it / kPStages) & 1, a.err);
        }
    } else if (warp == 9) {
        // ------------------------------------------------------ tensor cores
        if (lane == 0) {
            bool ok = mbar_wait(q_full, 0, a.err);
            auto slot_addr = [&](int it) { return sbase + (uint32_t)(kPOffKV + (it % kPStages) * kTile); };
            auto wait_item = [&](int it) {
                return mbar_wait(&kv_full[it % kPStages], (it / kPStages) & 1, a.err);
            };
            auto issue_s = [&](int t, int j) {
                const uint32_t kb = slot_addr(2 * j);
                const uint32_t qb = sbase + (uint32_t)(kPOffQ + t * kTile);
#pragma unroll
                for (int s = 0; s < HD / 16; ++s) {
                    const uint32_t off = (uint32_t)((s >> 2) * kHalf + (s & 3) * 32);
                    umma_bf16(tS[t], umma_desc_sw128(qb + off, 16, 1024), umma_desc_sw128(kb + off, 16, 1024),
                              kIdescS, s > 0 ? 1u : 0u);
                }
                umma_commit(&s_full[t]);
            };
            // O += P V: P (A operand) from TMEM over S, 8 columns per K16 step
            auto issue_pv = [&](int t, int j) {
                const uint32_t vb = slot_addr(2 * j + 1);
#pragma unroll
                for (int s = 0; s < kBN / 16; ++s)
                    umma_bf16_ta(tO[t], tS[t] + (uint32_t)(8 * s), umma_desc_sw128(vb + (uint32_t)s * 2048u, kHalf, 1024),
                                 kIdescO, (j > 0 || s > 0) ? 1u : 0u);
                umma_commit(&o_done[t]);
            };
            // block 0: S of both tiles
            if (ok && wait_item(0)) {
                tc_fence_after();
                issue_s(0, 0);
                if (nB > 0) issue_s(1, 0);
                umma_commit(&kv_empty[0]);
            } else {
                ok = false;
            }
            for (int j = 0; j < nblk && ok; ++j) {
                const bool useA = j < nA, useB = j < nB;
                if (!wait_item(2 * j + 1)) break;
                if (useA) {
                    if (!mbar_wait(&p_full[0], j & 1, a.err)) break;
                    tc_fence_after();
                    issue_pv(0, j);
                }
                // tile A's next S overlaps tile B's softmax of this block
                const bool nextA = j + 1 < nA, nextB = j + 1 < nB;
                if (nextA || nextB) {
                    if (!wait_item(2 * j + 2)) break;
                    tc_fence_after();
                    if (nextA) issue_s(0, j + 1);
                }
                if (useB) {
                    if (!mbar_wait(&p_full[1], j & 1, a.err)) break;
                    tc_fence_after();
                    issue_pv(1, j);
                }
                umma_commit(&kv_empty[(2 * j + 1) % kPStages]);
                if (nextB) issue_s(1, j + 1);
                if (nextA || nextB) umma_commit(&kv_empty[(2 * j + 2) % kPStages]);
            }
            umma_commit(drain);
            mbar_wait(drain, 0, a.err);
        }
    } else {
        // ------------------------------------------------------------ softmax
        const int t = warp >> 2;                // tile 0 (A) or 1 (B)
        const uint32_t tSm = tmem + (t ? 256u : 0u), tOm = tSm + 128u;  // this tile's S / O columns
        const int r = threadIdx.x & 127;        // query row within the tile
        const int qt = t ? tB : tA;
        const int nmine = t ? nB : nA;
        const uint32_t lrow = (uint32_t)((warp & 3) * 32) << 16;
        const float c = a.scale_log2;
        // Running max in log2 units (m = max * c). It is raised only when a
        // new score exceeds it by more than 8 (P values stay below 2^8, exact
        // enough in bf16 and fp32), so O in TMEM is rescaled rarely; l and O
        // always refer to the same m, so the result does not change.
        float m = -INFINITY, l = 0.f;
        bool ok = nmine > 0;
        for (int j = 0; j < nmine; ++j) {
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, a.err))) { ok = false; break; }
            tc_fence_after();
            const bool diag = a.causal && j == qt;
            // pass 1: row max (two TMEM loads in flight per wait; four
            // independent max chains)
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int q = 0; q < 4; q += 2) {
                uint32_t sv[2][32];
                tmem_ld32(tSm + lrow + 32 * q, sv[0]);
                tmem_ld32(tSm + lrow + 32 * (q + 1), sv[1]);
                tmem_wait_ld();
                if (diag) {
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (32 * (q + h2) + i <= r) mx4[i & 3] = fmaxf(mx4[i & 3], __uint_as_float(sv[h2][i]));
                } else {
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
                        for (int i = 0; i < 32; i += 2)
                            mx4[(i >> 1) & 3] = max3f(mx4[(i >> 1) & 3], __uint_as_float(sv[h2][i]),
                                                      __uint_as_float(sv[h2][i + 1]));
                }
            }
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
            const float mxc = mx * c;
            const bool raise = mxc > m + 8.0f;
            const float m_new = raise ? mxc : m;
            const float alpha = raise ? ex2_approx(m - m_new) : 1.0f;
            if (j > 0) {
                if (!__all_sync(0xffffffffu, mbar_wait(&o_done[t], (j - 1) & 1, a.err))) { ok = false; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, raise)) {
#pragma unroll
                    for (int q = 0; q < HD / 32; ++q) {
                        uint32_t ov[32];
                        tmem_ld32(tOm + lrow + 32 * q, ov);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
                        tmem_st32(tOm + lrow + 32 * q, ov);
                    }
                }
            }
            // pass 2: P = exp2(S * c - m) as bf16 pairs into TMEM over the S
            // columns already read (64 S columns in, 32 P columns out); the
            // causal mask only matters on the diagonal block
            uint64_t sum2 = 0;  // two partial row sums (packed)
            const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(-m_new, -m_new);
#pragma unroll
            for (int q = 0; q < 4; q += 2) {
                uint32_t sv[2][32];
                tmem_ld32(tSm + lrow + 32 * q, sv[0]);
                tmem_ld32(tSm + lrow + 32 * (q + 1), sv[1]);
                tmem_wait_ld();
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    uint32_t pk[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int i = 2 * e, col = 32 * (q + h2) + i;
                        const uint64_t x =
                            f2_fma(f2_pack(__uint_as_float(sv[h2][i]), __uint_as_float(sv[h2][i + 1])), c2, nm2);
                        float p0 = ex2_approx(f2_lo(x)), p1 = ex2_approx(f2_hi(x));
                        if (diag) {
                            p0 = col > r ? 0.f : p0;
                            p1 = col + 1 > r ? 0.f : p1;
                        }
                        sum2 = f2_add(sum2, f2_pack(p0, p1));
                        pk[e] = pack_bf16x2(p0, p1);
                    }
                    tmem_st16(tSm + lrow + (uint32_t)(16 * (q + h2)), pk);
                }
            }
            l = l * alpha + (f2_lo(sum2) + f2_hi(sum2));
            m = m_new;
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[t]);
        }
        if (ok && __all_sync(0xffffffffu, mbar_wait(&o_done[t], (nmine - 1) & 1, a.err))) {
            tc_fence_after();
            const float inv = 1.0f / l;
            uint16_t* orow = a.o + ((size_t)row0 + (size_t)qt * kBM + r) * HD;
#pragma unroll
            for (int q = 0; q < HD / 32; ++q) {
                uint32_t ov[32];
                tmem_ld32(tOm + lrow + 32 * q, ov);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i += 8) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        w[e] = (uint32_t)f32_to_bf16_bits(__uint_as_float(ov[i + 2 * e]) * inv) |
                               ((uint32_t)f32_to_bf16_bits(__uint_as_float(ov[i + 2 * e + 1]) * inv) << 16);
                    *reinterpret_cast<uint4*>(orow + 32 * q + i) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
        }
    }
    // End: every warp reports on an mbarrier and the TMEM-owning warp waits
    // for all of them before it frees TMEM (after the single-lane TMA and MMA
    // roles a CTA-wide bar.sync is not relied on to hold the other warps).
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(done);
    if (warp == 9) {
        mbar_wait(done, 0, a.err);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kPTmemCols);
    }
}

// ---- host ------------------------------------------------------------------------
// [rows][128] bf16 viewed as 64-column x 128-row boxes, 128-byte swizzle.
int make_map(CUtensorMap* m, const void* ptr, int64_t rows, int hd) {
    ForgeEncodeTiled enc = forge_tensor_map_encoder();
    if (!enc) return forge_fail(-1, "flash prefill: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0
                             : forge_fail(-1, "flash prefill: tensor map encode failed (%d): ptr %p rows %lld map%%64 %d",
                                          (int)r, ptr, (long long)rows, (int)((uintptr_t)m % 64));
}

int configure() {
    static bool done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return forge_fail(-1, "flash prefill: no device");
    if (done[dev]) return 0;
    cudaError_t e = cudaFuncSetAttribute(k_flash_prefill_pp<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, psmem<128>());
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_flash_prefill_pp<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, psmem<64>());
    if (e != cudaSuccess) return forge_fail(-1, "flash prefill: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    done[dev] = true;
    return 0;
}
}  // namespace

// cuTensorMapEncodeTiled from the driver (through the runtime, no -lcuda).
ForgeEncodeTiled forge_tensor_map_encoder() {
    static ForgeEncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<ForgeEncodeTiled>(p);
    });
    return fn;
}


extern "C" FORGE_API int forge_flash_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o,
                                             int B, int H, int S, int hd, int causal, void* stream) {
    if (!q || !k || !v || !o || B <= 0 || H <= 0 || S <= 0)
        return forge_fail(FORGE_INVALID_ARGS, "forge_flash_prefill: bad args");
    if (hd != 128 && hd != 64)
        return forge_fail(FORGE_KERNEL_UNSUPPORTED, "forge_flash_prefill: head_dim %d (128 or 64)", hd);
    if (S % kBM) return forge_fail(FORGE_KERNEL_UNSUPPORTED, "forge_flash_prefill: seq_len %d not a multiple of 128", S);
    if ((int64_t)B * H * S > (1ll << 31) - 1 || H > 65535 || B > 65535)
        return forge_fail(FORGE_INVALID_ARGS, "forge_flash_prefill: shape too large");
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15)
        return forge_fail(FORGE_INVALID_ARGS, "forge_flash_prefill: arrays must be 16-byte aligned");
    if (configure()) return -1;
    uint32_t* err = forge_ops_err_word();
    if (!err) return forge_fail(-1, "forge_flash_prefill: no device");
    const int64_t rows = (int64_t)B * H * S;
    CUtensorMap mq, mk, mv;
    if (make_map(&mq, q, rows, hd) || make_map(&mk, k, rows, hd) || make_map(&mv, v, rows, hd)) return -1;
    PrefillArgs a{o, B, H, S, causal ? 1 : 0, (float)(1.4426950408889634 / std::sqrt((double)hd)), err, H, S};
    dim3 grid((unsigned)((S / kBM + 1) / 2), (unsigned)H, (unsigned)B);
    if (hd == 128)
        k_flash_prefill_pp<128><<<grid, kPThreads, psmem<128>(), (cudaStream_t)stream>>>(mq, mk, mv, a);
    else
        k_flash_prefill_pp<64><<<grid, kPThreads, psmem<64>(), (cudaStream_t)stream>>>(mq, mk, mv, a);
    return forge_check_launch("forge_flash_prefill");
}

// Causal prefill of B sequences of S positions (S a multiple of 128) with
// Q and O as [B][H][S][hd] bf16 and K / V read in place from a decode KV
// cache layer [.. B ..][Hkv][kv_ld][hd] (kv_rows rows in all), GQA heads
// h -> h / (H / Hkv). Used by the engine's prompt prefill.
int forge_flash_prefill_kv(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, uint16_t* o, int B, int H,
                           int Hkv, int S, int hd, int kv_ld, int64_t kv_rows, cudaStream_t stream) {
    if (!q || !kc || !vc || !o || B <= 0 || H <= 0 || Hkv <= 0 || H % Hkv || S <= 0 || S % kBM || kv_ld < S ||
        (hd != 128 && hd != 64) ||
        (int64_t)B * Hkv * kv_ld > kv_rows || kv_rows > (1ll << 31) - 1 || (int64_t)B * H * S > (1ll << 31) - 1)
        return forge_fail(FORGE_INVALID_ARGS, "flash prefill (cache): bad shape");
    if (((uintptr_t)q | (uintptr_t)kc | (uintptr_t)vc | (uintptr_t)o) & 15)
        return forge_fail(FORGE_INVALID_ARGS, "flash prefill (cache): arrays must be 16-byte aligned");
    if (configure()) return -1;
    uint32_t* err = forge_ops_err_word();
    if (!err) return forge_fail(-1, "flash prefill (cache): no device");
    CUtensorMap mq, mk, mv;
    if (make_map(&mq, q, (int64_t)B * H * S, hd) || make_map(&mk, kc, kv_rows, hd) || make_map(&mv, vc, kv_rows, hd))
        return -1;
    PrefillArgs a{o, B, H, S, 1, (float)(1.4426950408889634 / std::sqrt((double)hd)), err, Hkv, kv_ld};
    dim3 grid((unsigned)((S / kBM + 1) / 2), (unsigned)H, (unsigned)B);
    if (hd == 128)
        k_flash_prefill_pp<128><<<grid, kPThreads, psmem<128>(), stream>>>(mq, mk, mv, a);
    else
        k_flash_prefill_pp<64><<<grid, kPThreads, psmem<64>(), stream>>>(mq, mk, mv, a);
    return forge_check_launch("forge_flash_prefill_kv");
}

// FLASH_PREFILL family: in = [Q, K, V (HexaFarrBf16, [B][H][S][hd]), causal],
// out = [O]; shape M = B, N = H, K = hd, batch = S.
int forge_prefill_dispatch(const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out) {
    if (in->count < 3 || out->count < 1 || s->M <= 0 || s->N <= 0 || s->K <= 0 || s->batch <= 0)
        return FORGE_INVALID_ARGS;
    const int64_t n = s->M * s->N * s->batch * s->K;
    HexaFarrBf16* F[4] = {(HexaFarrBf16*)(intptr_t)in->farr_ids[0], (HexaFarrBf16*)(intptr_t)in->farr_ids[1],
                          (HexaFarrBf16*)(intptr_t)in->farr_ids[2], (HexaFarrBf16*)(intptr_t)out->farr_ids[0]};
    for (int i = 0; i < 4; ++i)
        if (!F[i] || F[i]->len < n) return FORGE_INVALID_ARGS;
    for (int i = 0; i < 3; ++i)
        if (hexa_farr_bf16_to_device(F[i])) return FORGE_INVALID_ARGS;
    if (!F[3]->d_buf && cudaMalloc(&F[3]->d_buf, (size_t)F[3]->len * 2) != cudaSuccess) {
        cudaGetLastError();
        F[3]->d_buf = nullptr;
        return FORGE_INVALID_ARGS;
    }
    F[3]->loc = FARR_BF16_LOC_DEVICE;
    const int causal = in->count > 3 ? (int)in->farr_ids[3] : 1;
    const int rc = forge_flash_prefill((const uint16_t*)F[0]->d_buf, (const uint16_t*)F[1]->d_buf,
                                       (const uint16_t*)F[2]->d_buf, (uint16_t*)F[3]->d_buf, (int)s->M, (int)s->N,
                                       (int)s->batch, (int)s->K, causal, nullptr);
    return rc == 0 ? FORGE_OK : (rc == FORGE_INVALID_ARGS ? FORGE_INVALID_ARGS : FORGE_KERNEL_UNSUPPORTED);
}
