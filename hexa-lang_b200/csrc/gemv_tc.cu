// gemv_tc.cu — int4 decode GEMV for 5..32 sequences on the 5th-generation
// tensor cores (tcgen05.mma kind::i8, accumulators in TMEM).
//
// Arithmetic is that of the small-batch kernel (gemv.cu): int4 codes
// (code = q + 7) as unsigned 8-bit A, activations as int8 hi/lo pairs per
// 128-group as signed 8-bit B, an exact 32-bit integer dot product per group,
// then per group and sequence: remove the code bias (7 x column sum),
// recombine hi + lo / 256 and apply the weight and activation scales in
// fp32. Only the order of the fp32 sums over groups differs from the
// register-fragment kernels.
//
// Why tensor memory: at 32 sequences every 128-row weight tile meets 8 KB of
// activations per group. The register-fragment path re-loads them into every
// warp (latency- and register-bound at ~0.8 TB/s); here one MMA per 32 k
// takes both operands from shared memory and each group's 128 x 64 integer
// accumulator is read once from TMEM.
//
// Data: k_quant_x_tc writes, per 128-group g, one block of
//   [64 columns][128 k] int8, 128-byte swizzled (the layout a K-major SW128
//   UMMA operand has in shared memory; column 2b = hi, 2b+1 = lo of sequence
//   b), then sx[32] fp32 and per column 0x4B400000 - 7 x column sum (s32: the
//   code bias folded with the exponent bits of 1.5 x 2^23, so accumulator +
//   term read as fp32, minus 1.5 x 2^23, is the corrected dot product),
// so the producer moves it with one plain bulk copy.
//
// k_gemv_tc, one CTA per SM, 448 threads (four warps share a sub-partition,
// so at most 128 registers a thread):
//   warp 0       three copies per (tile, group) unit into a 6-slot ring: the
//                int4 chunks of the tile's eight 16-row blocks and their
//                scale blocks (2-D TMA boxes: a 16-row block is one row of
//                8-byte elements) and the group's activation block (8 slots);
//   warp 1       TMEM (4 accumulators of 64 columns, so the MMAs run up to
//                four groups ahead of the arithmetic) and the MMA issue:
//                4 x K32 per group;
//   warps 2-5    int4 -> u8 into a 128 x 128 swizzled A tile (4-slot ring);
//   warps 6-13   per group: tcgen05.ld of the row's accumulators (warp w:
//                TMEM lanes 32 (w % 4) .., sequences 16 ((w - 6) / 4) .. +15),
//                then the bias / hi-lo / scale arithmetic into fp32 sums.
// Work is split stream-K: the (tile, group) units of the matrix in tile-major
// order are cut into one contiguous range per CTA; a tile split between CTAs
// is finished by the last of them to arrive (atomic ticket), which adds the
// partial sums in CTA order and runs the fused epilogue.
// Every wait is bounded (error word, then the CTA drains and frees TMEM).
#include "common.cuh"
#include "layout.cuh"
#include "tcgen05.cuh"
#include "forge_internal.h"
#include "gemv_core.cuh"

namespace {
constexpr int kTM = 128;                       // weight rows per tile (MMA M)
constexpr int kMaxSeq = 32;                    // N = 2 x sequences <= 64
constexpr int kActTile = 64 * 128;             // B tile: 64 columns x 128 k
constexpr int kActAux = 128 + 256;             // sx[32] f32 + code-bias terms [64] s32
constexpr int kActGroup = kActTile + kActAux;  // one group's block in global memory
// A unit of work is two 128-groups of one 128-row tile (one group when the
// tile row has an odd group count and this is its last unit). Raw ring slot:
// per group its activation tile + sx + sums (one plain bulk copy each, the
// tiles 1024-aligned) | weights (8 blocks x 2 groups x 1 KB, one 2-D TMA
// box) | scale blocks (8 x 128 B, one box; a box holds 4 groups).
constexpr int kGU = 2;                          // groups per unit
constexpr int kSlotAct0 = 0, kSlotAct1 = 9216, kSlotW = 18432, kSlotS = 34816;
constexpr int kSlot = 35840;                    // 1024-aligned slots
constexpr int kNS = 4;
constexpr int kATile = kTM * 128;               // u8 A tile of one group, 16 KB
constexpr int kNA = 2;                          // A slots of a unit (kGU tiles each)
constexpr int kNAcc = 2;                        // TMEM accumulator sets of a unit (kGU x 64 columns)
constexpr int kOffA = kNS * kSlot;
constexpr int kOffBar = kOffA + kNA * kGU * kATile;
constexpr int kSmem = kOffBar + 512 + 1024;    // barriers + alignment slack
constexpr int kThreads = 448;
constexpr int kWarpMma = 1, kWarpUnpack = 2, kWarpEpi = 6;  // arithmetic: warps 6-13
constexpr int kEpiThreads = 256;
constexpr uint32_t kTmemCols = 64 * kGU * kNAcc;

// Byte offset of (row, byte kb) in a [rows][128 B] tile with 128-byte swizzle
// (8-row atoms of 1 KB; the 16-byte chunk index is XORed with row % 8).
__host__ __device__ __forceinline__ int swz128(int row, int kb) {
    return (row >> 3) * 1024 + (row & 7) * 128 + ((((kb >> 4) ^ row) & 7) << 4) + (kb & 15);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        ::"r"(tmem_d), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
// kind::i8 instruction descriptor: D s32 (2), A u8 (0), B s8 (1), both K-major.
__host__ __device__ constexpr uint32_t idesc_u8s8(int M, int N) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// One CTA per sequence: the small-batch staging (batch 1) into shared memory,
// then the per-group blocks of the tensor-core layout.
template <int PRO>
__global__ void __launch_bounds__(256) k_quant_x_tc(const ForgeGemvArgs a, uint8_t* xt) {
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
    for (int i = threadIdx.x; i < a.K / 2; i += 256) {  // 4-k words of the hi and lo columns
        const int k = (i >> 1) * 4, hl = i & 1;
        const int g = k >> 7, col = 2 * b + hl;
        *reinterpret_cast<uint32_t*>(xt + (size_t)g * kActGroup + swz128(col, k & 127)) =
            *reinterpret_cast<const uint32_t*>(xq + xq_index(k, hl, 2));
    }
    for (int g = threadIdx.x; g < G; g += 256) {
        uint8_t* aux = xt + (size_t)g * kActGroup + kActTile;
        reinterpret_cast<float*>(aux)[b] = sxf[g * 4];
        reinterpret_cast<int*>(aux + 128)[2 * b] = 0x4B400000 - 7 * ssum[g * 8];
        reinterpret_cast<int*>(aux + 128)[2 * b + 1] = 0x4B400000 - 7 * ssum[g * 8 + 1];
    }
}

struct TcArgs {
    const uint8_t* xt;   // activation blocks [G][kActGroup]
    float* partial;      // [grid][2][128][32]
    int* ticket;         // [tiles], zero between launches
    int npad;            // MMA N: 2 x sequences rounded up to 16
    int wbox;            // weight box width in 8-byte elements: 128 per group of a unit
};

// First unit of CTA c and the CTA that owns unit x, for U units over P CTAs.
__device__ __forceinline__ int64_t unit_begin(int c, int64_t U, int P) { return (int64_t)c * U / P; }
__device__ __forceinline__ int unit_owner(int64_t x, int64_t U, int P) { return (int)(((x + 1) * P - 1) / U); }

template <int EPI>
__global__ void __maxnreg__(128) k_gemv_tc(const __grid_constant__ CUtensorMap tw,
                                                         const __grid_constant__ CUtensorMap ts, const ForgeGemvArgs a,
                                                         const TcArgs t) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const uint32_t sbase = smem_u32(base);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + kOffBar);
    uint64_t* raw_full = bars;               // [kNS]
    uint64_t* raw_empty = bars + kNS;        // [kNS]
    uint64_t* a_full = bars + 2 * kNS;       // [kNA]
    uint64_t* a_empty = a_full + kNA;        // [kNA]
    uint64_t* acc_full = a_empty + kNA;      // [kNAcc]
    uint64_t* acc_empty = acc_full + kNAcc;  // [kNAcc]
    uint64_t* drain = acc_empty + kNAcc;
    uint64_t* done = drain + 1;              // every warp finished (one arrival per warp)
    uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int s_last, s_fail;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.K >> 7;
    const int G2 = (G + kGU - 1) / kGU;  // units per tile
    const int T = (a.N + kTM - 1) / kTM;
    const int nunit16 = a.N >> 4;
    const int64_t U = (int64_t)T * G2;
    const int P = gridDim.x;
    const int64_t u0 = unit_begin(blockIdx.x, U, P), u1 = unit_begin(blockIdx.x + 1, U, P);
    const int nmine = (int)(u1 - u0);
    // (tile, group pair) of the first unit; later units step through them
    // incrementally (a 64-bit division per unit and thread kept the
    // conversion unit ~50% busy in an earlier version)
    const int tl0 = (int)(u0 / G2), g0 = (int)(u0 - (int64_t)tl0 * G2);
    const int wrow = t.wbox * 8;  // bytes of one 16-row block in the weight box

    if (threadIdx.x == 0) {
        for (int i = 0; i < kNS; ++i) {
            mbar_init(&raw_full[i], 1);
            // one arrival per unpack and arithmetic warp (after every lane
            // has used what it read) and the MMA commit
            mbar_init(&raw_empty[i], 4 + 1 + kEpiThreads / 32);
        }
        for (int i = 0; i < kNA; ++i) {
            mbar_init(&a_full[i], 4);  // per unpack warp: every lane's stores and proxy fence, then one arrival
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < kNAcc; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiThreads / 32);
        }
        mbar_init(drain, 1);
        mbar_init(done, kThreads / 32);
        fence_mbar_init();
        s_fail = 0;
    }
    if (warp == kWarpMma) tmem_alloc(tslot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 0) {
        // ------------------------------------------------------------ copies
        if (lane == 0) {
            // weights: box {1 group = 128 x 8 B, 8 blocks} at (128 g, 8 tile);
            // scales: box {16 x 8 B, 8 blocks} at (16 (g / 4), 8 tile). Rows
            // past N read as zeros and count in full.
            // weights: box {2 groups = 256 x 8 B, 8 blocks} at (256 pr, 8
            // tile) (a group past K reads as zeros and counts in full);
            // scales: box {16 x 8 B, 8 blocks} at (16 (2 pr / 4), 8 tile)
            auto weights = [&](int i) {
                const int gi = g0 + i, tl = tl0 + gi / G2, pr = gi - (gi / G2) * G2;
                uint8_t* slot = base + (i % kNS) * kSlot;
                tma_load_2d(slot + kSlotW, &tw, 256 * pr, 8 * tl, &raw_full[i % kNS]);
                tma_load_2d(slot + kSlotS, &ts, 16 * (pr >> 1), 8 * tl, &raw_full[i % kNS]);
            };
            auto two = [&](int i) {
                const int gi = g0 + i, pr = gi - (gi / G2) * G2;
                return 2 * pr + 1 < G;
            };
            auto acts = [&](int i) {
                const int gi = g0 + i, g = 2 * (gi - (gi / G2) * G2);
                uint8_t* slot = base + (i % kNS) * kSlot;
                bulk_g2s(slot + kSlotAct0, t.xt + (size_t)g * kActGroup, kActGroup, &raw_full[i % kNS]);
                if (g + 1 < G)
                    bulk_g2s(slot + kSlotAct1, t.xt + (size_t)(g + 1) * kActGroup, kActGroup, &raw_full[i % kNS]);
            };
            auto wbytes = [&](int i) { return (uint32_t)(wrow * 8 + 8 * 128 + (two(i) ? 0 : -kActGroup)); };
            // weights do not depend on the previous kernel: the first ring's
            // worth is requested before the dependency wait
            const int pre = min(kNS, nmine);
            for (int i = 0; i < pre; ++i) {
                mbar_arrive_expect_tx(&raw_full[i], wbytes(i) + 2 * kActGroup);
                weights(i);
            }
            pdl_wait();
            for (int i = 0; i < pre; ++i) acts(i);
            int issued = pre;
            for (int i = pre; i < nmine; ++i) {
                const int s = i % kNS;
                if (!mbar_wait(&raw_empty[s], ((i / kNS) & 1) ^ 1, a.err)) break;
                mbar_arrive_expect_tx(&raw_full[s], wbytes(i) + 2 * kActGroup);
                weights(i);
                acts(i);
                issued = i + 1;
            }
            for (int i = issued > kNS ? issued - kNS : 0; i < issued; ++i)
                mbar_wait(&raw_full[i % kNS], (i / kNS) & 1, a.err);
        }
        __syncwarp();  // the warp reaches the final barrier converged
    } else if (warp == kWarpMma) {
        // ------------------------------------------------------ tensor cores
        if (lane == 0) {
            const uint32_t idesc = idesc_u8s8(kTM, t.npad);
            int done = 0;
            for (int i = 0; i < nmine; ++i) {
                const int s = i % kNS, as = i % kNA, tb = i % kNAcc;
                const int gi = g0 + i, pr = gi - (gi / G2) * G2;
                const int nh = 2 * pr + 1 < G ? 2 : 1;
                if (!mbar_wait(&raw_full[s], (i / kNS) & 1, a.err)) break;
                if (!mbar_wait(&a_full[as], (i / kNA) & 1, a.err)) break;
                if (!mbar_wait(&acc_empty[tb], ((i / kNAcc) & 1) ^ 1, a.err)) break;
                tc_fence_after();
                for (int h = 0; h < nh; ++h) {
                    const uint32_t ab = sbase + (uint32_t)(kOffA + (as * kGU + h) * kATile);
                    const uint32_t bb = sbase + (uint32_t)(s * kSlot + (h ? kSlotAct1 : kSlotAct0));
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        umma_i8(tmem + (uint32_t)((tb * kGU + h) * 64), umma_desc_sw128(ab + 32 * k, 16, 1024),
                                umma_desc_sw128(bb + 32 * k, 16, 1024), idesc, k > 0 ? 1u : 0u);
                }
                umma_commit(&acc_full[tb]);
                umma_commit(&a_empty[as]);
                umma_commit(&raw_empty[s]);
                done = i + 1;
            }
            (void)done;
            umma_commit(drain);
            mbar_wait(drain, 0, a.err);
        }
        __syncwarp();
    } else if (warp < kWarpEpi) {
        // ------------------------------------------- int4 -> u8 A operand
        const int ut = threadIdx.x - kWarpUnpack * 32;  // 0..127
        int pr = g0 - 1;
        for (int i = 0; i < nmine; ++i) {
            if (++pr == G2) pr = 0;
            const int s = i % kNS, as = i % kNA;
            const int nh = 2 * pr + 1 < G ? 2 : 1;
            const bool ok = mbar_wait(&raw_full[s], (i / kNS) & 1, a.err) &&
                            mbar_wait(&a_empty[as], ((i / kNA) & 1) ^ 1, a.err);
            if (!__all_sync(0xffffffffu, ok)) break;
            for (int h = 0; h < nh; ++h) {
            const uint8_t* src = base + s * kSlot + kSlotW + h * 1024;
            uint8_t* dst = base + kOffA + (as * kGU + h) * kATile;
            // records = (16-row block, 64-k chunk, lane) of the packed layout;
            // blocks past N arrived as zeros, so every record is converted
            uint4 v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int rec = ut + 128 * j;
                v[j] = *reinterpret_cast<const uint4*>(src + (rec >> 6) * wrow + (rec & 63) * 16);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int rec = ut + 128 * j;
                const int rb = rec >> 6, c = (rec >> 5) & 1, ln = rec & 31, gg = ln >> 2, tt = ln & 3;
                const int row = 16 * rb + gg;
                const uint32_t w4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const int kb = 64 * c + 32 * (w >> 1) + 16 * (w & 1) + 4 * tt;
                    *reinterpret_cast<uint32_t*>(dst + swz128(row, kb)) = w4[w] & 0x0F0F0F0Fu;
                    *reinterpret_cast<uint32_t*>(dst + swz128(row + 8, kb)) = (w4[w] >> 4) & 0x0F0F0F0Fu;
                }
            }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&a_full[as]);
                mbar_arrive(&raw_empty[s]);
            }
        }
    } else {
        // ------------------------------------------------- group arithmetic
        pdl_wait();  // outputs and the partial/ticket scratch of the previous launch
        const int q = warp & 3;                     // TMEM lane quarter this warp may read
        const int hcol = (warp - kWarpEpi) >> 2;    // sequences 16 hcol .. +15
        constexpr int kHalfSeq = kMaxSeq / 2;
        const int row = 32 * q + lane;              // row within the tile
        const int r16 = row & 15;
        const uint32_t tl_addr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(32 * hcol);
        const int nseq = a.batch;
        const int nchunk = t.npad >> 4;             // 16-column chunks in use (8 sequences each)
        float y[kHalfSeq];
#pragma unroll
        for (int b = 0; b < kHalfSeq; ++b) y[b] = 0.f;
        int piece_g0 = g0;
        // A wait that runs out sets the error word; the warp then stops
        // working but still takes the piece-end barriers with the others.
        bool ok = true;
        int tl = tl0, g = g0 - 1;
        for (int i = 0; i < nmine; ++i) {
            if (++g == G2) { g = 0; ++tl; }  // g: the unit's group pair within the tile
            const int s = i % kNS, tb = i % kNAcc;
            const int nh = 2 * g + 1 < G ? 2 : 1;
            if (ok) {
                const bool w1 = mbar_wait(&acc_full[tb], (i / kNAcc) & 1, a.err) &&
                                mbar_wait(&raw_full[s], (i / kNS) & 1, a.err);
                ok = __all_sync(0xffffffffu, w1);
            }
            if (ok) {
                tc_fence_after();
                const uint8_t* slot = base + s * kSlot;
                for (int h = 0; h < nh; ++h) {
                uint32_t acc[2][16];  // columns past 2 x batch hold stale values, never stored
                tmem_ld16(tl_addr + (uint32_t)((tb * kGU + h) * 64), acc[0]);
                tmem_ld16(tl_addr + (uint32_t)((tb * kGU + h) * 64 + 16), acc[1]);
                // this warp's scales and bias terms of group 2 g + h, loaded
                // while the accumulator load is in flight
                const int aux = (h ? kSlotAct1 : kSlotAct0) + kActTile;
                const float4* sx4 = reinterpret_cast<const float4*>(slot + aux);
                const int4* bias4 = reinterpret_cast<const int4*>(slot + aux + 128);
                const int gg = 2 * g + h;
                const float sw = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(
                    slot + kSlotS + (row >> 4) * 128 + (r16 & 7) * 16 + (gg & 3) * 4 + (r16 >> 3) * 2));
                float sxc[2][8];
                int bias[2][16];
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int cc = 2 * hcol + c;  // 16-column chunk of the accumulator
                    const float4 xa = sx4[2 * cc], xb = sx4[2 * cc + 1];
                    sxc[c][0] = xa.x; sxc[c][1] = xa.y; sxc[c][2] = xa.z; sxc[c][3] = xa.w;
                    sxc[c][4] = xb.x; sxc[c][5] = xb.y; sxc[c][6] = xb.z; sxc[c][7] = xb.w;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int4 bj = bias4[4 * cc + j];
                        bias[c][4 * j] = bj.x; bias[c][4 * j + 1] = bj.y; bias[c][4 * j + 2] = bj.z; bias[c][4 * j + 3] = bj.w;
                    }
                }
                tmem_wait_ld();
                if (h == nh - 1) {  // every accumulator of the unit read
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[tb]);
                }
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    if (2 * hcol + c < nchunk) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float fhi = __int_as_float((int)acc[c][2 * e] + bias[c][2 * e]) - 12582912.0f;
                            const float flo = __int_as_float((int)acc[c][2 * e + 1] + bias[c][2 * e + 1]) - 12582912.0f;
                            y[8 * c + e] = fmaf(sw * sxc[c][e], fmaf(flo, 1.0f / 256.0f, fhi), y[8 * c + e]);
                        }
                    }
                }
                }
                // the slot goes back to the copies only after the values read
                // from it have been used: releasing with those shared-memory
                // loads still outstanding let the next copy overwrite them
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[s]);
            }
            // end of this CTA's piece of tile tl (the same iterations in every warp)
            if (g == G2 - 1 || i == nmine - 1) {
                const bool whole = piece_g0 == 0 && g == G2 - 1;
                bool fin = whole && ok;
                if (!whole) {
                    const int k = (tl0 == tl) ? 0 : 1;  // first or last piece of this CTA
                    // 16 floats per thread (columns past the batch carry
                    // values that are never stored)
                    float4* pp = reinterpret_cast<float4*>(t.partial + (((size_t)blockIdx.x * 2 + k) * kTM + row) * kMaxSeq +
                                                           kHalfSeq * hcol);
                    if (ok) {
#pragma unroll
                        for (int j = 0; j < kHalfSeq / 4; ++j)
                            pp[j] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
                    } else if (lane == 0) {
                        s_fail = 1;
                    }
                    // ticket: the barrier orders the epilogue threads' partial
                    // stores before one acquire-release atomic; the last
                    // arrival's acquire reaches every epilogue thread through
                    // the second barrier
                    named_bar_sync(1, kEpiThreads);
                    if (threadIdx.x == kWarpEpi * 32) {
                        int last = 0;
                        if (!s_fail) {
                            const int n = g - piece_g0 + 1;
                            uint32_t old;
                            asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;"
                                         : "=r"(old) : "l"(t.ticket + tl), "r"((uint32_t)n) : "memory");
                            last = ((int)old + n == G2) ? 1 : 0;
                        }
                        s_last = last;
                    }
                    named_bar_sync(1, kEpiThreads);
                    fin = s_last != 0;
                    if (fin) {
                        // the tile's pieces in CTA order
                        const int c0 = unit_owner((int64_t)tl * G2, U, P);
                        const int c1 = unit_owner((int64_t)tl * G2 + G2 - 1, U, P);
#pragma unroll
                        for (int b = 0; b < kHalfSeq; ++b) y[b] = 0.f;
                        // vector loads, all of a piece in flight together
#pragma unroll 2
                        for (int c = c0; c <= c1; ++c) {
                            const int kk = (unit_begin(c, U, P) / G2 == tl) ? 0 : 1;
                            const float4* src = reinterpret_cast<const float4*>(
                                t.partial + (((size_t)c * 2 + kk) * kTM + row) * kMaxSeq + kHalfSeq * hcol);
                            float4 v[kHalfSeq / 4];
#pragma unroll
                            for (int j = 0; j < kHalfSeq / 4; ++j) v[j] = __ldcg(src + j);
#pragma unroll
                            for (int j = 0; j < kHalfSeq / 4; ++j) {
                                y[4 * j] += v[j].x; y[4 * j + 1] += v[j].y; y[4 * j + 2] += v[j].z; y[4 * j + 3] += v[j].w;
                            }
                        }
                        if (threadIdx.x == kWarpEpi * 32) t.ticket[tl] = 0;
                    }
                }
                if (fin) {
                    // rows r and r + 8 of a 16-row block are lanes l and l ^ 8
                    const int blk = 8 * tl + (row >> 4);
                    unsigned long long best = 0ull;
#pragma unroll
                    for (int b = 0; b < kHalfSeq; ++b) {
                        const float yhi = __shfl_xor_sync(0xffffffffu, y[b], 8);
                        const int bg = kHalfSeq * hcol + b;
                        if (bg < nseq && (lane & 8) == 0 && blk < nunit16)
                            epilogue<EPI>(a, blk, r16, bg, y[b], yhi, best);
                    }
                }
#pragma unroll
                for (int b = 0; b < kHalfSeq; ++b) y[b] = 0.f;
                piece_g0 = 0;
            }
        }
    }
    // End: every warp reports on an mbarrier and the TMEM-owning warp waits
    // for all of them before it frees TMEM and lets dependent launches in
    // (a CTA-wide bar.sync here was measured to release threads of the
    // single-lane roles before the arithmetic warps had arrived).
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(done);
    if (warp == kWarpMma) {
        mbar_wait(done, 0, a.err);
        __syncwarp();
        if (lane == 0) pdl_trigger();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

template <int PRO>
int launch_quant(const ForgeGemvArgs& a, uint8_t* xt, cudaStream_t stream, bool pdl) {
    const int smem = 16 * 4 + (a.K / 128) * 12 * 4 + a.K * 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.batch);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_quant_x_tc<PRO>, a, xt);
    return e == cudaSuccess ? 0 : forge_fail(-1, "tensor-core activation quantise launch: %s", cudaGetErrorString(e));
}

// A 2-D map of 8-byte elements over rows of `row_bytes` (one row per 16-row
// weight block), box {box_x elements, 8 rows}, no swizzle.
int map_rows(CUtensorMap* m, const void* ptr, int64_t row_bytes, int64_t rows, int box_x) {
    ForgeEncodeTiled enc = forge_tensor_map_encoder();
    if (!enc) return forge_fail(-1, "tc gemv: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)box_x, 8};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : forge_fail(-1, "tc gemv: tensor map encode failed (%d)", (int)r);
}

template <int EPI>
int launch_tc(const ForgeGemvArgs& a, const TcArgs& t, cudaStream_t stream, int grid) {
    CUtensorMap tw, ts;
    const int64_t blocks = a.N / 16;
    if (map_rows(&tw, a.w, (int64_t)a.K * 8, blocks, t.wbox) ||
        map_rows(&ts, a.s, q4_groups4(a.K, 128) * 128, blocks, 16))
        return -1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemv_tc<EPI>, tw, ts, a, t);
    return e == cudaSuccess ? 0 : forge_fail(-1, "tensor-core gemv launch: %s", cudaGetErrorString(e));
}

constexpr int kMaxGrid = 160;     // partial slots (>= SMs of a B200)
constexpr int kMaxTiles = 4096;   // ticket counters (N <= 524288)
constexpr int64_t kPartialBytes = (int64_t)kMaxGrid * 2 * kTM * kMaxSeq * 4;
}  // namespace

// Scratch of the batched GEMV paths: a fixed header holding the tensor-core
// path's ticket counters (zero when the scratch is first used, and left zero
// by every launch), which no other path writes; then, for the tensor-core
// path, the partial sums and the activation blocks.
int64_t forge_gemv_scratch_header() { return (int64_t)kMaxTiles * 4; }
int64_t forge_gemv_tc_scratch_bytes(int K) {
    return forge_gemv_scratch_header() + kPartialBytes + (int64_t)(K / 128) * kActGroup;
}

int forge_gemv_tc_configure() {
    static bool done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return forge_fail(-1, "tc gemv: no device");
    if (done[dev]) return 0;
    cudaError_t e = cudaSuccess;
    auto set = [&](const void* f, int bytes) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    };
    set((const void*)k_gemv_tc<FORGE_EPI_STORE>, kSmem);
    set((const void*)k_gemv_tc<FORGE_EPI_RESID>, kSmem);
    set((const void*)k_gemv_tc<FORGE_EPI_QKV>, kSmem);
    set((const void*)k_gemv_tc<FORGE_EPI_SWIGLU>, kSmem);
    set((const void*)k_quant_x_tc<FORGE_PRO_PLAIN>, 227 * 1024);
    set((const void*)k_quant_x_tc<FORGE_PRO_RMSNORM>, 227 * 1024);
    if (e != cudaSuccess) return forge_fail(-1, "tc gemv: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    done[dev] = true;
    return 0;
}

// One chunk of 1..32 sequences of an int4 GEMV: quantise the activations,
// then one weight stream through the tensor cores.
int forge_gemv_tc_launch(const ForgeGemvArgs& a, void* scratch, cudaStream_t stream, bool pdl) {
    if (a.wkind != FORGE_W_Q4 || a.batch <= 0 || a.batch > kMaxSeq || !scratch || (a.K % 128) || (a.N % 16))
        return forge_fail(-1, "tc gemv: int4, 1..%d sequences, K %% 128 == 0, N %% 16 == 0", kMaxSeq);
    if (a.pro == FORGE_PRO_EMBED_RMSNORM || a.epi == FORGE_EPI_LOGITS)
        return forge_fail(-1, "tc gemv: prologue/epilogue not supported");
    if (((uintptr_t)a.w | (uintptr_t)a.s) & 15) return forge_fail(-1, "tc gemv: weights and scales 16-byte aligned");
    const int T = (a.N + kTM - 1) / kTM;
    if (T > kMaxTiles) return forge_fail(-1, "tc gemv: N=%d too large", a.N);
    if (forge_gemv_tc_configure()) return -1;
    uint8_t* sc = static_cast<uint8_t*>(scratch);
    uint8_t* xt = sc + forge_gemv_scratch_header() + kPartialBytes;
    TcArgs t;
    t.xt = xt;
    t.ticket = reinterpret_cast<int*>(sc);
    t.partial = reinterpret_cast<float*>(sc + forge_gemv_scratch_header());
    t.npad = ((2 * a.batch + 15) / 16) * 16;
    t.wbox = a.K >= 256 ? 256 : 128;  // two groups a unit (one when K has a single group)
    const int64_t U = (int64_t)T * ((a.K / 128 + kGU - 1) / kGU);
    int grid = forge_sm_count();
    if (grid > kMaxGrid) grid = kMaxGrid;
    if (grid > U) grid = (int)U;
    int rc = a.pro == FORGE_PRO_RMSNORM ? launch_quant<FORGE_PRO_RMSNORM>(a, xt, stream, pdl)
                                        : launch_quant<FORGE_PRO_PLAIN>(a, xt, stream, pdl);
    if (rc) return rc;
    switch (a.epi) {
    case FORGE_EPI_STORE: return launch_tc<FORGE_EPI_STORE>(a, t, stream, grid);
    case FORGE_EPI_RESID: return launch_tc<FORGE_EPI_RESID>(a, t, stream, grid);
    case FORGE_EPI_QKV: return launch_tc<FORGE_EPI_QKV>(a, t, stream, grid);
    case FORGE_EPI_SWIGLU: return launch_tc<FORGE_EPI_SWIGLU>(a, t, stream, grid);
    default: return forge_fail(-1, "tc gemv: unknown epilogue %d", a.epi);
    }
}
