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
//   warp 8 (producer)  streams each unit's weight tiles in 8 KB pieces with
//                      cp.async.bulk into a 6-stage mbarrier ring; it never
//                      waits on the previous kernel, so under programmatic
//                      dependent launch the next layer's weights are already
//                      in flight while the previous kernel drains.
//   warps 0-7          build the bf16 B operand (hi/lo split of the fp32
//                      activations) in shared memory once per CTA, then for
//                      every piece dequantise int4 words straight into
//                      mma.sync A-fragment registers (lop3 + bf16 sub, no
//                      shared-memory round trip for weights beyond the TMA
//                      landing zone), accumulate one 128-group in fp32 and
//                      fold the group's bf16 scale in with one FMA per row.
//   The eight warps split each piece along K; a shared-memory reduction and
//   the fused epilogue finish every unit.
// Why mma.sync: at bs1 each SM must retire ~46 int4 weights per clock to keep
// up with HBM; FFMA dequant (~3-4 issue slots per weight) cannot, while the
// fragment path costs ~1.1 slots per weight and keeps A in registers (a
// tcgen05 A operand would have to round-trip bf16 through shared memory or
// TMEM, 8 bytes of on-chip traffic per HBM byte).
#include <cstdio>
#include "common.cuh"
#include "layout.cuh"
#include "forge_internal.h"

namespace {
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 6;
constexpr int kStageW = 8192;
constexpr int kStageS = 256;
constexpr int kStageBytes = kStageW + kStageS;
constexpr int kRedFloats = kConsumerWarps * 16 * 8;
constexpr int kFixedSmem = kStages * kStageBytes + 2 * kStages * 8 + kRedFloats * 4;
constexpr int kMaxSmem = 227 * 1024;

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t row) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - row);
}

template <int PRO>
__device__ __forceinline__ void stage_x(const ForgeGemvArgs& a, uint16_t* xs, float* red) {
    const int tid = threadIdx.x;  // consumer threads 0..255
    const int K = a.K, stride = K + 8;
    for (int b = 0; b < a.batch; ++b) {
        const float* xb = a.x + (size_t)b * a.x_stride;
        float inv = 1.0f;
        if (PRO == FORGE_PRO_RMSNORM) {
            float ss = 0.0f;
            for (int k = tid * 4; k < K; k += 256 * 4) {
                float4 v = *reinterpret_cast<const float4*>(xb + k);
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if ((tid & 31) == 0) red[tid >> 5] = ss;
            named_bar_sync(1, 256);
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) tot += red[w];
            inv = 1.0f / sqrtf(tot / (float)K + a.eps);
            named_bar_sync(1, 256);
        }
        for (int k = tid * 4; k < K; k += 256 * 4) {
            float4 v = *reinterpret_cast<const float4*>(xb + k);
            float e[4] = {v.x, v.y, v.z, v.w};
            if (PRO == FORGE_PRO_RMSNORM) {
                float4 gv = *reinterpret_cast<const float4*>(a.gain + k);
                e[0] = gv.x * (e[0] * inv); e[1] = gv.y * (e[1] * inv);
                e[2] = gv.z * (e[2] * inv); e[3] = gv.w * (e[3] * inv);
            }
            if (a.split) {
                uint16_t hi[4], lo[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) split_bf16(e[i], hi[i], lo[i]);
                uint2 h2 = make_uint2(hi[0] | ((uint32_t)hi[1] << 16), hi[2] | ((uint32_t)hi[3] << 16));
                uint2 l2 = make_uint2(lo[0] | ((uint32_t)lo[1] << 16), lo[2] | ((uint32_t)lo[3] << 16));
                *reinterpret_cast<uint2*>(xs + (size_t)(2 * b) * stride + k) = h2;
                *reinterpret_cast<uint2*>(xs + (size_t)(2 * b + 1) * stride + k) = l2;
            } else {
                uint16_t h[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) h[i] = f32_to_bf16_bits(e[i]);
                *reinterpret_cast<uint2*>(xs + (size_t)b * stride + k) =
                    make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
            }
        }
    }
}

template <int EPI>
__device__ __forceinline__ void epilogue(const ForgeGemvArgs& a, int u, int p, int b, float ylo, float yhi,
                                         unsigned long long& best) {
    const int row0 = u * 16;
    if (EPI == FORGE_EPI_STORE) {
        a.y[(size_t)b * a.y_stride + row0 + p] = ylo;
        a.y[(size_t)b * a.y_stride + row0 + p + 8] = yhi;
    } else if (EPI == FORGE_EPI_RESID) {
        a.y[(size_t)b * a.y_stride + row0 + p] += ylo;
        a.y[(size_t)b * a.y_stride + row0 + p + 8] += yhi;
    } else if (EPI == FORGE_EPI_LOGITS) {
        a.y[(size_t)b * a.y_stride + row0 + p] = ylo;
        a.y[(size_t)b * a.y_stride + row0 + p + 8] = yhi;
        if (row0 + p < a.nvalid) { unsigned long long k = argmax_key(ylo, row0 + p); best = k > best ? k : best; }
        if (row0 + p + 8 < a.nvalid) { unsigned long long k = argmax_key(yhi, row0 + p + 8); best = k > best ? k : best; }
    } else if (EPI == FORGE_EPI_SWIGLU) {
        // physical tile u = gate rows 8u..8u+7 (rows 0-7), up rows 8u..8u+7 (rows 8-15)
        float gte = ylo, upv = yhi;
        float sl = gte / (1.0f + expf(-gte));
        a.s_out[(size_t)b * a.F + 8 * u + p] = sl * upv;
    } else if (EPI == FORGE_EPI_QKV) {
        const int hd = a.hd, head = row0 / hd, i = (row0 % hd) >> 4;
        const int c = 8 * i + p, c2 = c + hd / 2;
        const int bg = a.b0 + b;
        const int P = a.pos[bg];
        if (P < 0 || P >= a.lmax) { atomicOr(a.err, FORGE_DEVERR_BAD_INDEX); return; }
        if (head < a.H + a.Hkv) {
            const float cs = a.rope_cos[(size_t)P * (hd / 2) + c];
            const float sn = a.rope_sin[(size_t)P * (hd / 2) + c];
            const float o1 = ylo * cs - yhi * sn;
            const float o2 = yhi * cs + ylo * sn;
            if (head < a.H) {
                float* q = a.q_out + (size_t)b * a.H * hd + (size_t)head * hd;
                q[c] = o1;
                q[c2] = o2;
            } else {
                uint16_t* k = a.kc + (((size_t)bg * a.Hkv + (head - a.H)) * a.lmax + P) * hd;
                k[c] = f32_to_bf16_bits(o1);
                k[c2] = f32_to_bf16_bits(o2);
            }
        } else {
            uint16_t* v = a.vc + (((size_t)bg * a.Hkv + (head - a.H - a.Hkv)) * a.lmax + P) * hd;
            v[c] = f32_to_bf16_bits(ylo);
            v[c2] = f32_to_bf16_bits(yhi);
        }
    }
}

template <int WK, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 1) k_gemv(const ForgeGemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    float* red = reinterpret_cast<float*>(empty + kStages);
    uint16_t* xs = reinterpret_cast<uint16_t*>(red + kRedFloats);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KT = a.K >> 4;
    constexpr int kItemKT = (WK == FORGE_W_Q4) ? 64 : 16;
    constexpr int kTileBytes = (WK == FORGE_W_Q4) ? 128 : 512;  // per 16x16 tile
    const int nitems = (KT + kItemKT - 1) / kItemKT;
    const int units = a.N >> 4;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == kConsumerWarps) {
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
                    const uint32_t wb = (uint32_t)nkt * kTileBytes;
                    uint32_t sb = 0;
                    if (WK == FORGE_W_Q4) sb = (uint32_t)(((nkt / 8) + 3) / 4) * 128u;
                    mbar_arrive_expect_tx(&full[s], wb + sb);
                    bulk_g2s(stages + s * kStageBytes, wbase + ((int64_t)u * KT + kt0) * kTileBytes, wb, &full[s]);
                    if (WK == FORGE_W_Q4)
                        bulk_g2s(stages + s * kStageBytes + kStageW,
                                 sbase + ((int64_t)u * G4 + kt0 / 32) * 128, sb, &full[s]);
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
    stage_x<PRO>(a, xs, red);
    named_bar_sync(1, 256);

    const int g = lane >> 2, t = lane & 3;
    const int ncols = a.split ? 2 * a.batch : a.batch;
    const int col = g < ncols ? g : ncols - 1;  // unused columns read a valid row
    const uint16_t* xcol = xs + (size_t)col * (a.K + 8) + 2 * t;
    unsigned long long best = 0ull;
    uint32_t it = 0;
    bool ok = true;

    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        float tot[4] = {0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < nitems; ++i) {
            const int s = it % kStages;
            const uint32_t ph = (it / kStages) & 1u;
            if (!mbar_wait(&full[s], ph, a.err)) { ok = false; break; }
            const int kt0 = i * kItemKT, nkt = min(kItemKT, KT - kt0);
            const uint8_t* st = stages + s * kStageBytes;
            if (WK == FORGE_W_Q4) {
                const int ktw = warp * 8;  // one 128-group per warp
                if (ktw < nkt) {
                    const uint4 c0 = *reinterpret_cast<const uint4*>(st + (ktw / 4) * 512 + lane * 16);
                    const uint4 c1 = *reinterpret_cast<const uint4*>(st + (ktw / 4 + 1) * 512 + lane * 16);
                    const uint32_t sc = *reinterpret_cast<const uint32_t*>(
                        st + kStageW + (((warp >> 2) * 64) + g * 8 + (warp & 3) * 2) * 2);
                    const uint16_t* xk = xcol + (size_t)(kt0 + ktw) * 16;
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};
                    const uint32_t wd[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        uint32_t af[4];
                        dequant_q4_word(wd[j], af);
                        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xk + j * 16);
                        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xk + j * 16 + 8);
                        mma_bf16_16816(acc, af, b0, b1, acc);
                    }
                    const float slo = bf16_lo_f32(sc), shi = bf16_hi_f32(sc);
                    tot[0] = fmaf(slo, acc[0], tot[0]);
                    tot[1] = fmaf(slo, acc[1], tot[1]);
                    tot[2] = fmaf(shi, acc[2], tot[2]);
                    tot[3] = fmaf(shi, acc[3], tot[3]);
                }
            } else {
                const int ktw = warp * 2;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    if (ktw + j < nkt) {
                        const uint4 av = *reinterpret_cast<const uint4*>(st + (ktw + j) * 512 + lane * 16);
                        const uint32_t af[4] = {av.x, av.y, av.z, av.w};
                        const uint16_t* xk = xcol + (size_t)(kt0 + ktw + j) * 16;
                        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xk);
                        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xk + 8);
                        mma_bf16_16816(tot, af, b0, b1, tot);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            ++it;
        }
        if (!ok) break;
        // cross-warp reduction: red[warp][row][col]
        float* rw = red + warp * 16 * 8;
        rw[g * 8 + 2 * t] = tot[0];
        rw[g * 8 + 2 * t + 1] = tot[1];
        rw[(g + 8) * 8 + 2 * t] = tot[2];
        rw[(g + 8) * 8 + 2 * t + 1] = tot[3];
        named_bar_sync(1, 256);
        const int tid = threadIdx.x;
        if (tid < 8 * a.batch) {
            const int p = tid & 7, b = tid >> 3;
            const int c = a.split ? 2 * b : b;
            float ylo = 0.f, yhi = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                ylo += red[(w * 16 + p) * 8 + c];
                yhi += red[(w * 16 + p + 8) * 8 + c];
                if (a.split) {
                    ylo += red[(w * 16 + p) * 8 + c + 1];
                    yhi += red[(w * 16 + p + 8) * 8 + c + 1];
                }
            }
            epilogue<EPI>(a, u, p, b, ylo, yhi, best);
        }
        named_bar_sync(1, 256);
    }

    if (EPI == FORGE_EPI_LOGITS && warp < 2) {
        // thread (p, b) = (tid & 7, tid >> 3): reduce over the 8 rows-pairs
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
    return e == cudaSuccess ? 0 : forge_fail(-1, "gemv: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
}
template <int WK, int PRO>
int configure_epi() {
    return configure_one<WK, PRO, FORGE_EPI_STORE>() | configure_one<WK, PRO, FORGE_EPI_RESID>() |
           configure_one<WK, PRO, FORGE_EPI_QKV>() | configure_one<WK, PRO, FORGE_EPI_SWIGLU>() |
           configure_one<WK, PRO, FORGE_EPI_LOGITS>();
}

template <int WK, int PRO, int EPI>
int launch_one(const ForgeGemvArgs& a, cudaStream_t stream, bool pdl, int smem) {
    auto kern = k_gemv<WK, PRO, EPI>;
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

int forge_gemv_launch(const ForgeGemvArgs& a0, cudaStream_t stream, bool pdl) {
    if (!a0.w || !a0.x || a0.N <= 0 || a0.K <= 0 || (a0.N % 16) || (a0.K % 16) || a0.batch <= 0)
        return forge_fail(-1, "gemv: bad shape N=%d K=%d batch=%d", a0.N, a0.K, a0.batch);
    if (a0.wkind == FORGE_W_Q4 && (!a0.s || (a0.K % 128)))
        return forge_fail(-1, "gemv: int4 weights need scales and K %% 128 == 0 (group 128)");
    if (a0.pro == FORGE_PRO_RMSNORM && !a0.gain) return forge_fail(-1, "gemv: RMSNorm prologue needs a gain");
    if ((a0.x_stride % 4) || (a0.K % 4)) return forge_fail(-1, "gemv: x rows must be 16-byte aligned");
    if (a0.epi == FORGE_EPI_SWIGLU && a0.N != 2 * a0.F) return forge_fail(-1, "gemv: SwiGLU needs N == 2F");
    if (a0.epi == FORGE_EPI_QKV && (a0.hd % 16 || a0.N != (a0.H + 2 * a0.Hkv) * a0.hd))
        return forge_fail(-1, "gemv: QKV epilogue shape mismatch");
    const int cols_per_seq = a0.split ? 2 : 1;
    const int xs_row = (a0.K + 8) * 2;
    int max_cols = (kMaxSmem - kFixedSmem) / xs_row;
    if (max_cols > 8) max_cols = 8;
    const int per_launch = max_cols / cols_per_seq;
    if (per_launch < 1) return forge_fail(-1, "gemv: K=%d too large for the staged activation", a0.K);
    for (int b0 = 0; b0 < a0.batch; b0 += per_launch) {
        ForgeGemvArgs a = a0;
        a.batch = a0.batch - b0 < per_launch ? a0.batch - b0 : per_launch;
        a.b0 = a0.b0 + b0;
        a.x = a0.x + (size_t)b0 * a0.x_stride;
        if (a.y) a.y = a0.y + (size_t)b0 * a0.y_stride;
        if (a.q_out) a.q_out = a0.q_out + (size_t)b0 * a0.H * a0.hd;
        if (a.s_out) a.s_out = a0.s_out + (size_t)b0 * a0.F;
        const int smem = kFixedSmem + a.batch * cols_per_seq * xs_row;
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
