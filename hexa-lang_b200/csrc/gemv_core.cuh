// gemv_core.cuh — device pieces shared by the standalone decode GEMV kernel
// and the persistent decode-step kernel: activation staging in mma fragment
// order (with RMSNorm and the hi/lo bf16 split), the fused epilogues, and
// the int4 dequantisation.
#pragma once
#include "common.cuh"
#include "forge_internal.h"

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t row) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - row);
}

// Shared-memory B operand in mma fragment order: for every pair of k-tiles
// kp and column c, the 4 lanes t = 0..3 each own 16 bytes holding
// {b0, b1} of k-tile 2kp and {b0, b1} of k-tile 2kp+1, so one LDS.128 per
// lane feeds two mma steps. Columns are (sequence, hi|lo) in exact mode.
__device__ __forceinline__ int xf_index(int k, int col, int ncols) {
    const int kt = k >> 4, kk = k & 15;
    const int kp = kt >> 1, which = kt & 1, t = (kk & 7) >> 1, half = kk >> 3, e = kk & 1;
    return (((kp * ncols + col) * 4 + t) * 8) + which * 4 + half * 2 + e;
}

// Activation row loads. Activations are written by other CTAs earlier in
// the same persistent kernel, so they bypass L1 (ld.global.cg). EMBED reads
// the sequence's embedding row (bf16) instead of the residual stream.
template <int PRO>
__device__ __forceinline__ float4 load_x4(const ForgeGemvArgs& a, int b, const float* xb, int k) {
    if (PRO == FORGE_PRO_EMBED_RMSNORM) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(a.emb + (size_t)a.emb_tok[a.b0 + b] * a.K + k));
        return make_float4(bf16_lo_f32(v.x), bf16_hi_f32(v.x), bf16_lo_f32(v.y), bf16_hi_f32(v.y));
    }
    return __ldcg(reinterpret_cast<const float4*>(xb + k));
}

// bf16-weight prologue (consumer warps): optional RMSNorm, hi/lo bf16 split,
// fragment-order store.
template <int PRO, int NT>
__device__ __forceinline__ void stage_x(const ForgeGemvArgs& a, uint16_t* xf, float* red) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.K;
    const int ncols = a.split ? 2 * a.batch : a.batch;
    for (int b = 0; b < a.batch; ++b) {
        const float* xb = a.x + (size_t)b * a.x_stride;
        float inv = 1.0f;
        if (PRO != FORGE_PRO_PLAIN) {
            float ss = 0.0f;
            for (int k = tid * 4; k < K; k += NT * 4) {
                const float4 v = load_x4<PRO>(a, b, xb, k);
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) red[warp] = ss;
            named_bar_sync(1, NT);
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < NT / 32; ++w) tot += red[w];
            inv = 1.0f / sqrtf(tot / (float)K + a.eps);
            named_bar_sync(1, NT);
        }
        // 4 consecutive k per thread; a warp covers one 128-group per pass
        for (int k = tid * 4; k < K; k += NT * 4) {
            const float4 v = load_x4<PRO>(a, b, xb, k);
            float e[4] = {v.x, v.y, v.z, v.w};
            if (PRO != FORGE_PRO_PLAIN) {
                float4 gv = *reinterpret_cast<const float4*>(a.gain + k);
                e[0] = gv.x * (e[0] * inv); e[1] = gv.y * (e[1] * inv);
                e[2] = gv.z * (e[2] * inv); e[3] = gv.w * (e[3] * inv);
            }
            uint16_t hi[4], lo[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (a.split) split_bf16(e[i], hi[i], lo[i]);
                else { hi[i] = f32_to_bf16_bits(e[i]); lo[i] = 0; }
            }
            const int ch = a.split ? 2 * b : b;
            *reinterpret_cast<uint32_t*>(xf + xf_index(k, ch, ncols)) = hi[0] | ((uint32_t)hi[1] << 16);
            *reinterpret_cast<uint32_t*>(xf + xf_index(k + 2, ch, ncols)) = hi[2] | ((uint32_t)hi[3] << 16);
            if (a.split) {
                *reinterpret_cast<uint32_t*>(xf + xf_index(k, ch + 1, ncols)) = lo[0] | ((uint32_t)lo[1] << 16);
                *reinterpret_cast<uint32_t*>(xf + xf_index(k + 2, ch + 1, ncols)) = lo[2] | ((uint32_t)lo[3] << 16);
            }
        }
    }
}

// When K/16 is odd the last k-tile pair is half padding: zero it so the
// padded mma step multiplies by exact zeros.
template <int NT>
__device__ __forceinline__ void zero_x_pad(const ForgeGemvArgs& a, uint16_t* xf) {
    const int K = a.K;
    if ((K & 31) == 0) return;
    const int ncols = a.split ? 2 * a.batch : a.batch;
    for (int i = threadIdx.x; i < ncols * 16; i += NT) {
        const int col = i >> 4, k = K + (i & 15);
        xf[xf_index(k, col, ncols)] = 0;
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
        if (row0 + p < a.nvalid) {
            const unsigned long long k = argmax_key(ylo, a.row_off + row0 + p);
            best = k > best ? k : best;
        }
        if (row0 + p + 8 < a.nvalid) {
            const unsigned long long k = argmax_key(yhi, a.row_off + row0 + p + 8);
            best = k > best ? k : best;
        }
    } else if (EPI == FORGE_EPI_SWIGLU) {
        // physical tile u = gate rows 8u..8u+7 (rows 0-7), up rows 8u..8u+7 (rows 8-15)
        const float gte = ylo, upv = yhi;
        const float sl = gte / (1.0f + expf(-gte));
        a.s_out[(size_t)b * a.F + 8 * u + p] = sl * upv;
    } else if (EPI == FORGE_EPI_QKV) {
        const int hd = a.hd, head = row0 / hd, i = (row0 % hd) >> 4;
        const int c = 8 * i + p, c2 = c + hd / 2;
        const int bg = a.b0 + b;
        const int P = a.pos[bg];
        const int sq = a.seq_of ? a.seq_of[bg] : bg;  // cache sequence of this row
        if (P < 0 || P >= a.lmax || sq < 0) { atomicOr(a.err, FORGE_DEVERR_BAD_INDEX); return; }
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
                uint16_t* k = a.kc + (((size_t)sq * a.Hkv + (head - a.H)) * a.lmax + P) * hd;
                k[c] = f32_to_bf16_bits(o1);
                k[c2] = f32_to_bf16_bits(o2);
            }
        } else {
            uint16_t* v = a.vc + (((size_t)sq * a.Hkv + (head - a.H - a.Hkv)) * a.lmax + P) * hd;
            v[c] = f32_to_bf16_bits(ylo);
            v[c2] = f32_to_bf16_bits(yhi);
        }
    }
}

// A values of the int4 path are 135 + q (0x4300 | code), so a group's
// accumulator carries 135 * sum(B) extra; it is removed per group from the
// precomputed column sums. The raw A values are exact in bf16 and every
// product is exact in fp32.
__device__ __forceinline__ void dequant_q4_biased(uint32_t w, uint32_t (&a)[4]) {
    const uint32_t mask = 0x000F000Fu, magic = 0x43004300u;
    a[0] = lop3_and_or(w, mask, magic);
    a[1] = lop3_and_or(w >> 4, mask, magic);
    a[2] = lop3_and_or(w >> 8, mask, magic);
    a[3] = lop3_and_or(w >> 12, mask, magic);
}


// ------------------------------------------------------------------ int8
// Byte offset of activation (k, col) in the int8 fragment-order buffer: for
// each pair of 32-wide k-tiles and column, lane t owns 16 bytes = {b0, b1} of
// the even tile and {b0, b1} of the odd tile of mma.m16n8k32 (b0: k 4t..4t+3,
// b1: k 16+4t..16+4t+3).
__device__ __forceinline__ int xq_index(int k, int col, int ncols) {
    const int kt = k >> 5, kk = k & 31;
    const int kp = kt >> 1, which = kt & 1, t = (kk & 15) >> 2, half = kk >> 4, i = kk & 3;
    return (((kp * ncols + col) * 4 + t) * 16) + which * 8 + half * 4 + i;
}

// The int8 hi/lo arithmetic of one group (shared by the staging below and
// the kernels that hand staged activations to the next GEMV, so every path
// writes the same bytes): s = max|x| / 127 (1 for an all-zero group), then
// per element hi = rint(x / s), lo = rint((x - s hi) 256 / s) clamped to
// +-127. Rounding to the nearest integer (ties to even) adds 1.5 * 2^23: for
// |v| < 2^22 the sum's unit in the last place is 1, so the addition rounds v
// and the integer is the low mantissa bits — rintf and (int)rintf on the
// FP32 pipe instead of the slower conversion pipe. Products are rounded first
// (__fmul_rn) and x - s hi is one fused multiply-add.
__device__ __forceinline__ void quant_scales(float amax, float& sc, float& is, float& is256) {
    sc = amax > 0.f ? amax / 127.0f : 1.0f;
    is = amax > 0.f ? 127.0f / amax : 0.0f;
    is256 = 256.0f * is;
}
__device__ __forceinline__ void quant_elem(float x, float sc, float is, float is256, int& hi, int& lo) {
    // |x| <= amax, so x * is rounds into [-127, 127]: no clamp for hi
    const float th = __fadd_rn(__fmul_rn(x, is), 12582912.0f);
    const float hq = __fsub_rn(th, 12582912.0f);
    const float tl = __fadd_rn(__fmul_rn(__fmaf_rn(-sc, hq, x), is256), 12582912.0f);
    hi = __float_as_int(th) - 0x4B400000;
    lo = min(max(__float_as_int(tl) - 0x4B400000, -127), 127);
}
__device__ __forceinline__ uint32_t pack4_low_bytes(const int (&v)[4]) {  // byte j = v[j]
    return __byte_perm(__byte_perm(v[0], v[1], 0x0040), __byte_perm(v[2], v[3], 0x0040), 0x5410);
}

// int4-weight prologue: activations become int8 pairs per 128-group and
// sequence b: s = max|x| / 127, hi = rint(x / s), lo = rint((x - s*hi)*256/s)
// (both clamped to +-127), so x = s*(hi + lo/256) to ~2^-16 of the group
// maximum. Columns 2b / 2b+1 hold hi / lo. Per group it records s (sxf[g][b])
// and the column sums of hi and lo (ssum[g][2b], ssum[g][2b+1]) that remove
// the +7 code bias of the weights after the integer dot product.
template <int PRO, int NT, int MAXP = 3>
__device__ __forceinline__ void stage_x_q8(const ForgeGemvArgs& a, uint8_t* xq, float* sxf, int* ssum,
                                        float* red) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.K;
    const int ncols = 2 * a.batch;
    // Each thread owns 16 consecutive k (four float4), so 8 lanes cover one
    // 128-group and the group reductions take 3 shuffle steps instead of 5;
    // one pass covers PK = NT * 16 k. The reads of the first MAXP passes (and
    // the first pass of RMSNorm gains) are all issued before the first use,
    // so a row up to MAXP * PK long costs one memory round trip; later passes
    // read in the pass.
    constexpr int PK = NT * 16;
    const int passes = (K + PK - 1) / PK;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    const int kt = tid * 16;  // this thread's first k within a pass
    for (int b = 0; b < a.batch; ++b) {
        const float* xb = a.x + (size_t)b * a.x_stride;
        float4 xv[MAXP][4];
        float4 gv[4];
#pragma unroll
        for (int p = 0; p < MAXP; ++p)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int k = p * PK + kt + 4 * c;
                xv[p][c] = k < K ? load_x4<PRO>(a, b, xb, k) : z4;
            }
        if (PRO != FORGE_PRO_PLAIN) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int k = kt + 4 * c;
                gv[c] = k < K ? __ldg(reinterpret_cast<const float4*>(a.gain + k)) : z4;
            }
        }
        float inv = 1.0f;
        if (PRO != FORGE_PRO_PLAIN) {
            float ss = 0.0f;
#pragma unroll
            for (int p = 0; p < MAXP; ++p)
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    ss += xv[p][c].x * xv[p][c].x + xv[p][c].y * xv[p][c].y + xv[p][c].z * xv[p][c].z +
                          xv[p][c].w * xv[p][c].w;
            for (int p = MAXP; p < passes; ++p)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int k = p * PK + kt + 4 * c;
                    const float4 v = k < K ? load_x4<PRO>(a, b, xb, k) : z4;
                    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            // two halves of red alternate between sequences, so one barrier
            // per sequence suffices
            float* rb = red + (b & 1) * (NT / 32);
            if (lane == 0) rb[warp] = ss;
            named_bar_sync(1, NT);
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < NT / 32; ++w) tot += rb[w];
            inv = 1.0f / sqrtf(tot / (float)K + a.eps);
        }
        auto quantise = [&](int p, const float4 (&v)[4]) {
            const int k0 = p * PK + kt;
            // lanes past K hold zeros and take part in the shuffles; only
            // whole 8-lane groups are ever past K (K % 128 == 0)
            float e[16];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                e[4 * c] = v[c].x; e[4 * c + 1] = v[c].y; e[4 * c + 2] = v[c].z; e[4 * c + 3] = v[c].w;
            }
            if (PRO != FORGE_PRO_PLAIN) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 g4 = p == 0 ? gv[c]
                                             : (k0 + 4 * c < K ? __ldg(reinterpret_cast<const float4*>(a.gain + k0 + 4 * c))
                                                               : z4);
                    e[4 * c] = g4.x * (e[4 * c] * inv); e[4 * c + 1] = g4.y * (e[4 * c + 1] * inv);
                    e[4 * c + 2] = g4.z * (e[4 * c + 2] * inv); e[4 * c + 3] = g4.w * (e[4 * c + 3] * inv);
                }
            }
            float amax = 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(e[j]));
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            float sc, is, is256;
            quant_scales(amax, sc, is, is256);
            int shi = 0, slo = 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                int hi[4], lo[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) quant_elem(e[4 * c + j], sc, is, is256, hi[j], lo[j]);
                // low bytes of four ints into one word (byte j = element j)
                const uint32_t hw = pack4_low_bytes(hi);
                const uint32_t lw = pack4_low_bytes(lo);
                shi = __dp4a((int)hw, 0x01010101, shi);  // sum of the four signed bytes
                slo = __dp4a((int)lw, 0x01010101, slo);
                if (k0 < K) {
                    *reinterpret_cast<uint32_t*>(xq + xq_index(k0 + 4 * c, 2 * b, ncols)) = hw;
                    *reinterpret_cast<uint32_t*>(xq + xq_index(k0 + 4 * c, 2 * b + 1, ncols)) = lw;
                }
            }
            // both column sums in one reduction: hi * 2^16 + lo
            // (|sum| <= 128 * 127 < 2^15 for each)
            int packed = shi * 65536 + slo;
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) packed += __shfl_xor_sync(0xffffffffu, packed, o);
            if ((lane & 7) == 0 && k0 < K) {
                const int lo_sum = (int)(short)(packed & 0xFFFF);
                const int hi_sum = (packed - lo_sum) / 65536;
                const int g = k0 >> 7;
                sxf[g * 4 + b] = sc;
                ssum[g * 8 + 2 * b] = hi_sum;
                ssum[g * 8 + 2 * b + 1] = lo_sum;
            }
        };
#pragma unroll
        for (int p = 0; p < MAXP; ++p)
            if (p * PK < K) quantise(p, xv[p]);
        for (int p = MAXP; p < passes; ++p) {
            float4 v[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int k = p * PK + kt + 4 * c;
                v[c] = k < K ? load_x4<PRO>(a, b, xb, k) : z4;
            }
            quantise(p, v);
        }
    }
}

// The staged form of 128-group g of sequence b, from its 128 values held
// four per lane (lane l: elements 4l .. 4l+3), into a handoff block
// (ForgeGemvArgs::pq_in layout, G groups, ncols = 2 x batch). Every lane of
// the warp calls it; the bytes equal stage_x_q8's for the same values.
__device__ __forceinline__ void pq_group_warp(float4 v, int g, int b, int ncols, int G, uint8_t* blk) {
    float* sxf = reinterpret_cast<float*>(blk);
    int* ssum = reinterpret_cast<int*>(sxf + G * 4);
    uint8_t* xq = reinterpret_cast<uint8_t*>(ssum + G * 8);
    const int lane = threadIdx.x & 31;
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float sc, is, is256;
    quant_scales(amax, sc, is, is256);
    int hi[4], lo[4];
    quant_elem(v.x, sc, is, is256, hi[0], lo[0]);
    quant_elem(v.y, sc, is, is256, hi[1], lo[1]);
    quant_elem(v.z, sc, is, is256, hi[2], lo[2]);
    quant_elem(v.w, sc, is, is256, hi[3], lo[3]);
    const uint32_t hw = pack4_low_bytes(hi), lw = pack4_low_bytes(lo);
    const int k = g * 128 + 4 * lane;
    *reinterpret_cast<uint32_t*>(xq + xq_index(k, 2 * b, ncols)) = hw;
    *reinterpret_cast<uint32_t*>(xq + xq_index(k, 2 * b + 1, ncols)) = lw;
    int shi = __dp4a((int)hw, 0x01010101, 0), slo = __dp4a((int)lw, 0x01010101, 0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        shi += __shfl_xor_sync(0xffffffffu, shi, o);
        slo += __shfl_xor_sync(0xffffffffu, slo, o);
    }
    if (lane == 0) {
        sxf[g * 4 + b] = sc;
        ssum[g * 8 + 2 * b] = shi;
        ssum[g * 8 + 2 * b + 1] = slo;
    }
}

// One 128-group of int4 weights against the int8 activations: 2 chunks
// (4 k-tiles of 32) in two independent integer accumulators, then the code
// bias (7 * column sum), the hi/lo recombination and the two scales.
// Returns the contributions to rows g and g+8 for sequence t (lanes with
// t >= batch compute garbage that is never stored).
__device__ __forceinline__ void q4_group(const uint4 w0, const uint4 w1, const uint8_t* xq, int gg, int ncols,
                                         int col, int t, uint32_t scale_pair, const float* sxf, const int* ssum,
                                         int batch, float& y0, float& y1) {
    int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
    const uint4* xa = reinterpret_cast<const uint4*>(xq) + (size_t)((2 * gg) * ncols + col) * 4 + t;
    const uint4 b0 = xa[0];
    const uint4 b1 = xa[(size_t)ncols * 4];
    uint32_t af[4];
    dequant_q4_u8(w0.x, w0.y, af);
    mma_u8s8_16832(c0, af, b0.x, b0.y);
    dequant_q4_u8(w0.z, w0.w, af);
    mma_u8s8_16832(c1, af, b0.z, b0.w);
    dequant_q4_u8(w1.x, w1.y, af);
    mma_u8s8_16832(c0, af, b1.x, b1.y);
    dequant_q4_u8(w1.z, w1.w, af);
    mma_u8s8_16832(c1, af, b1.z, b1.w);
    const int tb = t < batch ? t : batch - 1;
    const int shi = ssum[gg * 8 + 2 * tb], slo = ssum[gg * 8 + 2 * tb + 1];
    const float sx = sxf[gg * 4 + tb];
    // int -> float of the group sums (|n| <= 128 * 14 * 127 < 2^22): the
    // integer added to the bits of 1.5 * 2^23, minus 1.5 * 2^23 — exact, on
    // the integer and FP32 pipes instead of the conversion pipe
    auto i2f = [](int n) { return __fsub_rn(__int_as_float(n + 0x4B400000), 12582912.0f); };
    const float v0 = i2f(c0[0] + c1[0] - 7 * shi) + i2f(c0[1] + c1[1] - 7 * slo) * (1.0f / 256.0f);
    const float v1 = i2f(c0[2] + c1[2] - 7 * shi) + i2f(c0[3] + c1[3] - 7 * slo) * (1.0f / 256.0f);
    y0 = bf16_lo_f32(scale_pair) * sx * v0;
    y1 = bf16_hi_f32(scale_pair) * sx * v1;
}
