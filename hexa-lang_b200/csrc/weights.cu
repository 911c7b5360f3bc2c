// weights.cu — device-side weight preparation for the decode path:
// synthetic N(0, std) fill (bit-identical to the CPU oracle), group int4
// quantisation (quant_lib generalised to groups with bf16 scales), row
// permutations for the fused epilogues, and packing into the fragment tile
// layouts of layout.cuh.
#include "common.cuh"
#include "layout.cuh"
#include "forge_internal.h"

// ------------------------------------------------------------ synthetic fill
// N(0,1) from (seed, index): splitmix-style 64-bit hash -> two 32-bit
// uniforms -> Box–Muller, with ln and cos evaluated from their atanh/Taylor
// series using explicitly rounded IEEE ops (no FMA contraction), so the CPU
// oracle produces the same bits.
namespace {
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
#define DM(a, b) __dmul_rn((a), (b))
#define DA(a, b) __dadd_rn((a), (b))
#define DS(a, b) __dsub_rn((a), (b))
__device__ double ser_ln(double u) {
    uint64_t bits = (uint64_t)__double_as_longlong(u);
    int e = (int)((bits >> 52) & 0x7FF) - 1023;
    double m = __longlong_as_double((long long)((bits & 0x000FFFFFFFFFFFFFULL) | 0x3FF0000000000000ULL));
    if (m > 1.4142135623730951) { m = DM(m, 0.5); e = e + 1; }
    double s = __ddiv_rn(DS(m, 1.0), DA(m, 1.0));
    double s2 = DM(s, s);
    double p = 1.0 / 23.0;
    p = DA(DM(p, s2), 1.0 / 21.0);
    p = DA(DM(p, s2), 1.0 / 19.0);
    p = DA(DM(p, s2), 1.0 / 17.0);
    p = DA(DM(p, s2), 1.0 / 15.0);
    p = DA(DM(p, s2), 1.0 / 13.0);
    p = DA(DM(p, s2), 1.0 / 11.0);
    p = DA(DM(p, s2), 1.0 / 9.0);
    p = DA(DM(p, s2), 1.0 / 7.0);
    p = DA(DM(p, s2), 1.0 / 5.0);
    p = DA(DM(p, s2), 1.0 / 3.0);
    p = DA(DM(p, s2), 1.0);
    double lnm = DM(DM(2.0, s), p);
    return DA(DM((double)e, 0.6931471805599453), lnm);
}
__device__ double ser_cos(double x) {
    double x2 = DM(x, x);
    double p = 1.0 / 2432902008176640000.0;
    p = DS(DM(p, x2), 1.0 / 6402373705728000.0);
    p = DA(DM(p, x2), 1.0 / 20922789888000.0);
    p = DS(DM(p, x2), 1.0 / 87178291200.0);
    p = DA(DM(p, x2), 1.0 / 479001600.0);
    p = DS(DM(p, x2), 1.0 / 3628800.0);
    p = DA(DM(p, x2), 1.0 / 40320.0);
    p = DS(DM(p, x2), 1.0 / 720.0);
    p = DA(DM(p, x2), 1.0 / 24.0);
    p = DS(DM(p, x2), 1.0 / 2.0);
    p = DA(DM(p, x2), 1.0);
    return p;
}
__device__ double ser_sin(double x) {
    double x2 = DM(x, x);
    double p = 1.0 / 51090942171709440000.0;
    p = DS(DM(p, x2), 1.0 / 121645100408832000.0);
    p = DA(DM(p, x2), 1.0 / 355687428096000.0);
    p = DS(DM(p, x2), 1.0 / 1307674368000.0);
    p = DA(DM(p, x2), 1.0 / 6227020800.0);
    p = DS(DM(p, x2), 1.0 / 39916800.0);
    p = DA(DM(p, x2), 1.0 / 362880.0);
    p = DS(DM(p, x2), 1.0 / 5040.0);
    p = DA(DM(p, x2), 1.0 / 120.0);
    p = DS(DM(p, x2), 1.0 / 6.0);
    p = DA(DM(p, x2), 1.0);
    return DM(x, p);
}
__device__ double ser_cos2pi(double u) {
    const double two_pi = 6.283185307179586;
    double sign = 1.0;
    if (u > 0.5) u = DS(1.0, u);
    if (u > 0.25) { u = DS(0.5, u); sign = -1.0; }
    double r = (u > 0.125) ? ser_sin(DM(DS(0.25, u), two_pi)) : ser_cos(DM(u, two_pi));
    return DM(sign, r);
}
__device__ double normal_at(uint64_t seed, uint64_t idx) {
    uint64_t z = mix64(seed * 0x9E3779B97F4A7C15ULL + idx * 0xD1B54A32D192ED03ULL + 0x632BE59BD9B4E019ULL);
    uint32_t a = (uint32_t)(z >> 32), b = (uint32_t)z;
    double u1 = DM(DA((double)a, 1.0), 1.0 / 4294967296.0);
    double u2 = DM((double)b, 1.0 / 4294967296.0);
    double r = __dsqrt_rn(DM(-2.0, ser_ln(u1)));
    return DM(r, ser_cos2pi(u2));
}
#undef DM
#undef DA
#undef DS

__global__ void k_fill_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t offset, double sd) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float v = __double2float_rn(__dmul_rn(sd, normal_at(seed, offset + (uint64_t)i)));
        out[i] = f32_to_bf16_bits(v);
    }
}

// Block [nr][nc] of a row-major matrix with `stride` columns whose element
// (r, c) is stream position offset + r * stride + c: the same values the 1-D
// fill gives the whole matrix, so a tensor-parallel shard of a synthetic
// weight equals the slice of the single-GPU weight.
__global__ void k_fill_normal_bf16_2d(uint16_t* out, int64_t nr, int64_t nc, uint64_t seed, uint64_t offset,
                                      int64_t stride, double sd) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nr * nc;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / nc, c = i - r * nc;
        float v = __double2float_rn(__dmul_rn(sd, normal_at(seed, offset + (uint64_t)(r * stride + c))));
        out[i] = f32_to_bf16_bits(v);
    }
}

__global__ void k_fill_f32(float* out, int64_t n, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = v;
}

// --------------------------------------------------------- int4 quantise
// One warp per (row, group). quant_lib.hexa:33-74 + :103-129 with a bf16
// scale: s = bf16_rne(max|W_g| / 7.0f) (0 -> 1), q = clamp(trunc-half-away
// round((double)w / s), -7, 7), code = q + 7, even k in the low nibble.
__device__ __forceinline__ int q_code(double w, double s) {
    double x = w / s;
    double r = (x >= 0.0) ? (double)(long long)(x + 0.5) : 0.0 - (double)(long long)((0.0 - x) + 0.5);
    long long q = (long long)r;
    q = q > 7 ? 7 : (q < -7 ? -7 : q);
    return (int)q + 7;
}
__global__ void k_q4_quantize(const uint16_t* __restrict__ w, int64_t rows, int64_t K, int group,
                              uint8_t* __restrict__ codes, uint16_t* __restrict__ scales) {
    const int64_t G = K / group;
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t item = warp; item < rows * G; item += nwarps) {
        const int64_t r = item / G, g = item % G;
        const uint16_t* wg = w + r * K + g * group;
        float mx = 0.0f;
        for (int j = lane; j < group; j += 32) mx = fmaxf(mx, fabsf(bf16_bits_to_f32(wg[j])));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        uint16_t sb = f32_to_bf16_bits(mx / 7.0f);
        if (mx == 0.0f || (sb & 0x7FFF) == 0) sb = 0x3F80;
        if (lane == 0) scales[r * G + g] = sb;
        const double s = (double)bf16_bits_to_f32(sb);
        uint8_t* cp = codes + (r * K + g * group) / 2;
        for (int j = 2 * lane; j < group; j += 64) {
            int lo = q_code((double)bf16_bits_to_f32(wg[j]), s);
            int hi = q_code((double)bf16_bits_to_f32(wg[j + 1]), s);
            cp[j / 2] = (uint8_t)(lo | (hi << 4));
        }
    }
}

// ------------------------------------------------------- row permutations
__global__ void k_permute_rows(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst,
                               int64_t rows, int64_t K, int kind, int64_t param) {
    const int64_t n = rows * K / 8;  // 16-byte vectors (K % 8 == 0)
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t p = (i * 8) / K, k = (i * 8) % K;
        int64_t lr = p;
        if (kind == FORGE_PERM_QKV) lr = qkv_logical_row(p, (int)param);
        else if (kind == FORGE_PERM_GATEUP) lr = gateup_logical_row(p, param);
        *reinterpret_cast<uint4*>(dst + p * K + k) = *reinterpret_cast<const uint4*>(src + lr * K + k);
    }
}

// -------------------------------------------------------------- packing
// One thread per 16-byte output vector of the bf16 tile layout.
__global__ void k_pack_bf16_tiles(const uint16_t* __restrict__ w, int64_t N, int64_t K,
                                  uint8_t* __restrict__ out) {
    const int64_t nvec = N * K / 8;
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
         v += (int64_t)gridDim.x * blockDim.x) {
        int64_t tile = v >> 5;
        int lane = (int)(v & 31), g = lane >> 2, t = lane & 3;
        int64_t rt = tile / (K >> 4), kt = tile % (K >> 4);
        int64_t r0 = rt * 16 + g, k0 = kt * 16 + 2 * t;
        uint16_t e[8];
        e[0] = w[r0 * K + k0];           e[1] = w[r0 * K + k0 + 1];
        e[2] = w[(r0 + 8) * K + k0];     e[3] = w[(r0 + 8) * K + k0 + 1];
        e[4] = w[r0 * K + k0 + 8];       e[5] = w[r0 * K + k0 + 9];
        e[6] = w[(r0 + 8) * K + k0 + 8]; e[7] = w[(r0 + 8) * K + k0 + 9];
        uint4 o;
        o.x = e[0] | ((uint32_t)e[1] << 16);
        o.y = e[2] | ((uint32_t)e[3] << 16);
        o.z = e[4] | ((uint32_t)e[5] << 16);
        o.w = e[6] | ((uint32_t)e[7] << 16);
        reinterpret_cast<uint4*>(out)[v] = o;
    }
}

__device__ __forceinline__ uint32_t code_at(const uint8_t* codes, int64_t r, int64_t k, int64_t K) {
    uint8_t b = codes[(r * K + k) >> 1];
    return (k & 1) ? (b >> 4) : (b & 15u);
}
// One thread per packed 32-bit word of the q4 tile layout (layout.cuh).
__global__ void k_pack_q4_tiles(const uint8_t* __restrict__ codes, int64_t N, int64_t K,
                                uint32_t* __restrict__ out) {
    const int64_t nword = N * K / 8;
    for (int64_t wi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; wi < nword;
         wi += (int64_t)gridDim.x * blockDim.x) {
        const int w = (int)(wi & 3);
        const int lane = (int)((wi >> 2) & 31), g = lane >> 2, t = lane & 3;
        const int64_t chunk = wi >> 7;
        const int64_t rt = chunk / (K >> 6), c = chunk % (K >> 6);
        const int kt32 = w >> 1, h16 = w & 1;
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t k = c * 64 + kt32 * 32 + h16 * 16 + t * 4 + i;
            const uint32_t lo = code_at(codes, rt * 16 + g, k, K);
            const uint32_t hi = code_at(codes, rt * 16 + g + 8, k, K);
            word |= (lo | (hi << 4)) << (8 * i);
        }
        out[wi] = word;
    }
}
__global__ void k_pack_q4_scales(const uint16_t* __restrict__ scales, int64_t N, int64_t K, int group,
                                 uint16_t* __restrict__ out) {
    const int64_t G = K / group, G4 = q4_groups4(K, group);
    const int64_t n = (N / 16) * G4 * 64;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int up = (int)(i & 1), gi = (int)((i >> 1) & 3), g = (int)((i >> 3) & 7);
        int64_t gb = (i >> 6) % G4, rt = (i >> 6) / G4;
        int64_t grp = gb * 4 + gi, r = rt * 16 + g + 8 * up;
        out[i] = grp < G ? scales[r * G + grp] : (uint16_t)0;
    }
}
// Inverse of the two packings (used to prove the layouts round-trip).
__global__ void k_unpack_q4_tiles(const uint32_t* __restrict__ tiles, const uint16_t* __restrict__ stiles,
                                  int64_t N, int64_t K, int group, uint8_t* __restrict__ codes,
                                  uint16_t* __restrict__ scales) {
    const int64_t G = K / group;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N * K / 2;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = (2 * i) / K, k = (2 * i) % K;
        int n0, n1;
        int64_t o0 = q4_tile_word_offset(r, k, K, &n0), o1 = q4_tile_word_offset(r, k + 1, K, &n1);
        uint32_t c0 = (tiles[o0 / 4] >> (4 * n0)) & 15u, c1 = (tiles[o1 / 4] >> (4 * n1)) & 15u;
        codes[i] = (uint8_t)(c0 | (c1 << 4));
        if ((k % group) == 0) scales[r * G + k / group] = stiles[q4_scale_offset(r, k / group, K, group)];
    }
}
}  // namespace

static int grid_for(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    if (b > 148 * 64) b = 148 * 64;
    if (b < 1) b = 1;
    return (int)b;
}

extern "C" {
FORGE_API int forge_fill_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t offset,
                                     float std, void* stream) {
    if (!out || n < 0) return forge_fail(-1, "forge_fill_normal_bf16: bad args");
    if (n == 0) return 0;
    k_fill_normal_bf16<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(out, n, seed, offset, (double)std);
    return forge_check_launch("forge_fill_normal_bf16");
}
}  // extern "C"

int forge_fill_normal_bf16_2d(uint16_t* out, int64_t nr, int64_t nc, uint64_t seed, uint64_t offset, int64_t stride,
                              float std, cudaStream_t stream) {
    if (!out || nr < 0 || nc < 0 || stride < nc) return forge_fail(-1, "forge_fill_normal_bf16_2d: bad args");
    if (nr * nc == 0) return 0;
    k_fill_normal_bf16_2d<<<grid_for(nr * nc, 256), 256, 0, stream>>>(out, nr, nc, seed, offset, stride, (double)std);
    return forge_check_launch("forge_fill_normal_bf16_2d");
}

extern "C" {
FORGE_API int forge_fill_f32(float* out, int64_t n, float v, void* stream) {
    if (!out || n < 0) return forge_fail(-1, "forge_fill_f32: bad args");
    if (n == 0) return 0;
    k_fill_f32<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(out, n, v);
    return forge_check_launch("forge_fill_f32");
}
FORGE_API int forge_q4_quantize_bf16(const uint16_t* w, int64_t rows, int64_t K, int group,
                                     uint8_t* codes, uint16_t* scales, void* stream) {
    if (!w || !codes || !scales || rows <= 0 || K <= 0 || group <= 0 || (group % 64) || (K % group))
        return forge_fail(-1, "forge_q4_quantize_bf16: bad args (group must be a multiple of 64 dividing K)");
    int64_t items = rows * (K / group);
    k_q4_quantize<<<grid_for(items * 32, 256), 256, 0, (cudaStream_t)stream>>>(w, rows, K, group, codes, scales);
    return forge_check_launch("forge_q4_quantize_bf16");
}
FORGE_API int forge_permute_rows_bf16(const uint16_t* src, uint16_t* dst, int64_t rows, int64_t K,
                                      int kind, int64_t param, void* stream) {
    if (!src || !dst || src == dst || rows <= 0 || K <= 0 || (K % 8))
        return forge_fail(-1, "forge_permute_rows_bf16: bad args");
    if (kind == FORGE_PERM_QKV && (param <= 0 || (param % 16) || (rows % param)))
        return forge_fail(-1, "forge_permute_rows_bf16: QKV permutation needs head_dim % 16 == 0");
    if (kind == FORGE_PERM_GATEUP && (param <= 0 || (param % 8) || rows != 2 * param))
        return forge_fail(-1, "forge_permute_rows_bf16: gate/up permutation needs rows == 2F, F % 8 == 0");
    k_permute_rows<<<grid_for(rows * K / 8, 256), 256, 0, (cudaStream_t)stream>>>(src, dst, rows, K, kind, param);
    return forge_check_launch("forge_permute_rows_bf16");
}
FORGE_API int forge_bf16_pack_tiles(const uint16_t* w, int64_t N, int64_t K, void* tiles, void* stream) {
    if (!w || !tiles || N <= 0 || K <= 0 || (N % 16) || (K % 16))
        return forge_fail(-1, "forge_bf16_pack_tiles: N and K must be multiples of 16");
    k_pack_bf16_tiles<<<grid_for(N * K / 8, 256), 256, 0, (cudaStream_t)stream>>>(w, N, K, (uint8_t*)tiles);
    return forge_check_launch("forge_bf16_pack_tiles");
}
FORGE_API int forge_q4_pack_tiles(const uint8_t* codes, const uint16_t* scales, int64_t N, int64_t K,
                                  int group, void* tiles, void* scale_tiles, void* stream) {
    if (!codes || !scales || !tiles || !scale_tiles || N <= 0 || (N % 16) || K <= 0 || (K % 64) ||
        group <= 0 || (K % group) || (group % 64))
        return forge_fail(-1, "forge_q4_pack_tiles: bad shape");
    cudaStream_t s = (cudaStream_t)stream;
    k_pack_q4_tiles<<<grid_for(N * K / 8, 256), 256, 0, s>>>(codes, N, K, (uint32_t*)tiles);
    int64_t ns = (N / 16) * q4_groups4(K, group) * 64;
    k_pack_q4_scales<<<grid_for(ns, 256), 256, 0, s>>>(scales, N, K, group, (uint16_t*)scale_tiles);
    return forge_check_launch("forge_q4_pack_tiles");
}
FORGE_API int forge_q4_unpack_tiles(const void* tiles, const void* scale_tiles, int64_t N, int64_t K,
                                    int group, uint8_t* codes, uint16_t* scales, void* stream) {
    if (!tiles || !scale_tiles || !codes || !scales || N <= 0 || (N % 16) || K <= 0 || (K % 64) ||
        group <= 0 || (K % group))
        return forge_fail(-1, "forge_q4_unpack_tiles: bad shape");
    k_unpack_q4_tiles<<<grid_for(N * K / 2, 256), 256, 0, (cudaStream_t)stream>>>(
        (const uint32_t*)tiles, (const uint16_t*)scale_tiles, N, K, group, codes, scales);
    return forge_check_launch("forge_q4_unpack_tiles");
}
FORGE_API int64_t forge_q4_tile_bytes(int64_t N, int64_t K) { return N * K / 2; }
FORGE_API int64_t forge_q4_scale_tile_bytes(int64_t N, int64_t K, int group) {
    return (N / 16) * q4_groups4(K, group) * 64 * 2;
}
}  // extern "C"
