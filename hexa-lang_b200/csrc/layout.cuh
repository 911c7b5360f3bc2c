// layout.cuh — HBM layouts of the packed decode weights.
//
// All decode GEMVs run on mma.sync.m16n8k16 fragments with the weight as the
// A operand (16 output rows x 16 input columns per tile). Weights are stored
// pre-permuted so that one 16-byte load per lane yields A-fragment registers
// directly, with no shared-memory transpose:
//
//  bf16 tiles  : [N/16][K/16][32 lanes][8 bf16]          512 B per 16x16 tile
//      lane l = 4g + t holds A[g][2t,2t+1] A[g+8][2t,2t+1] A[g][2t+8,2t+9]
//      A[g+8][2t+8,2t+9] (the mma A-fragment order).
//  q4 tiles    : [N/16][K/64][32 lanes][4 words]          512 B per 16x64 chunk
//      int4 codes feed the int8 tensor-core path (mma.m16n8k32 .u8 x .s8):
//      words 2j and 2j+1 of lane l = 4g + t hold the 16x32 k-tile j of the
//      chunk; byte i of word 2j+h holds, in its low nibble, the code of
//      (row g, k 16h + 4t + i) and in its high nibble (row g+8, same k), so
//      (w & 0x0F0F0F0F) and ((w >> 4) & 0x0F0F0F0F) are A-fragment registers
//      of unsigned codes (code = q + 7).
//  q4 scales   : [N/16][ceil(G/4)][8 g][4 groups][2 (row g, row g+8)] bf16
//      one 16-byte load per lane gives the scales of rows g and g+8 for four
//      consecutive 128-groups (groups past G are zero padding).
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define FORGE_HD __host__ __device__ __forceinline__
#else
#define FORGE_HD inline
#endif

// Byte offset of element (r, k) inside the bf16 tile layout.
FORGE_HD int64_t bf16_tile_offset(int64_t r, int64_t k, int64_t K) {
    int64_t rt = r >> 4, kt = k >> 4;
    int rr = (int)(r & 15), kk = (int)(k & 15);
    int g = rr & 7, up = rr >> 3, t = (kk & 7) >> 1, kh = kk >> 3, e = kk & 1;
    int lane = g * 4 + t, j = kh * 4 + up * 2 + e;
    return (((rt * (K >> 4) + kt) * 32 + lane) * 8 + j) * 2;
}

// (word byte offset, nibble index) of element (r, k) in the q4 tile layout.
FORGE_HD int64_t q4_tile_word_offset(int64_t r, int64_t k, int64_t K, int* nibble) {
    int64_t rt = r >> 4, c = k >> 6;
    int kt32 = (int)((k >> 5) & 1), kk = (int)(k & 31);
    int rr = (int)(r & 15), g = rr & 7, up = rr >> 3;
    int t = (kk & 15) >> 2, i = kk & 3, h16 = kk >> 4;
    int lane = g * 4 + t, w = kt32 * 2 + h16;
    *nibble = i * 2 + up;
    return ((rt * (K >> 6) + c) * 32 + lane) * 16 + w * 4;
}

FORGE_HD int64_t q4_groups4(int64_t K, int group) { return ((K / group) + 3) / 4; }

// Element offset (in bf16 units) of scale (r, grp) in the q4 scale layout.
FORGE_HD int64_t q4_scale_offset(int64_t r, int64_t grp, int64_t K, int group) {
    int64_t rt = r >> 4, G4 = q4_groups4(K, group);
    int rr = (int)(r & 15), g = rr & 7, up = rr >> 3;
    int64_t gb = grp >> 2;
    int gi = (int)(grp & 3);
    return ((rt * G4 + gb) * 8 + g) * 8 + gi * 2 + up;
}

// Logical source row of physical row p for the fused QKV matrix: inside each
// head, physical tile i holds logical rows 8i..8i+7 (rows 0..7 of the tile)
// and 8i+hd/2..8i+hd/2+7 (rows 8..15), so a RoPE pair (c, c+hd/2) sits in
// the same lane of the accumulator fragment.
FORGE_HD int64_t qkv_logical_row(int64_t p, int hd) {
    int64_t head = p / hd;
    int ph = (int)(p % hd);
    int i = ph >> 4, rr = ph & 15;
    int c = 8 * i + (rr & 7) + ((rr >> 3) ? hd / 2 : 0);
    return head * hd + c;
}
// Inverse: physical row of logical row c within the concatenated QKV matrix.
FORGE_HD int64_t qkv_physical_row(int64_t lr, int hd) {
    int64_t head = lr / hd;
    int c = (int)(lr % hd), half = hd / 2;
    int up = c >= half ? 1 : 0;
    int cc = c - up * half;
    return head * hd + (cc >> 3) * 16 + up * 8 + (cc & 7);
}
// Gate/up interleave: physical tile i = gate rows 8i..8i+7 then up rows
// 8i..8i+7; logical rows are [Wg ; Wu] (2F rows).
FORGE_HD int64_t gateup_logical_row(int64_t p, int64_t F) {
    int64_t i = p >> 4;
    int rr = (int)(p & 15);
    return (rr < 8) ? (8 * i + rr) : (F + 8 * i + rr - 8);
}
