/* forge_clm.h — the .clm int4 checkpoint format (stdlib/flame/clm_ckpt.hexa:1-20)
 * read on the host, and converted to the group-128 int4 format of this
 * library.
 *
 * File: "CLM\x01", a u8 block count, then per block: u32-le Cout, u32-le
 * rest, ceil(Cout*rest/2) bytes of int4 levels (q + 8, element 2i in the low
 * nibble of byte i, element 2i+1 in the high one; clm_ckpt.hexa:47-61), Cout
 * fp32-le per-output-channel scales. A block is the weight [Cout][rest],
 * dequantised as q * scale[c] (load_block, clm_ckpt.hexa:63-80). */
#ifndef FORGE_CLM_H
#define FORGE_CLM_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ForgeClm ForgeClm;

typedef struct ForgeClmBlock {
    int64_t cout, rest;
    int64_t offset;          /* file offset of the block's Cout field */
} ForgeClmBlock;

/* Reads and checks the whole file (magic, block count, every block inside
 * the file, no trailing bytes). On failure *out is NULL and the error is in
 * forge_b200_last_error(). */
int  forge_clm_open(const char* path, ForgeClm** out);
void forge_clm_close(ForgeClm* c);
int  forge_clm_count(const ForgeClm* c);
int  forge_clm_block(const ForgeClm* c, int i, ForgeClmBlock* out);
/* Block i as int4 levels q in [-8, 7] ([Cout][rest], row-major) and its Cout
 * fp32 scales, exactly as stored (load_block). */
int  forge_clm_block_levels(const ForgeClm* c, int i, int8_t* q_out, float* scale_out);
/* Block i in the group-128 format: codes q + 7 as u8 [Cout][rest] and bf16
 * scales [Cout][rest / 128], each group taking its row's scale rounded to
 * bf16 (round to nearest even). The codes are exact; the scales are exact
 * when the row's fp32 scale is a bf16 value. Needs rest % 128 == 0 and every
 * level in [-7, 7] (what nn_int4_quant_fwd writes); codes and scales then
 * pack with forge_q4_pack_tiles. */
int  forge_clm_block_to_q4g128(const ForgeClm* c, int i, uint8_t* codes, uint16_t* scales);

#ifdef __cplusplus
}
#endif
#endif
