/* forge_farr.h — device-array descriptors the dispatch entries take.
 *
 * HexaFarrBf16 and its six functions keep the layout and contract of the
 * reference's bf16 storage class (self/cuda/runtime_bf16_emit.hexa:153-210):
 * a host buffer, a device buffer, an element count, a location tag saying
 * which copy is authoritative, and an ownership flag. A descriptor made by the
 * reference runtime can therefore be passed to forge_tier_dispatch_v1/_v2 as
 * it is, and one made here can be handed back to the runtime.
 *
 * The rest is new in this library, with the same five-field shape where the
 * data is a plain array:
 *   HexaFarrF32 / HexaFarrI32  fp32 activations and int32 token ids or
 *                              positions (4-byte elements);
 *   HexaFarrW                  a weight matrix in the packed decode layout
 *                              (bf16 tiles, or int4 group-128 codes with bf16
 *                              scales), produced on the device from a logical
 *                              row-major [rows][K] bf16 array;
 *   HexaKvCache                a contiguous bf16 K/V cache
 *                              [layer][batch][kv_head][max_ctx][head_dim] with
 *                              one device int32 position per sequence.
 *
 * All functions return 0 / a pointer on success and -1 / NULL on failure,
 * with one line in forge_b200_last_error(). Transfers are synchronous
 * (cudaMemcpy), as in the reference.
 */
#ifndef FORGE_FARR_H
#define FORGE_FARR_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

enum {
    FARR_BF16_LOC_HOST   = 0,  /* host buffer authoritative   */
    FARR_BF16_LOC_DEVICE = 1,  /* device buffer authoritative */
    FARR_BF16_LOC_MIRROR = 2   /* host and device in sync     */
};

typedef struct HexaFarrBf16 {
    void*   h_buf;   /* host bf16 bit patterns, or NULL   */
    void*   d_buf;   /* device bf16 buffer, or NULL        */
    int64_t len;     /* element count                      */
    int     loc;     /* FARR_BF16_LOC_*                    */
    int     owns;    /* 1: free() releases both buffers    */
} HexaFarrBf16;
#define HEXA_FARR_BF16_ELEM_BYTES 2

HexaFarrBf16* hexa_farr_bf16_alloc(int64_t len);              /* zeroed host buffer */
void          hexa_farr_bf16_free(HexaFarrBf16* f);
int           hexa_farr_bf16_from_f64(const double* src, HexaFarrBf16* dst, int64_t n);  /* RNE */
int           hexa_farr_bf16_to_f64(const HexaFarrBf16* src, double* dst, int64_t n);
int           hexa_farr_bf16_to_device(HexaFarrBf16* f);  /* uploads only when loc == HOST */
int           hexa_farr_bf16_to_host(HexaFarrBf16* f);

/* fp32 / int32 arrays: same fields, 4-byte elements. */
typedef struct HexaFarrF32 {
    void* h_buf; void* d_buf; int64_t len; int loc; int owns;
} HexaFarrF32;
typedef struct HexaFarrI32 {
    void* h_buf; void* d_buf; int64_t len; int loc; int owns;
} HexaFarrI32;

HexaFarrF32* hexa_farr_f32_alloc(int64_t len);
void         hexa_farr_f32_free(HexaFarrF32* f);
int          hexa_farr_f32_to_device(HexaFarrF32* f);
int          hexa_farr_f32_to_host(HexaFarrF32* f);
HexaFarrI32* hexa_farr_i32_alloc(int64_t len);
void         hexa_farr_i32_free(HexaFarrI32* f);
int          hexa_farr_i32_to_device(HexaFarrI32* f);
int          hexa_farr_i32_to_host(HexaFarrI32* f);

/* Packed decode weights. */
#define HEXA_FARR_W_BF16     0
#define HEXA_FARR_W_Q4_G128  1
typedef struct HexaFarrW {
    void*   d_tiles;      /* packed tiles (device)                        */
    void*   d_scales;     /* int4: packed bf16 scales (device); else NULL  */
    int64_t rows, cols;   /* logical [rows][cols], cols = K                */
    int64_t tile_bytes, scale_bytes;
    int32_t kind;         /* HEXA_FARR_W_*                                 */
    int32_t group;        /* 128 for int4, 0 for bf16                      */
    int32_t packed;       /* 1 once hexa_farr_w_pack succeeded             */
    int32_t owns;
} HexaFarrW;

HexaFarrW* hexa_farr_w_alloc(int kind, int64_t rows, int64_t K);
/* int4 sibling named after the bf16 allocator; group must be 128. */
HexaFarrW* hexa_farr_q4_alloc(int64_t rows, int64_t K, int group);
/* Quantises (int4) and packs a logical row-major [rows][K] bf16 array. The
 * source is uploaded first when only its host copy is current. */
int  hexa_farr_w_pack(HexaFarrW* w, HexaFarrBf16* logical);
/* int4 only: the logical codes [rows][K/2] (code = q + 7, even k in the low
 * nibble, as quant_lib packs them) and scales [rows][K/128] (bf16 bits)
 * back on the host, for checks. */
int  hexa_farr_q4_unpack(const HexaFarrW* w, uint8_t* codes, uint16_t* scales);
void hexa_farr_w_free(HexaFarrW* w);

/* KV cache. */
typedef struct HexaKvCache {
    void*    d_k;         /* bf16 [n_layer][batch][n_kv_head][max_ctx][head_dim] */
    void*    d_v;
    int32_t* d_pos;       /* [batch] position of the next token of each sequence */
    int64_t  n_layer, batch, n_kv_head, max_ctx, head_dim;
    int      owns;
    int      reserved;
} HexaKvCache;

HexaKvCache* hexa_kv_alloc(int64_t n_layer, int64_t batch, int64_t n_kv_head, int64_t max_ctx,
                           int64_t head_dim);          /* zeroed, positions 0 */
void         hexa_kv_free(HexaKvCache* kv);
int          hexa_kv_set_positions(HexaKvCache* kv, const int32_t* pos, int64_t batch);
/* Writes positions [0, n_pos) of one (layer, sequence) from host
 * [n_kv_head][n_pos][head_dim] bf16 arrays. */
int          hexa_kv_write(HexaKvCache* kv, int64_t layer, int64_t seq, const uint16_t* k, const uint16_t* v,
                           int64_t n_pos);

#ifdef __cplusplus
}
#endif
#endif
