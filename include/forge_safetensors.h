/* forge_safetensors.h — read-only memory-mapped safetensors files and the
 * model loader built on them (host code; no GPU needed except for
 * forge_b200_load_safetensors).
 *
 * Replaces the hexa runtime's RFC 025 builtins, declared at
 * self/runtime.h:1068-1082 and lowered by self/codegen.hexa:7181-7186:
 *   hexa_safetensors_mmap_open / _close        -> forge_st_open / forge_st_close
 *   hexa_safetensors_mmap_header               -> forge_st_header
 *   hexa_safetensors_mmap_data_offset / _size  -> forge_st_data_offset / forge_st_size
 *   hexa_safetensors_mmap_read_f32_farr        -> forge_st_read_f32
 *   hexa_safetensors_mmap_read_bf16_to_f32_farr-> forge_st_read_bf16_to_f32
 *   hexa_safetensors_mmap_read_bytes           -> forge_st_read_bytes
 * and the tensor views of self/alloc/safetensors_mmap.hexa:21-33
 * (safetensors_mmap_count / _name_at / _tensor / _total_bytes,
 * safetensors_view_u8) -> forge_st_count / forge_st_tensor_at /
 * forge_st_find / forge_st_total_bytes / forge_st_view_u8.
 *
 * File format: u64 little-endian header length H, H bytes of JSON
 * {"name": {"dtype": "BF16", "shape": [..], "data_offsets": [begin, end]},
 *  "__metadata__": {"key": "value", ..}}, then the data region; offsets are
 * relative to the data region (byte 8 + H of the file). Read offsets taken by
 * forge_st_read_* are absolute file offsets, as in the hexa builtins. */
#ifndef FORGE_SAFETENSORS_H
#define FORGE_SAFETENSORS_H
#include <stdint.h>
#include "forge_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define FORGE_ST_BOOL     0
#define FORGE_ST_U8       1
#define FORGE_ST_I8       2
#define FORGE_ST_I16      3
#define FORGE_ST_U16      4
#define FORGE_ST_F16      5
#define FORGE_ST_BF16     6
#define FORGE_ST_I32      7
#define FORGE_ST_U32      8
#define FORGE_ST_F32      9
#define FORGE_ST_F64      10
#define FORGE_ST_I64      11
#define FORGE_ST_U64      12
#define FORGE_ST_F8_E4M3  13
#define FORGE_ST_F8_E5M2  14

#define FORGE_ST_MAX_DIMS 8
#define FORGE_ST_NOT_FOUND (-6)

typedef struct ForgeSafetensors ForgeSafetensors;

typedef struct ForgeStTensor {
    const char* name;        /* owned by the handle                          */
    int32_t dtype;           /* FORGE_ST_*                                   */
    int32_t ndim;
    int64_t shape[FORGE_ST_MAX_DIMS];
    int64_t offset;          /* absolute file offset of the first byte       */
    int64_t nbytes;
    const void* data;        /* into the read-only mapping (valid until close) */
} ForgeStTensor;

/* Maps and validates the file (header JSON, dtypes, shapes against byte
 * counts, offsets inside the file). On failure *out is NULL and the error is
 * in forge_b200_last_error(). */
int         forge_st_open(const char* path, ForgeSafetensors** out);
int         forge_st_close(ForgeSafetensors* st);   /* NULL: no-op, 0 */
const char* forge_st_header(const ForgeSafetensors* st, int64_t* len); /* raw JSON, not NUL-terminated */
int64_t     forge_st_data_offset(const ForgeSafetensors* st);  /* 8 + header length */
int64_t     forge_st_size(const ForgeSafetensors* st);         /* file bytes */
int         forge_st_count(const ForgeSafetensors* st);        /* tensors, in header order */
int64_t     forge_st_total_bytes(const ForgeSafetensors* st);  /* sum of tensor byte counts */
int         forge_st_tensor_at(const ForgeSafetensors* st, int i, ForgeStTensor* out);
int         forge_st_find(const ForgeSafetensors* st, const char* name, ForgeStTensor* out);
/* __metadata__ value for key, NULL when absent (NUL-terminated, owned). */
const char* forge_st_metadata(const ForgeSafetensors* st, const char* key);
/* Byte i of a tensor view; 0 outside [0, nbytes) (safetensors_view_u8). */
int         forge_st_view_u8(const ForgeStTensor* v, int64_t i);
/* n elements from absolute file offset off; returns n, or a negative code
 * when [off, off + bytes) leaves the file. */
int64_t     forge_st_read_bytes(const ForgeSafetensors* st, int64_t off, int64_t n, void* out);
int64_t     forge_st_read_f32(const ForgeSafetensors* st, int64_t off, int64_t n, float* out);
int64_t     forge_st_read_bf16_to_f32(const ForgeSafetensors* st, int64_t off, int64_t n, float* out);
/* Converts a tensor to bf16 bit patterns (BF16 copied; F32 / F16 / F64
 * rounded to nearest even) or to fp32 (BF16 / F16 / F32 exactly, F64
 * rounded); n must equal the tensor's element count. */
int         forge_st_tensor_to_bf16(const ForgeStTensor* v, uint16_t* out, int64_t n);
int         forge_st_tensor_to_f32(const ForgeStTensor* v, float* out, int64_t n);

/* Loads a Llama-layout checkpoint (one or more .safetensors shards) into a
 * model handle through forge_b200_load_layer / forge_b200_load_embedding:
 *   model.embed_tokens.weight [V][d], model.norm.weight [d],
 *   lm_head.weight [V][d] (ignored when the model ties its head),
 *   model.layers.{l}.input_layernorm.weight, .post_attention_layernorm.weight [d],
 *   model.layers.{l}.self_attn.{q,k,v,o}_proj.weight, .mlp.{gate,up,down}_proj.weight
 * in W[out][in] orientation; shapes are checked against the handle's
 * description. Under tensor parallelism every rank loads the same files and
 * keeps its shard. Synchronous. */
int forge_b200_load_safetensors(ForgeB200* h, int n_files, const char* const* paths);
/* The checks forge_b200_load_safetensors makes before it uploads anything
 * (every tensor present once, with the shape the description gives and a
 * floating-point dtype), without a model handle or a GPU. 0 when the
 * checkpoint loads; otherwise the first problem in forge_b200_last_error(). */
int forge_safetensors_check_llama(const ForgeModelDesc* desc, int n_files, const char* const* paths);

#ifdef __cplusplus
}
#endif
#endif
