/* forge_b200.h — B200 (sm_100a) decode engine behind forge's C ABI.
 *
 * This is the _v2 surface that sits beside the unchanged forge_tier_v1.h
 * (reference self/forge/forge_tier_v1.h:24-130, which says any ABI change
 * needs a _v2 bump, :5-7). It adds:
 *   1. the whole-model decode engine (ForgeB200 handle) that flame's decode
 *      loop drives in place of nn_decoder_fwd + nn_decoder_predict
 *      (stdlib/flame/decoder_lib.hexa:93-208, 485-500), with a KV cache;
 *   2. per-op kernel entries on caller-owned device memory (the B200
 *      replacements of _hx_cuda_farr_packed_gemv_offset_gpu,
 *      self/cuda/runtime_cuda_emit.hexa:1858-1967, and of the attention
 *      kernel _hx_cuda_kern_attn_dt_fwd, :2819-2895);
 *   3. the int4 group-128 weight format (a generalisation of
 *      stdlib/flame/quant_lib.hexa:41-141) and its packing;
 *   4. the bf16 / int4 device-array descriptors (HexaFarrBf16 mirrors
 *      self/cuda/runtime_bf16_emit.hexa:164-210).
 * Every entry returns 0 on success or a negative FORGE_* code and leaves one
 * line in forge_b200_last_error() (printed once to stderr). Streams are
 * passed as `void*` (a cudaStream_t); no entry synchronises the device
 * unless it says so. There is no CPU fallback: without a usable sm_100
 * device every compute entry fails.
 */
#ifndef FORGE_B200_H
#define FORGE_B200_H
#include <stdint.h>
#include "forge_tier_v1.h"
#include "forge_farr.h"
#ifdef __cplusplus
extern "C" {
#endif

#define FORGE_API_VERSION_V2_ENCODED ((uint32_t)0x00020000u)
uint32_t forge_api_version_v2(void);

/* ---- v2 kernel families (dispatched by forge_tier_dispatch_v2) --------- */
#define FORGE_KERNEL_GEMV_W4A16_G128  16
#define FORGE_KERNEL_GEMV_BF16        17
#define FORGE_KERNEL_QKV_ROPE_FUSED   18
#define FORGE_KERNEL_FLASH_DECODE     19
#define FORGE_KERNEL_SWIGLU_FUSED     20
#define FORGE_KERNEL_LMHEAD_ARGMAX    21
#define FORGE_KERNEL_FLASH_PREFILL    22
#define FORGE_KERNEL_DECODE_STEP      23
#define FORGE_PREC_W4A16_G128_BF16    3

/* Dispatch of the v2 families; same arguments and return codes as
 * forge_tier_dispatch_v1 (v1 families are forwarded to it unchanged).
 * Slots hold descriptor pointers cast through intptr_t, or plain integers
 * where marked. Device work runs on the legacy default stream (handle
 * families: on the handle's stream) and is not waited for, except
 * DECODE_STEP, which is synchronous.
 *   GEMV_W4A16_G128 (precision FORGE_PREC_W4A16_G128_BF16), GEMV_BF16
 *   (FORGE_PREC_PURE_BF16): in = [HexaFarrW* W, HexaFarrF32* X [M][K]],
 *     out = [HexaFarrF32* Y [M][N]]; shape N = rows of W, K, M = sequences.
 *   FLASH_DECODE (PURE_BF16): in = [HexaFarrF32* Q [M][N*hd],
 *     HexaKvCache*, layer (integer)], out = [HexaFarrF32* O [M][N*hd]];
 *     shape M = sequences, N = query heads; attends to positions 0..pos.
 *   QKV_ROPE_FUSED, SWIGLU_FUSED, LMHEAD_ARGMAX, DECODE_STEP (either
 *   precision; the handle's weights decide): in[0] = ForgeB200*, shape
 *   batch (or M) = sequences.
 *     QKV_ROPE_FUSED: in = [h, layer, HexaFarrF32* X [B][d]],
 *       out = [HexaFarrF32* Q [B][H*hd]]; K/V appended at the positions.
 *     SWIGLU_FUSED: in = [h, layer, X [B][d]], out = [Y [B][d]],
 *       Y = X + Wd (silu(Wg n) * Wu n), n = RMSNorm(X).
 *     LMHEAD_ARGMAX: in = [h, X [B][d]], out = [HexaFarrI32* TOK [B],
 *       optional HexaFarrF32* LOGITS [B][V]].
 *     DECODE_STEP: in = [h, HexaFarrI32* TOK [B] (host copy)],
 *       out = [HexaFarrI32* NEXT [B], optional HexaFarrF32* LOGITS] (host).
 *   FLASH_PREFILL (PURE_BF16): in = [HexaFarrBf16* Q, K, V [M][N][S][K]],
 *     out = [HexaFarrBf16* O [M][N][S][K]]; shape M = batch, N = heads,
 *     K = head_dim (128), batch = S; causal. */
int forge_tier_dispatch_v2(int kernel_family, const ForgeShapeInfo* shape, int regime_hint,
                           int precision_policy, int det_mode, const ForgeArgs* in, const ForgeArgs* out);

/* Reads and clears the error word of the per-op kernels (synchronises). */
int forge_ops_check(void);

/* ---- model ------------------------------------------------------------- */
#define FORGE_WEIGHT_BF16     0
#define FORGE_WEIGHT_Q4_G128  1

typedef struct ForgeModelDesc {
    int32_t n_layer, d_model, n_head, n_kv_head, head_dim, ffn, vocab;
    float   rms_eps, rope_theta;  /* rope_theta <= 0: no rotary embedding */
    int32_t weight_kind;   /* FORGE_WEIGHT_*                                      */
    int32_t tied_head;     /* 1: LM head = embedding table (flame ties them)      */
    int32_t max_batch;     /* sequences decoded together                          */
    int32_t max_ctx;       /* KV-cache positions per sequence                     */
    int32_t tp_rank, tp_size; /* tensor parallel slot (1 = single GPU)           */
    int32_t act_mode;      /* 0 auto, 1 exact (hi/lo bf16 split of fp32 activations),
                              2 bf16 activations                                  */
    int32_t reserved[5];
} ForgeModelDesc;

/* Host weights of one block in flame's orientation (W[out][in], row-major,
 * decoder_block_lib.hexa:49-72): bf16 bit patterns; gains fp32. */
typedef struct ForgeLayerWeights {
    const uint16_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const float *g1, *g2;
} ForgeLayerWeights;

typedef struct ForgeB200 ForgeB200;

int         forge_b200_create(const ForgeModelDesc* desc, int device, ForgeB200** out);
/* The description the handle was created with. */
int         forge_b200_get_desc(const ForgeB200* h, ForgeModelDesc* out);
/* Tensor-parallel handle: rank desc->tp_rank of desc->tp_size, one process
 * (or thread) per GPU. Every rank passes the same 128-byte NCCL unique id
 * (made once by forge_b200_tp_unique_id and shared out of band) and calls
 * this at the same time (it blocks until all ranks joined). Heads are split
 * evenly (n_head and n_kv_head divisible by tp_size), the FFN in whole
 * 128-row groups (int4) or 16-row tiles (bf16) with the first ranks taking one
 * more when they do not divide, the vocabulary in equal 16-row slices. Each
 * decode step then runs one NCCL fp32 all-reduce after the O and after the
 * down projection and one max all-reduce of the argmax keys; tokens, positions
 * and the residual stream are identical on every rank. Entries that return
 * logits gather them from all ranks: call them on all ranks alike. NCCL is
 * opened at run time (libnccl.so.2, or the path in FORGE_NCCL_LIB). */
int         forge_b200_create_tp(const ForgeModelDesc* desc, int device, const void* nccl_unique_id,
                                 ForgeB200** out);
int         forge_b200_tp_unique_id(void* out128);
/* Shard of n items in units of gran for rank of size (the split the TP
 * handle uses for the FFN): first rank offset and length. */
int         forge_tp_split(int64_t n, int64_t gran, int rank, int size, int64_t* off, int64_t* len);
void        forge_b200_destroy(ForgeB200* h);
const char* forge_b200_last_error(void);
void*       forge_b200_stream(ForgeB200* h);

/* Weights: upload logical bf16 (quantised on the device when the model is
 * int4), or generate N(0, std) synthetic weights on the device with gains
 * 1.0 (tensor t of the model uses stream (seed, t << 40)). */
int forge_b200_load_layer(ForgeB200* h, int layer, const ForgeLayerWeights* w);
int forge_b200_load_embedding(ForgeB200* h, const uint16_t* emb, const float* final_gain,
                              const uint16_t* head /* NULL when tied */);
int forge_b200_init_synthetic(ForgeB200* h, uint64_t seed, float std);
/* The same, std as a double (FFIs that pass floats as doubles: hexa's extern fn). */
int forge_b200_init_synthetic_d(ForgeB200* h, uint64_t seed, double std);

/* KV cache / positions. fill_kv_synthetic writes N(0, std) K/V for positions
 * [0, ctx_len) of every sequence and sets every position to ctx_len. */
int forge_b200_reset(ForgeB200* h);
int forge_b200_fill_kv_synthetic(ForgeB200* h, uint64_t seed, int ctx_len, float std);
int forge_b200_set_positions(ForgeB200* h, const int32_t* pos, int batch);
int forge_b200_get_kv(ForgeB200* h, int layer, int seq, uint16_t* k_out, uint16_t* v_out);
/* Writes positions [0, n_pos) of one sequence's K/V cache from host
 * [n_kv_head][n_pos][head_dim] bf16 arrays (synchronous). */
int forge_b200_set_kv(ForgeB200* h, int layer, int seq, const uint16_t* k, const uint16_t* v, int n_pos);
/* Reads positions [0, n_pos) of one sequence's K/V cache into host
 * [n_kv_head][n_pos][head_dim] bf16 arrays (synchronous): with set_kv, the
 * copy that moves a sequence's cache out of HBM and back (KV swap). */
int forge_b200_get_kv_rows(ForgeB200* h, int layer, int seq, uint16_t* k, uint16_t* v, int n_pos);

/* One decode step from host buffers (H2D tokens, graph launch, D2H next
 * tokens and optional logits [batch][vocab]); synchronous. */
int forge_b200_decode_step(ForgeB200* h, int batch, const int32_t* tokens, int32_t* next_tokens,
                           float* logits);
/* One decode step whose next tokens are drawn from the step's logits by the
 * sampler of self/ml/gpu_sampler.hexa:89-277 (GpuSamplerConfig: temperature
 * <= 0 is argmax; top_k 0 and top_p >= 1 switch those filters off), on the
 * device; rng_state [batch] holds each sequence's 64-bit RNG state
 * (gpu_sampler_set_seed) and is advanced. Single-GPU handles; synchronous. */
int forge_b200_decode_step_sampled(ForgeB200* h, int batch, const int32_t* tokens, int32_t* next_tokens,
                                   double temperature, int top_k, double top_p, int64_t* rng_state);
/* Packed-argument forms for callers whose FFI passes at most six integer
 * arguments and writes 8-byte fields (the hexa interpreter's 6-argument
 * host call; the pattern of hxflash_attn_fwd_packed, self/ml/hxflash.hexa:40-62):
 * one pointer to a block of 8-byte little-endian fields, int64 unless marked
 * f64, at these byte offsets.
 *   create:  0 n_layer  8 d_model  16 n_head  24 n_kv_head  32 head_dim
 *            40 ffn  48 vocab  56 rms_eps (f64)  64 rope_theta (f64)
 *            72 weight_kind  80 tied_head  88 max_batch  96 max_ctx
 *            104 act_mode  112 device  120 address of the ForgeB200* result
 *            (128 bytes; tensor parallel stays forge_b200_create_tp)
 *   sampled step: 0 handle  8 batch  16 tokens  24 next_tokens
 *            32 temperature (f64)  40 top_k  48 top_p (f64)  56 rng_state
 *            (64 bytes) */
int forge_b200_desc_from_packed(const void* args, ForgeModelDesc* out);
int forge_b200_create_packed(const void* args);
int forge_b200_decode_step_sampled_packed(const void* args);
/* n_steps device-resident greedy steps (each feeds its argmax to the next);
 * asynchronous on the handle's stream. */
int forge_b200_decode_device(ForgeB200* h, int batch, int n_steps);
/* Prompt prefill: every position of prompt [batch][n_prompt] through the
 * model in one pass (decoder_block_lib.hexa:217-508, all positions; the
 * batched GEMVs stream each weight tile once per 32 prompt rows, causal
 * attention of every row over its own sequence's cache), K/V of positions
 * 0..n_prompt-1 written to the cache, then the final norm, LM head and
 * argmax of the last position: next_tok [batch] (may be NULL) and logits
 * [batch][vocab] (may be NULL). The handle is reset first and left at
 * position n_prompt, ready for forge_b200_decode_step / _decode_device.
 * exact: 1 keeps hi/lo activations for bf16 weights at any row count, 0
 * follows the model's act_mode (bf16 activations above 4 rows). Synchronous.
 * Under tensor parallelism every rank calls it with the same prompt. */
int forge_b200_prefill(ForgeB200* h, int batch, const int32_t* prompt, int n_prompt, int exact,
                       int32_t* next_tok, float* logits);
/* One pass over n_rows ragged rows, the iteration of a continuous-batching
 * scheduler (prompt chunks of new requests and one row per decoding request
 * in the same pass): row r is token tok[r] of sequence slot seq[r] at
 * position pos[r]; its K/V go to that slot's cache at pos[r] and it attends
 * over positions 0..pos[r] of the slot (earlier positions cached by earlier
 * passes or by rows of this one). Then the final norm, LM head and argmax of
 * the n_out (1..max_batch) rows out_rows[]: next_tok [n_out] and logits
 * [n_out][vocab] (either may be NULL). Two rows may not write the same
 * (slot, position). exact as for forge_b200_prefill. The handle's own
 * positions and step history are untouched. Synchronous. */
int forge_b200_forward_rows(ForgeB200* h, int n_rows, const int32_t* tok, const int32_t* pos, const int32_t* seq,
                            int n_out, const int32_t* out_rows, int exact, int32_t* next_tok, float* logits);
/* Greedy generation: prompt [batch][n_prompt] prefilled in one pass (hi/lo
 * activations unless act_mode is 2), then n_gen argmax tokens into out
 * [batch][n_gen] (the first from the prefill, the rest one decode step
 * each); synchronous. Replaces flame's decode loop (decoder_lib.hexa:93-208,
 * 485-500: full recompute per token). */
int forge_b200_generate(ForgeB200* h, int batch, const int32_t* prompt, int n_prompt, int n_gen,
                        int32_t* out);
/* Waits for the handle's stream; fails if a kernel raised its error word. */
int forge_b200_sync(ForgeB200* h);
/* Algorithmic HBM bytes of one decode step (weights + scales + head + KV
 * read/write) at the given batch and context length. */
int64_t forge_b200_step_bytes(ForgeB200* h, int batch, int ctx_len);
/* Timeline of the last fused step when FORGE_STEP_TRACE is set at handle
 * creation: [sm][phase][4] %globaltimer ns (entry, barrier passed, -, done).
 * Returns the phase count, or -1. */
int forge_b200_step_trace(ForgeB200* h, unsigned long long* out, int cap);
/* 1 when steps at this batch size run as the single persistent kernel, 0
 * when they run as the captured multi-kernel graph, -1 on bad arguments. */
int forge_b200_uses_fused_step(ForgeB200* h, int batch);
/* Kernel launches per decode step (for the bench's launch count). */
int forge_b200_launches_per_step(ForgeB200* h, int batch);

/* Block-level entries: one block of one layer on the handle's stream, on
 * device fp32 arrays the caller owns, at the handle's current positions
 * (the pieces forge_b200_decode_step chains, with the same kernels).
 *   embed:     x[b] = emb[tok[b]]                      (tok: device int32)
 *   qkv_rope:  q = RoPE(Wq n), K/V = (RoPE(Wk n), Wv n) appended at pos,
 *              n = RMSNorm(x) * g1
 *   attention: ctx = softmax(q K^T / sqrt(hd)) V over positions 0..pos
 *   o_proj:    x += Wo ctx
 *   mlp:       y = x + Wd (silu(Wg n) * Wu n), n = RMSNorm(x) * g2 (x may be y)
 *   lm_head:   tok = argmax(head RMSNorm(x) * gF), lowest index on ties;
 *              logits [batch][vocab] when not NULL
 *   advance:   pos += 1 for the first `batch` sequences */
int forge_b200_embed(ForgeB200* h, int batch, const int32_t* tok, float* x);
int forge_b200_qkv_rope(ForgeB200* h, int layer, int batch, const float* x, float* q);
int forge_b200_attention(ForgeB200* h, int layer, int batch, const float* q, float* ctx);
int forge_b200_o_proj(ForgeB200* h, int layer, int batch, const float* ctx, float* x);
int forge_b200_mlp(ForgeB200* h, int layer, int batch, const float* x, float* y);
int forge_b200_lm_head(ForgeB200* h, int batch, const float* x, int32_t* tok, float* logits);
int forge_b200_advance(ForgeB200* h, int batch);

/* ---- per-op entries on caller-owned device memory ------------------------ */
/* y[b][n] = sum_k W[n][k] x[b][k]: W packed int4 (forge_q4_pack_tiles) or
 * bf16 (forge_bf16_pack_tiles); x [batch][K] fp32, y [batch][N] fp32.
 * exact = 1 feeds fp32 activations as hi/lo bf16 pairs. */
int forge_gemv_w4a16_g128(const void* tiles, const void* scale_tiles, int64_t N, int64_t K,
                          const float* x, int batch, float* y, int exact, void* stream);
int forge_gemv_bf16(const void* tiles, int64_t N, int64_t K, const float* x, int batch, float* y,
                    int exact, void* stream);

/* Split-K flash-decode: q [B][H*hd] fp32, caches [B][Hkv][lmax][hd] bf16,
 * pos [B] int32 (device), out [B][H*hd] fp32. workspace: at least
 * forge_flash_decode_workspace_bytes(...) bytes, zeroed once before first use
 * (the kernel leaves its counters at zero). */
int64_t forge_flash_decode_workspace_bytes(int B, int H, int Hkv, int hd, int lmax);
int forge_flash_decode(const float* q, const uint16_t* kc, const uint16_t* vc, const int32_t* pos,
                       int B, int H, int Hkv, int hd, int lmax, float* out, void* workspace,
                       void* stream);

/* Allocation-free split-K flash-decode, for callers that cannot allocate
 * device memory (their device memory belongs to another allocator, they run
 * during stream capture, or their memory budget is fixed): same arguments and
 * results as forge_flash_decode, but the scratch comes from one fixed
 * library-owned device array of forge_flash_decode_noalloc_capacity() bytes
 * (4 MiB) per GPU, held until the process exits; shapes needing more are
 * rejected with FORGE_INVALID_ARGS. Calls share that array, so calls that
 * overlap on the GPU race; order them on one stream. The first call on a
 * device looks up the array's device address and should happen before any
 * stream capture; that address is kept for the process, so the entry must
 * not be used after cudaDeviceReset. Kernel errors go to an error word of
 * this entry alone: forge_flash_decode_noalloc_status waits for the whole
 * device, then reads and clears it (-1 once per error). No other entry of
 * the library uses the array or the word. No counterpart in the reference:
 * it is an addition of this library. */
int64_t forge_flash_decode_noalloc_capacity(void);
int forge_flash_decode_noalloc(const float* q, const uint16_t* kc, const uint16_t* vc, const int32_t* pos,
                               int B, int H, int Hkv, int hd, int lmax, float* out, void* stream);
int forge_flash_decode_noalloc_status(void);

/* The sampler alone on device arrays (gpu_sampler.hexa:89-277, per row):
 * logits [batch][ld] f32, probs [batch][vocab] f32 (working buffer; holds
 * the final distribution), rng_state [batch] int64 (advanced; may be NULL
 * when temperature <= 0), tokens [batch] int32. Asynchronous on stream. */
int forge_sample(const float* logits, int64_t ld, int batch, int vocab, double temperature, int top_k,
                 double top_p, int64_t* rng_state, float* probs, int32_t* tokens, void* stream);

/* Causal (or full) flash-attention prefill on the tcgen05 tensor cores:
 * q, k, v, o [B][H][S][hd] bf16 device arrays (16-byte aligned), hd = 128 or 64,
 * S a multiple of 128; O = softmax(Q K^T / sqrt(hd) + mask) V with fp32
 * accumulation. Asynchronous on `stream`; kernel errors (a wait that ran
 * out) show in forge_ops_check(). */
int forge_flash_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, int B, int H, int S,
                        int hd, int causal, void* stream);

/* Weight preparation (device memory). */
int forge_fill_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t offset, float std,
                           void* stream);
int forge_fill_f32(float* out, int64_t n, float v, void* stream);
int forge_q4_quantize_bf16(const uint16_t* w, int64_t rows, int64_t K, int group, uint8_t* codes,
                           uint16_t* scales, void* stream);
int forge_permute_rows_bf16(const uint16_t* src, uint16_t* dst, int64_t rows, int64_t K, int kind,
                            int64_t param, void* stream);
int forge_bf16_pack_tiles(const uint16_t* w, int64_t N, int64_t K, void* tiles, void* stream);
int forge_q4_pack_tiles(const uint8_t* codes, const uint16_t* scales, int64_t N, int64_t K,
                        int group, void* tiles, void* scale_tiles, void* stream);
int forge_q4_unpack_tiles(const void* tiles, const void* scale_tiles, int64_t N, int64_t K,
                          int group, uint8_t* codes, uint16_t* scales, void* stream);
int64_t forge_q4_tile_bytes(int64_t N, int64_t K);
int64_t forge_q4_scale_tile_bytes(int64_t N, int64_t K, int group);

/* Failure-detection self-test of the tensor-parallel peer exchange on one
 * GPU: the exchange buffers of T ranks (2..8) live in this process and only
 * rank 0 runs its all-reduce of n floats, so its waits for the other ranks'
 * flags run out after wait_ns (>= 1 ms). Writes the device error bits
 * (2 = a flag wait ran out) and the kernel's time in ms, then checks that
 * the context still runs work. 0 when the launch ended and the context is
 * usable. The engine's own limit is 2 s, or FORGE_WAIT_NS (ns) read when a
 * tensor-parallel handle is created. */
int forge_tp_selftest_absent_peer(int T, int n, unsigned long long wait_ns, uint32_t* err_bits, double* ms);

/* ---- Training-side families (float64, as the reference's forge kernels in
 * self/cuda/runtime_cuda_emit.hexa) on caller-owned device arrays; 0 or an
 * error code; asynchronous on `stream`. Same contracts as the reference's
 * _hx_cuda_farr_*_gpu entries, minus its farr table (device pointers here).
 *   rmsnorm_rows      y[r] = x[r] / sqrt(mean(x[r]^2) + eps)          (:1098, :1577)
 *   rmsnorm_bwd_rows  dx = inv dxn - inv^3 x dot(dxn, x) / C, eps 1e-6 (:1130, :1609)
 *   adamw_step        decoupled-wd AdamW; m, v updated in place; out may be w
 *                     (step_t >= 1; bias corrections 1 - beta^t)       (:1170-1230, :1640-1780)
 *   rope              rotate-half RoPE on [T][nheads][hd], tables [T][hd];
 *                     bwd = its transpose                              (:2228-2280, :2582-2596)
 *   silu              mode 0 silu(x), 1 d silu / dx, 2 silu(x) * gate_b
 *                     (the gate with flame's series exp)               (:2171-2195, :3033)
 *   attn_fwd          causal GQA attention, P [nh][T][T] kept, ctx [T][nh*hd];
 *                     q [T][nh][hd], k and v [T][nkv][hd]              (:2819-2895, :3159)
 *   attn_bwd          dq, dk, dv from q, k, v, P, dctx; scratch [nh][T][T] (:2896-3031, :3237) */
int forge_train_rmsnorm_rows(const double* x, int64_t R, int64_t C, double eps, double* y, void* stream);
int forge_train_rmsnorm_bwd_rows(const double* x, const double* dxn, int64_t R, int64_t C, double* dx, void* stream);
int forge_train_adamw_step(double* w, double* m, double* v, const double* g, int64_t n, double lr, double b1,
                           double b2, double eps, double wd, int64_t step_t, double* out, void* stream);
int forge_train_rope(const double* t, const double* cos_t, const double* sin_t, int64_t T, int64_t nheads,
                     int64_t hd, int bwd, double* out, void* stream);
int forge_train_silu(const double* x, const double* gate_b, int64_t n, int mode, double* out, void* stream);
int forge_train_attn_fwd(const double* q, const double* k, const double* v, int64_t T, int64_t nh, int64_t nkv,
                         int64_t hd, double* p, double* ctx, void* stream);
int forge_train_attn_bwd(const double* q, const double* k, const double* v, const double* p, const double* dctx,
                         int64_t T, int64_t nh, int64_t nkv, int64_t hd, double* dq, double* dk, double* dv,
                         double* scratch, void* stream);

#ifdef __cplusplus
}
#endif
#endif
