// forge_internal.h — shared host-side declarations of the forge_b200 library.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define FORGE_API __attribute__((visibility("default")))

enum { FORGE_PERM_NONE = 0, FORGE_PERM_QKV = 1, FORGE_PERM_GATEUP = 2 };

// Records a one-line error (returned by forge_b200_last_error and printed once
// to stderr, the reference's "one stderr line, return -1" contract) and
// returns `code`.
int forge_fail(int code, const char* fmt, ...);
// Reference sampler over logits rows (sample.cu); probs is the working
// distribution [batch][pld], tokens and RNG states per row.
int forge_sample_launch(const float* logits, int64_t ld, int batch, int vocab, double temperature, int top_k,
                        double top_p, int64_t* rng_state, float* probs, int64_t pld, int32_t* tokens,
                        cudaStream_t stream);
// The logical (unsharded) description a model handle was created with.
extern "C" const struct ForgeModelDesc* forge_b200_desc_of(const struct ForgeB200* h);
// Checks cudaGetLastError after a launch; 0 or -1.
int forge_check_launch(const char* what);
// Number of SMs of the current device (cached per device).
int forge_sm_count();

// ------------------------------------------------------------ GEMV launch
enum { FORGE_W_BF16 = 0, FORGE_W_Q4 = 1 };
enum { FORGE_PRO_PLAIN = 0, FORGE_PRO_RMSNORM = 1, FORGE_PRO_EMBED_RMSNORM = 2 };
enum {
    FORGE_EPI_STORE = 0,  // y[b][row] = W x
    FORGE_EPI_RESID = 1,  // y[b][row] += W x   (residual stream, in place)
    FORGE_EPI_QKV = 2,    // RoPE + KV append + q out
    FORGE_EPI_SWIGLU = 3, // s[b][f] = silu(gate) * up
    FORGE_EPI_LOGITS = 4, // logits + running argmax key
    FORGE_EPI_RESID_TP = 5, // y[b][row] += sum over tensor-parallel ranks of W x (peer memory, batch <= 4)
};

struct ForgeGemvArgs {
    const void* w;         // packed tiles
    const void* s;         // q4 scale tiles (NULL for bf16)
    int32_t N, K;          // physical rows / input columns
    int32_t wkind;         // FORGE_W_*
    int32_t batch;         // sequences in this call
    int32_t b0;            // global index of the first sequence (cache/pos indexing)
    int32_t split;         // 1: hi/lo bf16 activations (exact fp32 inputs), 0: bf16
    const float* x;        // [batch][x_stride] fp32 input
    int32_t x_stride;
    int32_t pro;           // FORGE_PRO_*
    const float* gain;     // RMSNorm gain [K]
    float eps;
    const uint16_t* emb;   // EMBED prologue: embedding table [V][K] bf16
    const int32_t* emb_tok;// EMBED prologue: token per sequence (global index)
    int32_t epi;           // FORGE_EPI_*
    float* y;              // STORE/RESID/LOGITS output [batch][y_stride]
    int32_t y_stride;
    // QKV epilogue
    float* q_out;          // [batch][H*hd]
    uint16_t* kc;          // layer base of the K cache: [Btot][Hkv][lmax][hd] bf16
    uint16_t* vc;
    const int32_t* pos;    // [Btot] position of the token being decoded
    int32_t H, Hkv, hd, lmax;
    const float* rope_cos; // [lmax][hd/2]
    const float* rope_sin;
    // SwiGLU epilogue
    float* s_out;          // [batch][F]
    int32_t F;
    // LOGITS epilogue
    unsigned long long* argmax_key;  // [Btot]
    int32_t nvalid;        // rows >= nvalid (zero padding) never win the argmax
    int32_t row_off;       // global index of row 0 in the argmax key (vocabulary shard)
    void* bscratch;        // int4, batch > 4: forge_gemv_b_scratch_bytes(K) bytes for the batched path
    const struct ForgeTpFusedDev* tpf;  // FORGE_EPI_RESID_TP: the ranks' exchange buffers (device memory)
    uint32_t* err;         // device error word
    // Optional timeline [grid][4] %globaltimer stamps (CTA start, dependency
    // released, activations staged, units done), FORGE_GRAPH_TRACE only.
    unsigned long long* trace;
    // Prompt prefill: row b of the launch is position pos[b] of cache
    // sequence seq_of[b] (null: row b is sequence b).
    const int32_t* seq_of;
    // Quantised-activation handoff (int4 weights, plain prologue, batch <= 4):
    // pq_in, when set, is the staged block of this GEMV's input, written by
    // the kernel before it — [K/128][4] f32 scales, [K/128][8] s32 column
    // sums, [K][2 batch] int8 hi/lo in the shared-memory layout of the
    // staging — and is copied instead of staged.
    const uint8_t* pq_in;
    // With an RMSNorm prologue: pq_in holds the codes of gain * x and pq_ssq
    // [batch][K/128] the sums of squares of x per group; the GEMV forms the
    // RMSNorm factor from them and folds it into the group scales.
    const float* pq_ssq;
};

// Bytes of a handoff block for K inputs and `batch` sequences.
__host__ __device__ inline int64_t forge_pq_bytes(int K, int batch) {
    return (int64_t)(K / 128) * 48 + (int64_t)K * 2 * batch;
}

// Launches the decode GEMV (one or more launches when the batch exceeds one
// mma column block). pdl: launch with programmatic stream serialization.
int forge_gemv_launch(const ForgeGemvArgs& a, cudaStream_t stream, bool pdl);
int forge_gemv_configure();
int forge_gemv_launch_count(int K, int batch, bool split, bool q4, bool batched);
// x [B][x_stride] (K % 128 == 0, B <= 4) staged into an int4 GEMV's input
// block (layout of ForgeGemvArgs::pq_in), one warp per 128-group; with a
// gain, the block of an RMSNorm GEMV (codes of gain * x, and the groups'
// sums of squares of x in ssq [B][K / 128], see ForgeGemvArgs::pq_ssq).
int forge_stage_groups_launch(const float* x, int x_stride, int K, int B, uint8_t* blk, const float* gain, float* ssq,
                              cudaStream_t stream, bool pdl);
// Batched int4 path (gemv_batched.cu): up to forge_gemv_b_max_seq()
// sequences per weight stream.
int forge_gemv_b_max_seq();
int64_t forge_gemv_b_scratch_bytes(int K);
int forge_gemv_b_configure();
int forge_gemv_b_launch(const ForgeGemvArgs& a, void* scratch, cudaStream_t stream, bool pdl);
// int4 chunks of the batched path on the tensor cores (gemv_tc.cu); the
// scratch must start zeroed (ticket counters) and is kept so by the kernel.
int64_t forge_gemv_tc_scratch_bytes(int K);
int64_t forge_gemv_scratch_header();
// cuTensorMapEncodeTiled through the runtime's driver entry point (NULL if
// unavailable); prefill.cu.
using ForgeEncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
ForgeEncodeTiled forge_tensor_map_encoder();  // bytes at the start of the scratch the other batched paths skip
int forge_gemv_tc_configure();
int forge_gemv_tc_launch(const ForgeGemvArgs& a, void* scratch, cudaStream_t stream, bool pdl);

// ------------------------------------------------------ flash-decode launch
struct ForgeAttnArgs {
    const float* q;        // [B][H*hd] fp32 (RoPE applied)
    const uint16_t* kc;    // layer base [B][Hkv][lmax][hd] bf16
    const uint16_t* vc;
    const int32_t* pos;    // [B]; attends to positions 0..pos[b]
    int32_t B, H, Hkv, hd, lmax;
    int32_t nsplit;        // KV splits per (b, kv head)
    float* partial;        // [B][H][nsplit][hd + 2] scratch
    uint32_t* counters;    // [B][Hkv] zero-initialised merge counters
    float* out;            // [B][H*hd] fp32 context
    uint32_t* err;
    // Paged cache (table != nullptr): kc / vc are page pools
    // [num_pages][Hkv][page_tokens][hd]; row r of sequence b lives on page
    // table[b * max_pages + r / page_tokens]; lmax = max_pages * page_tokens.
    const int32_t* table;
    int32_t max_pages, page_tokens, num_pages;
    // Flat kernel (attn_flat.cu): partial slots per (b, kv head); partial is
    // [B][Hkv][flat_slots][H/Hkv][hd + 2].
    int32_t flat_slots;
    // Optional timeline (FORGE_GRAPH_TRACE only), [CTA][4] %globaltimer
    // stamps. Flat kernel: start, dependency released, first query loaded,
    // done. Split kernel, for the first trace_ctas CTAs (x fastest): start,
    // dependency released, partial written, merge done (merging CTA only).
    unsigned long long* trace;
    int32_t trace_ctas;
    // Prompt prefill (split kernel, contiguous cache): query row b attends
    // to rows 0..pos[b] of cache sequence seq_of[b] (null: sequence b).
    const int32_t* seq_of;
    // Handoff (hd 128, B <= 4): the merged context of every head, one
    // 128-group of the O projection's input, also written staged into this
    // block (layout of ForgeGemvArgs::pq_in for K = H * hd).
    uint8_t* pq_out;
};
int forge_attn_launch(const ForgeAttnArgs& a, cudaStream_t stream, bool pdl);
// Flat small-batch flash-decode (attn_flat.cu).
bool forge_attn_flat_supported(int B, int H, int Hkv, int hd);
int forge_attn_flat_slots(int hd, int lmax);
int64_t forge_attn_flat_partial_floats(int B, int H, int hd, int lmax);
int forge_attn_flat_configure();
int forge_attn_flat_launch(const ForgeAttnArgs& a, cudaStream_t stream, bool pdl);
int forge_attn_configure();
int forge_attn_pick_splits(int B, int Hkv, int lmax);
int64_t forge_attn_partial_floats(int B, int H, int hd, int nsplit);

// ------------------------------------------------------------- misc kernels
int forge_embed_launch(const uint16_t* emb, int d, int vocab, const int32_t* tok, int B, float* x,
                       uint32_t* err, cudaStream_t stream, bool pdl);
int forge_argmax_finalize_launch(unsigned long long* keys, int B, int32_t* tok_out,
                                 int32_t* hist, int32_t* step_counter, int32_t* pos, int hist_cap,
                                 cudaStream_t stream, bool pdl);

// ------------------------------------------------- persistent decode step
enum { FORGE_PH_GEMV = 0, FORGE_PH_ATTN = 1, FORGE_PH_FIN = 2 };
struct ForgePhase {
    int32_t type;          // FORGE_PH_*
    ForgeGemvArgs g;       // GEMV: full description; ATTN: g.kc / g.vc layer caches
};
struct ForgeStepArgs {
    const ForgePhase* phases;  // device array
    int32_t nphases;
    int32_t grid, stages;
    int32_t B, H, Hkv, hd, lmax, nsplit;
    const float* q;
    float* ctx;
    int32_t* pos;
    float* partial;
    uint32_t* counters;
    unsigned long long* amax;
    int32_t *tok, *hist, *step;
    int32_t hist_cap;
    unsigned long long* bar;   // monotonic grid-barrier counter
    uint32_t* epoch;           // completed fused steps since the last reset
    uint32_t* err;
    unsigned long long* trace; // optional [grid][nphases][4] %globaltimer stamps
};
// 0 launched (or fits, with probe_only), 1 does not fit / unsupported, -1 error.
int forge_step_launch(const ForgeStepArgs& sa, int xf_bytes, cudaStream_t stream, bool probe_only);
int forge_step_attn_tile(int hd);

// ------------------------------------------------------------ dispatch glue
struct ForgeB200;
struct ForgeShapeInfo;
struct ForgeArgs;
// Row widths of a handle's activations: 0 model dim, 1 query width H*hd,
// 2 vocabulary; 0 for a null handle.
extern "C" int64_t forge_b200_width(const ForgeB200* h, int which);
// Synthetic weights: block [nr][nc] of a matrix with `stride` columns.
int forge_fill_normal_bf16_2d(uint16_t* out, int64_t nr, int64_t nc, uint64_t seed, uint64_t offset, int64_t stride,
                              float std, cudaStream_t stream);

// Tensor parallel (tp.cu): NCCL opened at run time.
int forge_tp_comm_init(void** comm, const void* unique_id, int rank, int size);
void forge_tp_comm_destroy(void* comm);
int forge_tp_allreduce_sum_f32(void* comm, float* buf, size_t count, cudaStream_t stream);
int forge_tp_allreduce_max_u64(void* comm, unsigned long long* buf, size_t count, cudaStream_t stream);
int forge_tp_allgather_f32(void* comm, const float* send, float* recv, size_t count, cudaStream_t stream);

// One-shot all-reduce over NVLink peer memory (tp_allreduce.cu).
struct ForgeTpAr;
// Peer-memory exchange of the GEMV epilogue FORGE_EPI_RESID_TP (device
// memory, one per rank): every rank's receive buffer [2 generations][T][cap]
// floats and per-tile flags [2][T][max_tiles] mapped from all peers, and
// this rank's per-tile call counters.
struct ForgeTpFusedDev {
    float* buf[8];
    uint32_t* flag[8];
    uint32_t* tile_epoch;  // [max_tiles], local
    int T, rank, cap, max_tiles;
};
const ForgeTpFusedDev* forge_tp_fused_dev(const ForgeTpAr* ar);
int forge_tp_ar_init(void* comm, int rank, int T, int cap, cudaStream_t stream, ForgeTpAr** out);
void forge_tp_ar_destroy(ForgeTpAr* ar);
int forge_tp_ar_capacity(const ForgeTpAr* ar);
// Handoff from the one-shot all-reduce to the next GEMV (batch <= 4, int4):
// the summed x staged as that GEMV's input block (codes of gain * x, see
// ForgeGemvArgs::pq_in) plus per (sequence, 128-group) sums of squares of x.
struct ForgeArHandoff {
    uint8_t* pq;          // null: no handoff
    float* ssq;           // [batch][d / 128]
    const float* gain;    // RMSNorm gain of the next GEMV [d]
    int batch, d;
};
int forge_tp_ar_sum_f32(ForgeTpAr* ar, float* x, int n, uint32_t* err, cudaStream_t stream,
                        const ForgeArHandoff* handoff = nullptr);

// Per-device error word of the per-op entries (created on first use).
uint32_t* forge_ops_err_word();
int forge_flash_prefill_kv(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, uint16_t* o, int B, int H,
                           int Hkv, int S, int hd, int kv_ld, int64_t kv_rows, cudaStream_t stream);
// v2 FLASH_PREFILL family.
int forge_prefill_dispatch(const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out);
