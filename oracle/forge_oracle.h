/* forge_oracle.h — CPU oracle for the flame -> forge decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.
 * The product library (libforge_b200.so) never links or calls it.
 *
 * It restates, in plain C, the reference's decode semantics:
 *   - nn_decoder_fwd / nn_decoder_predict   stdlib/flame/decoder_lib.hexa:93-208, 485-500
 *   - nn_decoder_block_fwd                  stdlib/flame/decoder_block_lib.hexa:217-508
 *   - RMSNorm / attention core / SwiGLU / RoPE / embedding / LM head
 *                                           stdlib/flame/nn_lib.hexa:150-171, 221-278,
 *                                           385-412, 509-562, 589-651
 *   - int4 fake-quant / pack / unpack       stdlib/flame/quant_lib.hexa:33-141
 *   - bf16 RNE rounding                     self/cuda/runtime_bf16_emit.hexa:264-286
 *   - flame LCG fill                        stdlib/flame/tensor_lib.hexa:67-88
 *   - split-K decode merge (flash-decode)   self/ml/flash_decode.hexa:1-45
 * plus the KV-cache decode step (new work; proven equal to the full-recompute
 * path by the tests) and the group-128 int4 generalisation of quant_lib.
 */
#ifndef FORGE_ORACLE_H
#define FORGE_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* ---- bf16 ------------------------------------------------------------ */
uint16_t or_f32_to_bf16(float v);
float    or_bf16_to_f32(uint16_t b);
void     or_f32_to_bf16_n(const float* src, uint16_t* dst, int64_t n);
void     or_bf16_to_f32_n(const uint16_t* src, float* dst, int64_t n);

/* ---- flame LCG + quant_lib (f64, exactly as the reference) ------------ */
void or_flame_fill_lcg(double* t, int64_t n, int64_t seed, double scale);
void or_int4_quant_fwd(const double* w, double* wq_out, double* scale_out,
                       double* qlevel_out, double* mask_out, int cout, int rest);
void or_int4_pack(const double* w, uint8_t* packed_out, int n, double scale, int zero);
void or_int4_unpack(const uint8_t* packed, double* w_out, int n, double scale, int zero);

/* ---- group int4 (bf16 scales) ----------------------------------------- */
/* codes: [rows][K/2] bytes, even k in the low nibble, code = q + 7.
 * scales: [rows][K/group] bf16 bits. Returns 0, or -1 on bad shape. */
int  or_q4g_quantize_bf16(const uint16_t* w, int64_t rows, int64_t K, int group,
                          uint8_t* codes, uint16_t* scales);
int  or_q4g_dequant(const uint8_t* codes, const uint16_t* scales, int64_t rows,
                    int64_t K, int group, float* out);

/* ---- synthetic data ---------------------------------------------------- */
/* N(0, std) from a counter-based hash: element i of stream `seed` is a
 * function of (seed, offset + i) only. Bit-identical to the device fill. */
void   or_fill_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t offset, float std);
double or_normal_at(uint64_t seed, uint64_t idx);
/* RoPE tables [lmax][hd/2], float, built in double. */
void   or_rope_table(float* cos_t, float* sin_t, int lmax, int hd, double theta);

/* ---- model ------------------------------------------------------------- */
enum { OR_MAT_F32 = 0, OR_MAT_BF16 = 1, OR_MAT_Q4 = 2 };
typedef struct OrMat {
    int32_t kind;        /* OR_MAT_*                                     */
    int32_t group;       /* q4 group size along cols                     */
    int64_t rows, cols;  /* W is [rows][cols] row-major: y = W x         */
    const void* w;       /* float* / uint16_t* (bf16) / uint8_t* codes    */
    const uint16_t* scales; /* q4 only: [rows][cols/group] bf16           */
} OrMat;

typedef struct OrLayer {
    const float* g1;
    OrMat wq, wk, wv, wo;
    const float* g2;
    OrMat wg, wu, wd;
} OrLayer;

typedef struct OrModel {
    int32_t n_layer, d, n_head, n_kv, hd, ffn, vocab;
    float   eps, theta;
    const OrLayer* layers;  /* n_layer entries */
    OrMat   emb;            /* [vocab][d]      */
    const float* gF;        /* [d]             */
    OrMat   head;           /* [vocab][d]; tied -> same as emb */
} OrModel;

/* decode flags */
#define OR_KV_BF16   1   /* store K/V rounded to bf16 (device cache format) */
#define OR_ACT_BF16  2   /* round every GEMV input vector to bf16           */
#define OR_NO_ROPE   4   /* skip RoPE (pins the reference's rope-free decode_eager cpu_ref) */

/* One KV-cache decode step for B sequences. kc/vc: [L][B][Hkv][lmax][hd]
 * floats. Token b sits at position pos[b] (its K/V are written there) and
 * attends to positions 0..pos[b]. logits: [B][V] (may be NULL); argmax: [B]
 * (first max wins, decoder_lib.hexa:485-500). hidden_out: [B][d] final
 * residual stream before the final norm (may be NULL). Returns 0 / -1. */
int or_decode_step(const OrModel* m, float* kc, float* vc, int lmax, int B,
                   const int32_t* tok, const int32_t* pos, int flags,
                   float* logits, int32_t* argmax, double* hidden_out);

/* Full recompute of the last-position logits over ids[0..T), no cache,
 * f64 throughout — nn_decoder_fwd + tied/untied head (decoder_lib.hexa:93-208). */
int or_full_forward(const OrModel* m, const int32_t* ids, int T, double* logits);

/* Greedy decode: prompt of n_prompt ids, then n_gen argmax steps (batch 1).
 * out_ids receives n_gen generated ids; margins (may be NULL) the top-1 minus
 * top-2 logit gap of each generated step. */
int or_greedy(const OrModel* m, int lmax, const int32_t* prompt, int n_prompt,
              int n_gen, int flags, int32_t* out_ids, float* margins);

/* Single-query split-K attention with LSE merge (flash_decode.hexa:14-27).
 * q [hd], K/V [L][hd]; returns out [hd]. Used to pin the merge algebra. */
void or_flash_decode_single(const float* q, const float* K, const float* V,
                            int L, int hd, int chunk, double* out);

/* Dense helpers used by known-answer tests: C[M][N] = A[M][K] B[K][N] (f64). */
void or_matmul_f64(const double* A, const double* B, double* C, int M, int K, int N);

int  or_num_threads(void);

/* Input generator of the reference's single-layer decode check
 * (tool/decode_eager_baseline.cu:53-54): state = state*1664525 + 1013904223
 * (mod 2^32), value = (state >> 8) / 2^24 - 0.5 in float. Writes n values
 * and advances *state. */
void or_ref_lcg_f32(uint32_t* state, float* out, int64_t n);

/* Sampler RNG step (self/ml/gpu_sampler.hexa:57-65): 64-bit two's-complement
 * state, x ^= x*8192; x ^= x/131072 (division truncating toward zero);
 * x ^= x*32; x = |x|; returns (x % 1000000) / 1e6. */
double or_sampler_rand(int64_t* state);
/* One token from logits [V] (gpu_sampler.hexa:89-277): temperature <= 0 is
 * the first-max argmax; otherwise temperature scaling, softmax, top-k
 * (0 < k < V: entries below the k-th largest probability zeroed,
 * renormalised), top-p (0 < p < 1: nonzero entries sorted descending by
 * selection sort with swaps, the shortest prefix whose running sum reaches p
 * kept, renormalised), then the first index whose running sum exceeds one
 * draw of the RNG (V - 1 if none). f64 arithmetic, every stored value
 * rounded to f32, sums in the reference's order. probs (may be NULL)
 * receives the final distribution. */
int or_sample_token(const float* logits, int V, double temperature, int top_k, double top_p,
                    int64_t* rng_state, float* probs);
/* ---- Training-side forge families, float64, the reference's sequential
 * order of operations (self/cuda/runtime_cuda_emit.hexa), no contraction. */
/* flame's series exp (runtime_cuda_emit.hexa:2709-2725): halve until
 * |x| <= 1/4 (r times), 12 Taylor terms, square r times. */
double or_dt_exp(double x);
/* 1 / dt_sqrt(hd): 24 Newton steps from max(x, 1) (:2726-2740). */
double or_attn_scale(int64_t hd);
/* y = x / sqrt(mean(x^2) + eps) per row (:1095-1120). */
void or_train_rmsnorm_rows(const double* x, int64_t R, int64_t C, double eps, double* y);
/* dx = inv dxn - inv^3 x dot(dxn, x) / C, eps 1e-6 (:1123-1165). */
void or_train_rmsnorm_bwd_rows(const double* x, const double* dxn, int64_t R, int64_t C, double* dx);
/* AdamW with decoupled weight decay; m, v in place (:1167-1230, host
 * bias corrections :1640-1705). out may be w. */
void or_train_adamw(double* w, double* m, double* v, const double* g, int64_t n, double lr, double b1, double b2,
                    double eps, double wd, int64_t step_t, double* out);
/* rotate-half RoPE on [T][nheads][hd], tables [T][hd]; bwd = transpose (:2228-2280). */
void or_train_rope(const double* t, const double* c, const double* s, int64_t T, int64_t nheads, int64_t hd, int bwd,
                   double* out);
/* mode 0 silu, 1 silu', 2 silu(a) b with or_dt_exp (:2171-2195, :3033-3045). */
void or_train_silu(const double* a, const double* b, int64_t n, int mode, double* out);
/* causal GQA attention, P [nh][T][T], ctx [T][nh*hd] (:2819-2895). */
void or_train_attn_fwd(const double* q, const double* k, const double* v, int64_t T, int64_t nh, int64_t nkv,
                       int64_t hd, double* p, double* ctx);
/* its backward: dq [T][nh][hd], dk and dv [T][nkv][hd] (:2896-3031). */
void or_train_attn_bwd(const double* q, const double* k, const double* v, const double* p, const double* dctx,
                       int64_t T, int64_t nh, int64_t nkv, int64_t hd, double* dq, double* dk, double* dv);
#ifdef __cplusplus
}
#endif
#endif
