// model.cu — the decode engine: one ForgeB200 handle per GPU owns the packed
// weights, the bf16 KV cache, the step's activation buffers and one CUDA graph
// per batch size. A decode step is
//     embed -> L x [QKV(+RMSNorm,RoPE,KV append) -> flash-decode ->
//                   O(+residual) -> gate/up(+RMSNorm,SwiGLU) -> down(+residual)]
//     -> LM head(+final RMSNorm, logits, argmax) -> finalize(next token)
// i.e. decoder_lib.hexa:93-208 + decoder_block_lib.hexa:217-508 +
// nn_decoder_predict (:485-500) for one new position per sequence, with the
// KV cache replacing the reference's full recompute. All launches after the
// first use programmatic dependent launch, so each GEMV's weight stream
// starts while the previous kernel drains; the whole step is captured once
// per batch size and replayed.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <vector>
#include "common.cuh"
#include "layout.cuh"
#include "forge_internal.h"
#include "../../include/forge_b200.h"

namespace {
struct LayerDev {
    void *qkv_w = nullptr, *qkv_s = nullptr;
    void *o_w = nullptr, *o_s = nullptr;
    void *gu_w = nullptr, *gu_s = nullptr;
    void *dn_w = nullptr, *dn_s = nullptr;
    float *g1 = nullptr, *g2 = nullptr;
};

__global__ void k_embed(const uint16_t* __restrict__ emb, int d, int vocab, const int32_t* __restrict__ tok,
                        float* __restrict__ x, uint32_t* err) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x;
    int t = tok[b];
    if (t < 0 || t >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, FORGE_DEVERR_BAD_INDEX);
        t = 0;
    }
    const uint16_t* row = emb + (size_t)t * d;
    for (int k = threadIdx.x * 2; k < d; k += blockDim.x * 2) {
        const uint32_t v = *reinterpret_cast<const uint32_t*>(row + k);
        x[(size_t)b * d + k] = bf16_lo_f32(v);
        x[(size_t)b * d + k + 1] = bf16_hi_f32(v);
    }
}

__global__ void k_finalize(unsigned long long* keys, int B, int32_t* tok, int32_t* hist, int32_t* step,
                           int32_t* pos, int hist_cap, int hist_stride) {
    pdl_trigger();
    pdl_wait();
    const int b = threadIdx.x;
    const int s = *step;
    if (b < B) {
        const unsigned long long k = keys[b];
        const int32_t t = k ? (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0;
        tok[b] = t;
        if (s < hist_cap) hist[(size_t)s * hist_stride + b] = t;
        keys[b] = 0ull;
        pos[b] += 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) *step = s + 1;
}

// Token ids out of the packed argmax keys (keys reset for the next use),
// without touching positions or the step history.
__global__ void k_argmax_extract(unsigned long long* keys, int B, int32_t* tok) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) {
        const unsigned long long k = keys[b];
        tok[b] = k ? (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0;
        keys[b] = 0ull;
    }
}

// Prompt rows (row b * n + p of a [rows][H * hd] fp32 array) to and from
// the [B][H][S][hd] bf16 layout of the tensor-core prefill; positions n..S-1
// of the bf16 side are zero.
__global__ void k_rows_to_heads_bf16(const float* __restrict__ q, int B, int n, int S, int H, int hd,
                                     uint16_t* __restrict__ qb) {
    const int64_t total = (int64_t)B * H * S * hd;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int e = (int)(i % hd);
        const int64_t r = i / hd;
        const int p = (int)(r % S);
        const int64_t bh = r / S;
        const int hh = (int)(bh % H), b = (int)(bh / H);
        qb[i] = p < n ? f32_to_bf16_bits(q[(((int64_t)b * n + p) * H + hh) * hd + e]) : (uint16_t)0;
    }
}
__global__ void k_heads_bf16_to_rows(const uint16_t* __restrict__ ob, int B, int n, int S, int H, int hd,
                                     float* __restrict__ ctx) {
    const int64_t total = (int64_t)B * n * H * hd;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int e = (int)(i % hd);
        const int64_t t = i / hd;
        const int hh = (int)(t % H);
        const int64_t r = t / H;
        const int p = (int)(r % n), b = (int)(r / n);
        ctx[i] = bf16_bits_to_f32(ob[(((int64_t)b * H + hh) * S + p) * hd + e]);
    }
}

// dst[r] = src[rows[r]] for r < n, rows of d floats (one CTA per row).
__global__ void k_gather_rows(const float* __restrict__ src, const int32_t* __restrict__ rows, int d,
                              float* __restrict__ dst) {
    const float* a = src + (size_t)rows[blockIdx.x] * d;
    float* o = dst + (size_t)blockIdx.x * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) o[i] = a[i];
}

__global__ void k_add_i32(int32_t* p, int n, int32_t v) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] += v;
}

__global__ void k_set_i32(int32_t* p, int n, int32_t v) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = v;
}

int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }
}  // namespace

struct ForgeB200 {
    ForgeModelDesc desc{};
    int device = 0;
    cudaStream_t stream = nullptr;
    int L = 0, d = 0, H = 0, Hkv = 0, hd = 0, F = 0, V = 0, Vpad = 0, qd = 0, kvd = 0, nqkv = 0;
    int Bmax = 0, lmax = 0;
    bool q4 = false;
    std::vector<LayerDev> layers;
    uint16_t* emb = nullptr;
    void* head_w = nullptr;
    float* gF = nullptr;
    uint16_t *kc = nullptr, *vc = nullptr;
    size_t kv_layer = 0;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    int32_t *tok = nullptr, *pos = nullptr, *hist = nullptr, *step = nullptr;
    int hist_cap = 0;
    float *x = nullptr, *q = nullptr, *ctx = nullptr, *s = nullptr, *logits = nullptr;
    unsigned long long* amax = nullptr;
    float* partial = nullptr;
    uint32_t* counters = nullptr;
    int nsplit = 1;
    bool flat_attn = false;  // small batches on attn_flat.cu (FORGE_ATTN=flat)
    // Staged-input handoffs of the decode step for batch <= 4 (int4
    // weights; FORGE_PREQUANT=0 turns them all off): the GEMV copies its
    // input block (int8 hi/lo groups, scales, column sums) instead of
    // staging it.
    // - context: the flash-decode merge stages each head's context for the O
    //   projection (head dim 128; a rank's own heads under tensor parallelism)
    bool prequant = false;
    uint8_t* pq_ctx = nullptr;
    // - s: a small kernel stages the SwiGLU output for the down projection
    //   (FORGE_PREQUANT_S=0 turns it off); same bytes as the staging
    bool pq_s_on = false;
    uint8_t* pq_s = nullptr;
    // - x: the residual stream for the next RMSNorm GEMV (QKV after down,
    //   gate/up after O) as codes of gain * x plus the groups' sums of squares
    //   [4][d / 128], from which the GEMV forms its RMSNorm factor; written by
    //   the peer-memory all-reduce under tensor parallelism, else by the small
    //   kernel (FORGE_PREQUANT_NORM=0 turns it off; logits within the last
    //   bits of the staging's)
    bool pq_norm = false;
    uint8_t* pq_x = nullptr;
    float* pq_ssq = nullptr;
    uint32_t* err = nullptr;
    uint16_t *stA = nullptr, *stB = nullptr;
    uint8_t* codes = nullptr;
    uint16_t* scales = nullptr;
    int32_t* h_tok = nullptr;  // pinned staging [Bmax]
    float* samp_probs = nullptr;     // sampler distribution [Bmax][Vpad] (first sampled step)
    int64_t* samp_rng = nullptr;     // sampler RNG states [Bmax]
    std::map<int, cudaGraphExec_t> graphs;
    std::map<int, ForgeStepArgs> fused;   // per batch size: fused-step arguments (phases on device)
    std::map<int, int> fused_ok;          // per batch size: 1 fused path fits, 0 no
    unsigned long long* bar = nullptr;
    uint32_t* epoch = nullptr;
    int force_graph = 0;
    unsigned long long* trace = nullptr;  // fused-step timeline (FORGE_STEP_TRACE)
    int trace_n = 0;
    // prompt prefill rows (grown on demand): activations, per-row token /
    // position / sequence, split partials and merge counters
    struct {
        int64_t cap = 0;
        float *x = nullptr, *q = nullptr, *ctx = nullptr, *s = nullptr, *partial = nullptr;
        int32_t *tok = nullptr, *pos = nullptr, *seq = nullptr;
        int32_t* sel = nullptr;  // [2][Bmax]: rows that take the LM head, their tokens
        uint32_t* counters = nullptr;
        // tensor-core prompt attention: Q and O as [B][H][S][hd] bf16
        uint16_t *qb = nullptr, *ob = nullptr;
        int64_t qb_cap = 0;
    } pre;
    // multi-kernel step timeline (FORGE_GRAPH_TRACE): [node][grid][4] stamps
    unsigned long long* gtrace = nullptr;
    int gtrace_cap = 0, gtrace_next = 0;
    std::vector<void*> allocs;
    bool weights_ready = false;
    // tensor parallel shard (tp_size 1: the whole model). H, Hkv, F, V and
    // Vpad above are this rank's; the *full fields are the model's.
    int tp_rank = 0, tp_size = 1;
    int Hfull = 0, Hkvfull = 0, Ffull = 0, Vfull = 0;
    int h0 = 0, kv0 = 0, f0 = 0, v0 = 0;  // first head / kv head / FFN row / vocabulary row of this rank
    void* comm = nullptr;                 // NCCL communicator
    void* bscratch = nullptr;             // int4 activations of the batched GEMV path
    ForgeTpAr* ar = nullptr;              // peer-memory all-reduce (tensor parallel)
    float* logits_all = nullptr;          // [tp][Bmax][Vpad] all-gathered logits

    void* alloc(size_t bytes) {
        void* p = nullptr;
        if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) return nullptr;
        allocs.push_back(p);
        return p;
    }
    bool split_for(int B) const {
        if (desc.act_mode == 1) return true;
        if (desc.act_mode == 2) return false;
        return B <= 4;
    }
};

namespace {
size_t tile_bytes(bool q4, int64_t N, int64_t K) { return q4 ? (size_t)(N * K / 2) : (size_t)(N * K * 2); }
size_t scale_bytes(bool q4, int64_t N, int64_t K) {
    return q4 ? (size_t)forge_q4_scale_tile_bytes(N, K, 128) : 0;
}

// Packs the physical-order bf16 matrix in h->stB ([N][K]) into (w, s).
int pack_matrix(ForgeB200* h, int64_t N, int64_t K, void* w, void* s, bool q4) {
    if (q4) {
        int rc = forge_q4_quantize_bf16(h->stB, N, K, 128, h->codes, h->scales, h->stream);
        if (!rc) rc = forge_q4_pack_tiles(h->codes, h->scales, N, K, 128, w, s, h->stream);
        return rc;
    }
    return forge_bf16_pack_tiles(h->stB, N, K, w, h->stream);
}

int alloc_layer(ForgeB200* h, LayerDev& Ld) {
    const bool q4 = h->q4;
    Ld.qkv_w = h->alloc(tile_bytes(q4, h->nqkv, h->d));
    Ld.o_w = h->alloc(tile_bytes(q4, h->d, h->qd));
    Ld.gu_w = h->alloc(tile_bytes(q4, 2 * h->F, h->d));
    Ld.dn_w = h->alloc(tile_bytes(q4, h->d, h->F));
    if (q4) {
        Ld.qkv_s = h->alloc(scale_bytes(q4, h->nqkv, h->d));
        Ld.o_s = h->alloc(scale_bytes(q4, h->d, h->qd));
        Ld.gu_s = h->alloc(scale_bytes(q4, 2 * h->F, h->d));
        Ld.dn_s = h->alloc(scale_bytes(q4, h->d, h->F));
    }
    Ld.g1 = (float*)h->alloc(sizeof(float) * h->d);
    Ld.g2 = (float*)h->alloc(sizeof(float) * h->d);
    if (!Ld.qkv_w || !Ld.o_w || !Ld.gu_w || !Ld.dn_w || !Ld.g1 || !Ld.g2 ||
        (q4 && (!Ld.qkv_s || !Ld.o_s || !Ld.gu_s || !Ld.dn_s)))
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200: out of device memory for layer weights");
    return 0;
}

// Source of one logical matrix: either host bf16 or a synthetic stream.
struct Src {
    const uint16_t* host;
    uint64_t seed, offset;
    float std;
};
int fill_rows(ForgeB200* h, uint16_t* dst, int64_t rows, int64_t K, const Src& s) {
    if (s.host) {
        cudaError_t e = cudaMemcpyAsync(dst, s.host, (size_t)rows * K * 2, cudaMemcpyHostToDevice, h->stream);
        return e == cudaSuccess ? 0 : forge_fail(-1, "forge_b200: H2D weights: %s", cudaGetErrorString(e));
    }
    return forge_fill_normal_bf16(dst, rows * K, s.seed, s.offset, s.std, h->stream);
}
// dst [nr][nc] = rows r0.., columns c0.. of the logical matrix with `cols`
// columns (a tensor-parallel shard; the whole matrix when r0 = c0 = 0).
int fill_block(ForgeB200* h, uint16_t* dst, int64_t cols, int64_t r0, int64_t nr, int64_t c0, int64_t nc,
               const Src& s) {
    if (c0 == 0 && nc == cols) {
        Src t = s;
        if (t.host) t.host += r0 * cols;
        else t.offset += (uint64_t)(r0 * cols);
        return fill_rows(h, dst, nr, nc, t);
    }
    if (s.host) {
        cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)nc * 2, s.host + r0 * cols + c0, (size_t)cols * 2,
                                          (size_t)nc * 2, (size_t)nr, cudaMemcpyHostToDevice, h->stream);
        return e == cudaSuccess ? 0 : forge_fail(-1, "forge_b200: H2D weights: %s", cudaGetErrorString(e));
    }
    return forge_fill_normal_bf16_2d(dst, nr, nc, s.seed, s.offset + (uint64_t)(r0 * cols + c0), cols, s.std,
                                     h->stream);
}

int load_layer_impl(ForgeB200* h, int l, const Src src[7], const float* g1, const float* g2, bool gains_one) {
    LayerDev& Ld = h->layers[l];
    const int d = h->d, qd = h->qd, kvd = h->kvd, F = h->F, hd = h->hd;
    const int64_t qfull = (int64_t)h->Hfull * hd;
    int rc = 0;
    // QKV: this rank's heads of [Wq; Wk; Wv] -> RoPE-pair permutation -> pack
    rc |= fill_block(h, h->stA, d, (int64_t)h->h0 * hd, qd, 0, d, src[0]);
    rc |= fill_block(h, h->stA + (size_t)qd * d, d, (int64_t)h->kv0 * hd, kvd, 0, d, src[1]);
    rc |= fill_block(h, h->stA + (size_t)(qd + kvd) * d, d, (int64_t)h->kv0 * hd, kvd, 0, d, src[2]);
    if (rc) return -1;
    if (forge_permute_rows_bf16(h->stA, h->stB, h->nqkv, d, FORGE_PERM_QKV, hd, h->stream)) return -1;
    if (pack_matrix(h, h->nqkv, d, Ld.qkv_w, Ld.qkv_s, h->q4)) return -1;
    // O: the columns of this rank's heads (row-split along K)
    if (fill_block(h, h->stB, qfull, 0, d, (int64_t)h->h0 * hd, qd, src[3]) ||
        pack_matrix(h, d, qd, Ld.o_w, Ld.o_s, h->q4))
        return -1;
    // gate/up: this rank's FFN rows, interleaved
    if (fill_block(h, h->stA, d, h->f0, F, 0, d, src[4]) ||
        fill_block(h, h->stA + (size_t)F * d, d, h->f0, F, 0, d, src[5]))
        return -1;
    if (forge_permute_rows_bf16(h->stA, h->stB, 2 * F, d, FORGE_PERM_GATEUP, F, h->stream)) return -1;
    if (pack_matrix(h, 2 * F, d, Ld.gu_w, Ld.gu_s, h->q4)) return -1;
    // down: the columns of this rank's FFN rows
    if (fill_block(h, h->stB, h->Ffull, 0, d, h->f0, F, src[6]) || pack_matrix(h, d, F, Ld.dn_w, Ld.dn_s, h->q4))
        return -1;
    // gains
    if (gains_one) {
        if (forge_fill_f32(Ld.g1, d, 1.0f, h->stream) || forge_fill_f32(Ld.g2, d, 1.0f, h->stream)) return -1;
    } else {
        if (cudaMemcpyAsync(Ld.g1, g1, sizeof(float) * d, cudaMemcpyHostToDevice, h->stream) != cudaSuccess ||
            cudaMemcpyAsync(Ld.g2, g2, sizeof(float) * d, cudaMemcpyHostToDevice, h->stream) != cudaSuccess)
            return forge_fail(-1, "forge_b200: H2D gains failed");
    }
    // staging buffers are reused by the next matrix: keep uploads ordered
    return cudaStreamSynchronize(h->stream) == cudaSuccess ? 0 : forge_fail(-1, "forge_b200: weight prep failed");
}

int load_embed_impl(ForgeB200* h, const Src& emb, const Src* head, const float* gF, bool gains_one) {
    const int64_t V = h->V, Vp = h->Vpad, d = h->d;
    if (fill_rows(h, h->emb, h->Vfull, d, emb)) return -1;  // replicated on every rank
    // head tiles (this rank's vocabulary rows) from a zero-padded [Vpad][d] copy
    if (cudaMemsetAsync(h->stB, 0, (size_t)Vp * d * 2, h->stream) != cudaSuccess) return forge_fail(-1, "memset");
    if (V > 0) {
        if (head) {
            if (fill_block(h, h->stB, d, h->v0, V, 0, d, *head)) return -1;
        } else if (cudaMemcpyAsync(h->stB, h->emb + (size_t)h->v0 * d, (size_t)V * d * 2, cudaMemcpyDeviceToDevice,
                                   h->stream) != cudaSuccess) {
            return forge_fail(-1, "forge_b200: head copy failed");
        }
    }
    if (forge_bf16_pack_tiles(h->stB, Vp, d, h->head_w, h->stream)) return -1;
    if (gains_one) {
        if (forge_fill_f32(h->gF, d, 1.0f, h->stream)) return -1;
    } else if (cudaMemcpyAsync(h->gF, gF, sizeof(float) * d, cudaMemcpyHostToDevice, h->stream) != cudaSuccess) {
        return forge_fail(-1, "forge_b200: H2D final gain failed");
    }
    return cudaStreamSynchronize(h->stream) == cudaSuccess ? 0 : forge_fail(-1, "forge_b200: embedding prep failed");
}

// The launches of one decode step, block by block. Each helper reads and
// writes the given device arrays; the step itself passes the handle's own.
ForgeGemvArgs gemv_base(const ForgeB200* h, int B) {
    ForgeGemvArgs a{};
    a.bscratch = h->bscratch;
    a.wkind = h->q4 ? FORGE_W_Q4 : FORGE_W_BF16;
    a.batch = B;
    a.split = h->split_for(B);
    a.err = h->err;
    return a;
}

// Row-split projections under tensor parallelism: rank 0 adds its partial
// product to the residual stream, the other ranks store theirs, and one
// all-reduce (sum) leaves x + sum of all partials on every rank.
int resid_epi(const ForgeB200* h) { return h->tp_rank == 0 ? FORGE_EPI_RESID : FORGE_EPI_STORE; }
// small vectors (up to 32K floats, 8 sequences of 4096): one-shot through
// peer memory; larger ones: NCCL's bandwidth-efficient protocols
bool tp_oneshot(const ForgeB200* h, int B) {
    return h->ar && B * h->d <= 32768 && B * h->d <= forge_tp_ar_capacity(h->ar);
}
bool tp_fused(const ForgeB200* h, int B);
// Whether the decode step at batch B hands the residual stream x staged to
// the next RMSNorm GEMV (written by the all-reduce or the staging kernel).
bool pq_x_on(const ForgeB200* h, int B) {
    return h->pq_norm && B <= 4 && forge_gemv_launch_count(h->d, B, h->split_for(B), true, false) == 1;
}
// whether the peer-memory all-reduce writes the x block
bool pq_by_ar(const ForgeB200* h, int B) { return h->comm && tp_oneshot(h, B) && !tp_fused(h, B); }
// next_gain: the RMSNorm gain of the GEMV that reads x next, when the
// all-reduce hands it x staged (the decode step's own chain only)
int tp_sum(ForgeB200* h, float* x, int B, const float* next_gain = nullptr) {
    if (!h->comm) return 0;
    if (tp_oneshot(h, B)) {
        ForgeArHandoff ho{};
        if (next_gain && pq_x_on(h, B)) ho = ForgeArHandoff{h->pq_x, h->pq_ssq, next_gain, B, h->d};
        return forge_tp_ar_sum_f32(h->ar, x, B * h->d, h->err, h->stream, &ho);
    }
    return forge_tp_allreduce_sum_f32(h->comm, x, (size_t)B * h->d, h->stream);
}

// Up to 4 sequences over peer memory: the O / down GEMV's epilogue exchanges
// each finished 16-row tile with the peers and sums the partials in rank
// order (the bits of GEMV + tp_sum, without the all-reduce launch).
// Opt-in with FORGE_TP_FUSED_RESID=1.
bool tp_fused(const ForgeB200* h, int B) {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("FORGE_TP_FUSED_RESID");
        on = (e && e[0] == '1') ? 1 : 0;
    }
    return on && h->ar && B <= 4 && B * h->d <= forge_tp_ar_capacity(h->ar);
}
int resid_gemv(ForgeB200* h, ForgeGemvArgs& g, float* x, int B, bool pdl, const float* next_gain = nullptr) {
    if (tp_fused(h, B)) {
        g.epi = FORGE_EPI_RESID_TP;
        g.tpf = forge_tp_fused_dev(h->ar);
        if (forge_gemv_launch(g, h->stream, pdl)) return -1;
    } else {
        if (forge_gemv_launch(g, h->stream, pdl) || tp_sum(h, x, B, next_gain)) return -1;
    }
    if (next_gain && pq_x_on(h, B) && !pq_by_ar(h, B))
        return forge_stage_groups_launch(x, h->d, h->d, B, h->pq_x, next_gain, h->pq_ssq, h->stream, pdl);
    return 0;
}
// An RMSNorm GEMV reads x as staged after the kernel that wrote it.
void take_x_handoff(const ForgeB200* h, ForgeGemvArgs& g, int B) {
    if (pq_x_on(h, B)) {
        g.pq_in = h->pq_x;
        g.pq_ssq = h->pq_ssq;
    }
}

// Next node's slot of the multi-kernel step timeline (or null).
unsigned long long* trace_slot(ForgeB200* h) {
    if (!h->gtrace || h->gtrace_next >= h->gtrace_cap) return nullptr;
    return h->gtrace + (size_t)(h->gtrace_next++) * forge_sm_count() * 4;
}

// Prompt prefill: every row of a launch is one prompt position of one
// sequence (row -> position, row -> cache sequence), with its own split
// partials and merge counters; `exact` keeps hi/lo activations for bf16
// weights at any row count.
struct RowMap {
    const int32_t* pos;
    const int32_t* seq;
    float* partial;
    uint32_t* counters;
    bool exact;
};

// RMSNorm + QKV + RoPE, K/V appended at each sequence's position.
// handoff: the decode step's own chain, where x was staged after the
// previous layer's down projection.
int enqueue_qkv(ForgeB200* h, int l, int B, const float* x, float* q, bool pdl, const RowMap* rm = nullptr,
                bool handoff = false) {
    const LayerDev& Ld = h->layers[l];
    ForgeGemvArgs g = gemv_base(h, B);
    if (rm && rm->exact) g.split = 1;
    g.w = Ld.qkv_w; g.s = Ld.qkv_s; g.N = h->nqkv; g.K = h->d;
    g.x = x; g.x_stride = h->d; g.pro = FORGE_PRO_RMSNORM; g.gain = Ld.g1; g.eps = h->desc.rms_eps;
    g.epi = FORGE_EPI_QKV; g.q_out = q; g.kc = h->kc + (size_t)l * h->kv_layer; g.vc = h->vc + (size_t)l * h->kv_layer;
    g.pos = h->pos; g.H = h->H; g.Hkv = h->Hkv; g.hd = h->hd; g.lmax = h->lmax;
    g.rope_cos = h->rope_cos; g.rope_sin = h->rope_sin;
    g.trace = trace_slot(h);
    if (rm) {
        g.pos = rm->pos;
        g.seq_of = rm->seq;
    }
    if (handoff && !rm && l > 0) take_x_handoff(h, g, B);
    return forge_gemv_launch(g, h->stream, pdl);
}

// Whether the decode step at batch B hands the staged context from the
// flash-decode merge to the O projection.
bool pq_ctx_on(const ForgeB200* h, int B) { return h->prequant && B <= 4 && h->hd == 128 && !h->flat_attn; }

// Split-K flash-decode over positions 0..pos of every sequence.
// handoff: the decode step's own chain (attention then O projection of the
// same context); block-level callers pass their own context to the O
// projection, so they never take it.
int enqueue_attn(ForgeB200* h, int l, int B, const float* q, float* ctx, bool pdl, const RowMap* rm = nullptr,
                 bool handoff = false) {
    ForgeAttnArgs at{};
    at.q = q; at.kc = h->kc + (size_t)l * h->kv_layer; at.vc = h->vc + (size_t)l * h->kv_layer; at.pos = h->pos;
    at.B = B; at.H = h->H; at.Hkv = h->Hkv; at.hd = h->hd; at.lmax = h->lmax;
    at.partial = h->partial; at.counters = h->counters; at.out = ctx; at.err = h->err;
    at.trace = trace_slot(h);
    at.trace_ctas = forge_sm_count();
    if (rm) {
        // every cached row of a prompt row was written by this pass's QKV
        // kernel: no copies before the dependency, so no programmatic launch
        at.pos = rm->pos; at.seq_of = rm->seq; at.partial = rm->partial; at.counters = rm->counters;
        at.nsplit = forge_attn_pick_splits(B, h->Hkv, h->lmax);
        return forge_attn_launch(at, h->stream, false);
    }
    if (h->flat_attn && forge_attn_flat_supported(B, h->H, h->Hkv, h->hd)) {
        at.flat_slots = forge_attn_flat_slots(h->hd, h->lmax);
        return forge_attn_flat_launch(at, h->stream, pdl);
    }
    if (handoff && pq_ctx_on(h, B)) at.pq_out = h->pq_ctx;
    at.nsplit = forge_attn_pick_splits(B, h->Hkv, h->lmax);
    return forge_attn_launch(at, h->stream, pdl);
}

// x += Wo ctx
int enqueue_oproj(ForgeB200* h, int l, int B, const float* ctx, float* x, bool pdl, const RowMap* rm = nullptr,
                  bool handoff = false) {
    const LayerDev& Ld = h->layers[l];
    ForgeGemvArgs g = gemv_base(h, B);
    if (rm && rm->exact) g.split = 1;
    g.w = Ld.o_w; g.s = Ld.o_s; g.N = h->d; g.K = h->qd; g.x = ctx; g.x_stride = h->qd;
    g.pro = FORGE_PRO_PLAIN; g.epi = resid_epi(h); g.y = x; g.y_stride = h->d;
    g.trace = trace_slot(h);
    if (handoff && !rm && pq_ctx_on(h, B)) g.pq_in = h->pq_ctx;
    return resid_gemv(h, g, x, B, pdl, handoff && !rm ? Ld.g2 : nullptr);
}

// x += Wd (silu(Wg n) * (Wu n)), n = RMSNorm(x) * g2
// handoff: the decode step's own chain (gate/up reads x as staged after the
// O projection; s is staged for the down projection; x is staged after it
// for the next layer's QKV).
int enqueue_mlp(ForgeB200* h, int l, int B, float* x, bool pdl, const RowMap* rm = nullptr, float* s = nullptr,
                bool handoff = false) {
    const LayerDev& Ld = h->layers[l];
    const bool exact = rm && rm->exact;
    if (!s) s = h->s;
    ForgeGemvArgs g = gemv_base(h, B);
    if (exact) g.split = 1;
    g.w = Ld.gu_w; g.s = Ld.gu_s; g.N = 2 * h->F; g.K = h->d; g.x = x; g.x_stride = h->d;
    g.pro = FORGE_PRO_RMSNORM; g.gain = Ld.g2; g.eps = h->desc.rms_eps;
    g.epi = FORGE_EPI_SWIGLU; g.s_out = s; g.F = h->F;
    g.trace = trace_slot(h);
    if (handoff && !rm) take_x_handoff(h, g, B);
    if (forge_gemv_launch(g, h->stream, pdl)) return -1;
    g = gemv_base(h, B);
    if (exact) g.split = 1;
    g.w = Ld.dn_w; g.s = Ld.dn_s; g.N = h->d; g.K = h->F; g.x = s; g.x_stride = h->F;
    g.pro = FORGE_PRO_PLAIN; g.epi = resid_epi(h); g.y = x; g.y_stride = h->d;
    if (handoff && !rm && h->pq_s_on && B <= 4 && forge_gemv_launch_count(h->F, B, g.split, true, false) == 1) {
        if (forge_stage_groups_launch(s, h->F, h->F, B, h->pq_s, nullptr, nullptr, h->stream, pdl)) return -1;
        g.pq_in = h->pq_s;
    }
    g.trace = trace_slot(h);
    return resid_gemv(h, g, x, B, pdl, handoff && !rm && l + 1 < h->L ? h->layers[l + 1].g1 : nullptr);
}

// final RMSNorm + LM head into the handle's logits, argmax keys updated
int enqueue_head(ForgeB200* h, int B, const float* x, bool pdl, int x_stride = 0) {
    ForgeGemvArgs g = gemv_base(h, B);
    g.wkind = FORGE_W_BF16;
    g.w = h->head_w; g.s = nullptr; g.N = h->Vpad; g.K = h->d; g.x = x; g.x_stride = x_stride ? x_stride : h->d;
    g.pro = FORGE_PRO_RMSNORM; g.gain = h->gF; g.eps = h->desc.rms_eps;
    g.epi = FORGE_EPI_LOGITS; g.y = h->logits; g.y_stride = h->Vpad; g.argmax_key = h->amax; g.nvalid = h->V;
    g.row_off = h->v0;
    g.trace = trace_slot(h);
    if (forge_gemv_launch(g, h->stream, pdl)) return -1;
    return h->comm ? forge_tp_allreduce_max_u64(h->comm, h->amax, (size_t)B, h->stream) : 0;
}

int enqueue_step(ForgeB200* h, int B) {
    cudaStream_t st = h->stream;
    if (forge_embed_launch(h->emb, h->d, h->Vfull, h->tok, B, h->x, h->err, st, false)) return -1;
    for (int l = 0; l < h->L; ++l) {
        if (enqueue_qkv(h, l, B, h->x, h->q, true, nullptr, true) ||
            enqueue_attn(h, l, B, h->q, h->ctx, true, nullptr, true) ||
            enqueue_oproj(h, l, B, h->ctx, h->x, true, nullptr, true) ||
            enqueue_mlp(h, l, B, h->x, true, nullptr, nullptr, true))
            return -1;
    }
    if (enqueue_head(h, B, h->x, true)) return -1;
    return forge_argmax_finalize_launch(h->amax, B, h->tok, h->hist, h->step, h->pos, h->hist_cap, st, true);
}

// Context splits per (sequence, KV head) for the fused step: CTA work items
// are spread over the SMs in as few, as full waves as possible, with at least
// ~64 keys per item at full context (4 per consumer warp).
int fused_splits(const ForgeB200* h, int B) {
    const int grid = forge_sm_count();
    const int pairs = B * h->Hkv;
    int cap = h->lmax / 64;
    if (cap < 1) cap = 1;
    int best = 1;
    double best_score = -1e9;
    for (int ns = 1; ns <= cap; ++ns) {
        const int items = pairs * ns;
        const int waves = (items + grid - 1) / grid;
        const double eff = (double)items / ((double)waves * grid);
        const double score = eff - 0.02 * waves;
        if (score > best_score + 1e-9) { best_score = score; best = ns; }
    }
    return best;
}

// Builds (once per batch size) the phase list of the fused step and checks
// that it fits one CTA per SM. Returns the args or nullptr.
const ForgeStepArgs* fused_for(ForgeB200* h, int B) {
    if (h->force_graph || h->tp_size > 1) return nullptr;
    // one mma column block per GEMV: int4 (hi/lo int8) and exact bf16 use two
    // columns per sequence, plain bf16 one
    if ((h->q4 || h->split_for(B)) ? B > 4 : B > 8) return nullptr;
    auto ok = h->fused_ok.find(B);
    if (ok != h->fused_ok.end() && !ok->second) return nullptr;
    auto it = h->fused.find(B);
    if (it != h->fused.end()) return &it->second;
    const bool split = h->split_for(B);
    std::vector<ForgePhase> ph;
    ForgeGemvArgs a{};
    a.wkind = h->q4 ? FORGE_W_Q4 : FORGE_W_BF16;
    a.batch = B; a.split = split; a.err = h->err; a.eps = h->desc.rms_eps;
    a.H = h->H; a.Hkv = h->Hkv; a.hd = h->hd; a.lmax = h->lmax; a.pos = h->pos;
    a.rope_cos = h->rope_cos; a.rope_sin = h->rope_sin; a.emb = h->emb; a.emb_tok = h->tok;
    int kmax = 0;
    for (int l = 0; l < h->L; ++l) {
        const LayerDev& Ld = h->layers[l];
        uint16_t* kc = h->kc + (size_t)l * h->kv_layer;
        uint16_t* vc = h->vc + (size_t)l * h->kv_layer;
        ForgePhase p{};
        p.type = FORGE_PH_GEMV; p.g = a;
        p.g.w = Ld.qkv_w; p.g.s = Ld.qkv_s; p.g.N = h->nqkv; p.g.K = h->d; p.g.x = h->x; p.g.x_stride = h->d;
        p.g.pro = l == 0 ? FORGE_PRO_EMBED_RMSNORM : FORGE_PRO_RMSNORM; p.g.gain = Ld.g1;
        p.g.epi = FORGE_EPI_QKV; p.g.q_out = h->q; p.g.kc = kc; p.g.vc = vc; p.g.y = h->x; p.g.y_stride = h->d;
        ph.push_back(p);
        ForgePhase at{};
        at.type = FORGE_PH_ATTN; at.g = a; at.g.kc = kc; at.g.vc = vc;
        ph.push_back(at);
        p = ForgePhase{}; p.type = FORGE_PH_GEMV; p.g = a;
        p.g.w = Ld.o_w; p.g.s = Ld.o_s; p.g.N = h->d; p.g.K = h->qd; p.g.x = h->ctx; p.g.x_stride = h->qd;
        p.g.pro = FORGE_PRO_PLAIN; p.g.epi = FORGE_EPI_RESID; p.g.y = h->x; p.g.y_stride = h->d;
        ph.push_back(p);
        p = ForgePhase{}; p.type = FORGE_PH_GEMV; p.g = a;
        p.g.w = Ld.gu_w; p.g.s = Ld.gu_s; p.g.N = 2 * h->F; p.g.K = h->d; p.g.x = h->x; p.g.x_stride = h->d;
        p.g.pro = FORGE_PRO_RMSNORM; p.g.gain = Ld.g2; p.g.epi = FORGE_EPI_SWIGLU; p.g.s_out = h->s; p.g.F = h->F;
        ph.push_back(p);
        p = ForgePhase{}; p.type = FORGE_PH_GEMV; p.g = a;
        p.g.w = Ld.dn_w; p.g.s = Ld.dn_s; p.g.N = h->d; p.g.K = h->F; p.g.x = h->s; p.g.x_stride = h->F;
        p.g.pro = FORGE_PRO_PLAIN; p.g.epi = FORGE_EPI_RESID; p.g.y = h->x; p.g.y_stride = h->d;
        ph.push_back(p);
    }
    ForgePhase hp{};
    hp.type = FORGE_PH_GEMV; hp.g = a; hp.g.wkind = FORGE_W_BF16;
    hp.g.w = h->head_w; hp.g.s = nullptr; hp.g.N = h->Vpad; hp.g.K = h->d; hp.g.x = h->x; hp.g.x_stride = h->d;
    hp.g.pro = FORGE_PRO_RMSNORM; hp.g.gain = h->gF; hp.g.epi = FORGE_EPI_LOGITS; hp.g.y = h->logits;
    hp.g.y_stride = h->Vpad; hp.g.argmax_key = h->amax; hp.g.nvalid = h->V;
    ph.push_back(hp);
    ForgePhase fin{};
    fin.type = FORGE_PH_FIN;
    ph.push_back(fin);
    int xf_bytes = 0;
    for (const auto& p : ph)
        if (p.type == FORGE_PH_GEMV) {
            kmax = std::max(kmax, p.g.K);
            const int need = p.g.wkind == FORGE_W_Q4 ? 2 * B * p.g.K
                                                     : (split ? 2 * B : B) * ((p.g.K + 31) / 32) * 32 * 2;
            xf_bytes = std::max(xf_bytes, need);
        }
    ForgeStepArgs sa{};
    sa.nphases = (int)ph.size();
    sa.grid = forge_sm_count();
    sa.B = B; sa.H = h->H; sa.Hkv = h->Hkv; sa.hd = h->hd; sa.lmax = h->lmax; sa.nsplit = fused_splits(h, B);
    sa.q = h->q; sa.ctx = h->ctx; sa.pos = h->pos; sa.partial = h->partial; sa.counters = h->counters;
    sa.amax = h->amax; sa.tok = h->tok; sa.hist = h->hist; sa.step = h->step; sa.hist_cap = h->hist_cap;
    sa.bar = h->bar; sa.epoch = h->epoch; sa.err = h->err;
    if (getenv("FORGE_STEP_TRACE")) {
        sa.trace = (unsigned long long*)h->alloc(sizeof(unsigned long long) * 4 * ph.size() * sa.grid);
        if (sa.trace) cudaMemset(sa.trace, 0, sizeof(unsigned long long) * 4 * ph.size() * sa.grid);
        h->trace = sa.trace;
        h->trace_n = (int)ph.size();
    }
    const bool need_q4_fit = h->q4 && kmax / 128 > 128;
    int fits = need_q4_fit ? 1 : forge_step_launch(sa, xf_bytes, h->stream, true);
    if (fits != 0) {
        if (getenv("FORGE_VERBOSE")) fprintf(stderr, "[forge_b200] batch %d: fused step does not fit, using the multi-kernel graph\n", B);
        h->fused_ok[B] = 0;
        return nullptr;
    }
    ForgePhase* dph = (ForgePhase*)h->alloc(sizeof(ForgePhase) * ph.size());
    if (!dph || cudaMemcpy(dph, ph.data(), sizeof(ForgePhase) * ph.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
        h->fused_ok[B] = 0;
        return nullptr;
    }
    sa.phases = dph;
    sa.stages = xf_bytes;  // carried to the launcher (which picks the stage count)
    h->fused_ok[B] = 1;
    h->fused[B] = sa;
    return &h->fused[B];
}

int launch_fused(ForgeB200* h, const ForgeStepArgs* sa) {
    return forge_step_launch(*sa, sa->stages, h->stream, false) ? -1 : 0;
}

cudaGraphExec_t graph_for(ForgeB200* h, int B) {
    auto it = h->graphs.find(B);
    if (it != h->graphs.end()) return it->second;
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        forge_fail(-1, "forge_b200: begin capture failed");
        return nullptr;
    }
    h->gtrace_next = 0;
    int rc = enqueue_step(h, B);
    if (h->gtrace) {
        h->trace = h->gtrace;
        h->trace_n = h->gtrace_next;
    }
    cudaError_t e = cudaStreamEndCapture(h->stream, &graph);
    if (rc || e != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        forge_fail(-1, "forge_b200: step capture failed (%s)", cudaGetErrorString(e));
        return nullptr;
    }
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) {
        forge_fail(-1, "forge_b200: graph instantiate: %s", cudaGetErrorString(e));
        return nullptr;
    }
    h->graphs[B] = exec;
    return exec;
}

int check_ready(ForgeB200* h, int B) {
    if (!h) return forge_fail(FORGE_INVALID_ARGS, "forge_b200: null handle");
    if (!h->weights_ready) return forge_fail(FORGE_INVALID_ARGS, "forge_b200: weights not loaded");
    if (B <= 0 || B > h->Bmax) return forge_fail(FORGE_INVALID_ARGS, "forge_b200: batch %d outside 1..%d", B, h->Bmax);
    return cudaSetDevice(h->device) == cudaSuccess ? 0 : forge_fail(-1, "forge_b200: cudaSetDevice failed");
}

int read_err(ForgeB200* h) {
    uint32_t e = 0;
    if (cudaMemcpy(&e, h->err, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return forge_fail(-1, "forge_b200: device error: %s", cudaGetErrorString(cudaGetLastError()));
    if (e) {
        cudaMemset(h->err, 0, 4);
        return forge_fail(-1, "forge_b200: kernel raised error word 0x%x (1 wait timeout, 2 flag timeout, 4 bad index)", e);
    }
    return 0;
}
}  // namespace

int forge_embed_launch(const uint16_t* emb, int d, int vocab, const int32_t* tok, int B, float* x,
                       uint32_t* err, cudaStream_t stream, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(B);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_embed, emb, d, vocab, tok, x, err);
    return e == cudaSuccess ? 0 : forge_fail(-1, "embed launch: %s", cudaGetErrorString(e));
}

int forge_argmax_finalize_launch(unsigned long long* keys, int B, int32_t* tok_out, int32_t* hist,
                                 int32_t* step_counter, int32_t* pos, int hist_cap, cudaStream_t stream,
                                 bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3((B + 31) / 32 * 32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    // hist rows are [hist_cap][B_max]; the stride is passed through hist_cap's owner
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_finalize, keys, B, tok_out, hist, step_counter, pos, hist_cap, B);
    return e == cudaSuccess ? 0 : forge_fail(-1, "finalize launch: %s", cudaGetErrorString(e));
}

extern "C" {
namespace {
int create_impl(const ForgeModelDesc* desc, int device, const void* nccl_id, ForgeB200** out) {
    if (!desc || !out) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: null argument");
    *out = nullptr;
    const ForgeModelDesc& m = *desc;
    if (m.n_layer <= 0 || m.d_model <= 0 || m.n_head <= 0 || m.n_kv_head <= 0 || m.head_dim <= 0 ||
        m.ffn <= 0 || m.vocab <= 0 || m.max_batch <= 0 || m.max_ctx <= 0)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: non-positive dimension");
    if (m.n_head % m.n_kv_head) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: n_head %% n_kv_head != 0");
    if (m.head_dim != 64 && m.head_dim != 128)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: head_dim must be 64 or 128");
    if (m.d_model % 64 || m.ffn % 16) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: d %% 64, ffn %% 16 required");
    if (m.weight_kind == FORGE_WEIGHT_Q4_G128 && (m.d_model % 128 || m.ffn % 128 || (m.n_head * m.head_dim) % 128))
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: int4 group-128 needs every K %% 128 == 0");
    if (m.weight_kind != FORGE_WEIGHT_BF16 && m.weight_kind != FORGE_WEIGHT_Q4_G128)
        return forge_fail(FORGE_PRECISION_UNSUPPORTED, "forge_b200_create: unknown weight kind %d", m.weight_kind);
    const int T = m.tp_size > 0 ? m.tp_size : 1, R = m.tp_size > 0 ? m.tp_rank : 0;
    if (R < 0 || R >= T) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: tp_rank %d outside 0..%d", R, T - 1);
    if (m.n_head % T || m.n_kv_head % T)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: %d / %d heads do not split over %d ranks", m.n_head,
                          m.n_kv_head, T);
    if ((int64_t)m.n_head / T * m.head_dim % 128 && m.weight_kind == FORGE_WEIGHT_Q4_G128)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: a rank's O-projection K must be a multiple of 128");
    int64_t f_off = 0, f_len = m.ffn;
    if (T > 1 && forge_tp_split(m.ffn, m.weight_kind == FORGE_WEIGHT_Q4_G128 ? 128 : 16, R, T, &f_off, &f_len))
        return FORGE_INVALID_ARGS;
    if (m.max_batch > 1024) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: max_batch <= 1024");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: no CUDA device %d", device);
    if (cudaSetDevice(device) != cudaSuccess) return forge_fail(-1, "forge_b200_create: cudaSetDevice failed");
    cudaDeviceProp prop{};
    cudaGetDeviceProperties(&prop, device);
    if (prop.major != 10) return forge_fail(FORGE_KERNEL_UNSUPPORTED, "forge_b200_create: needs an sm_100 device (got sm_%d%d)", prop.major, prop.minor);

    if (forge_gemv_configure() || forge_gemv_b_configure() || forge_attn_configure() || forge_attn_flat_configure())
        return -1;
    forge_sm_count();
    ForgeB200* h = new ForgeB200();
    h->desc = m;
    h->device = device;
    h->L = m.n_layer; h->d = m.d_model; h->hd = m.head_dim;
    h->tp_rank = R; h->tp_size = T;
    h->Hfull = m.n_head; h->Hkvfull = m.n_kv_head; h->Ffull = m.ffn; h->Vfull = m.vocab;
    h->H = m.n_head / T; h->Hkv = m.n_kv_head / T; h->h0 = R * h->H; h->kv0 = R * h->Hkv;
    h->F = (int)f_len; h->f0 = (int)f_off;
    {
        // equal vocabulary slices of whole 16-row tiles (all-gather needs equal counts)
        const int vs = (int)round_up((m.vocab + T - 1) / T, 16);
        h->Vpad = vs;
        h->v0 = R * vs;
        h->V = std::max(0, std::min(vs, m.vocab - h->v0));
    }
    h->qd = h->H * h->hd; h->kvd = h->Hkv * h->hd; h->nqkv = h->qd + 2 * h->kvd;
    h->Bmax = m.max_batch; h->lmax = m.max_ctx; h->q4 = m.weight_kind == FORGE_WEIGHT_Q4_G128;
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete h;
        return forge_fail(-1, "forge_b200_create: stream creation failed");
    }
    h->layers.resize(h->L);
    int rc = 0;
    for (auto& Ld : h->layers) rc |= alloc_layer(h, Ld);
    const size_t d = h->d;
    h->emb = (uint16_t*)h->alloc((size_t)h->Vfull * d * 2);
    if (T > 1) h->logits_all = (float*)h->alloc(sizeof(float) * (size_t)T * h->Bmax * h->Vpad);
    h->head_w = h->alloc((size_t)h->Vpad * d * 2);
    h->gF = (float*)h->alloc(sizeof(float) * d);
    h->kv_layer = (size_t)h->Bmax * h->Hkv * h->lmax * h->hd;
    h->kc = (uint16_t*)h->alloc(h->kv_layer * h->L * 2);
    h->vc = (uint16_t*)h->alloc(h->kv_layer * h->L * 2);
    h->rope_cos = (float*)h->alloc(sizeof(float) * (size_t)h->lmax * h->hd / 2);
    h->rope_sin = (float*)h->alloc(sizeof(float) * (size_t)h->lmax * h->hd / 2);
    h->tok = (int32_t*)h->alloc(4 * h->Bmax);
    h->pos = (int32_t*)h->alloc(4 * h->Bmax);
    h->hist_cap = h->lmax + 1;
    h->hist = (int32_t*)h->alloc((size_t)4 * h->Bmax * h->hist_cap);
    h->step = (int32_t*)h->alloc(16);
    h->x = (float*)h->alloc(sizeof(float) * h->Bmax * d);
    h->q = (float*)h->alloc(sizeof(float) * h->Bmax * h->qd);
    h->ctx = (float*)h->alloc(sizeof(float) * h->Bmax * h->qd);
    h->s = (float*)h->alloc(sizeof(float) * (size_t)h->Bmax * h->F);
    h->logits = (float*)h->alloc(sizeof(float) * (size_t)h->Bmax * h->Vpad);
    h->amax = (unsigned long long*)h->alloc(8 * h->Bmax);
    int max_split = 1;
    for (int B = 1; B <= h->Bmax; ++B) {
        int ns = forge_attn_pick_splits(B, h->Hkv, h->lmax);
        if (ns * B > max_split) max_split = ns * B;
    }
    for (int B = 1; B <= h->Bmax; ++B) {
        int ns = fused_splits(h, B);
        if (ns * B > max_split) max_split = ns * B;
    }
    size_t partial_floats = (size_t)max_split * h->H * (h->hd + 2);
    {
        // FORGE_ATTN=flat: the flat small-batch flash-decode (attn_flat.cu) for up to 32
        // sequences; by default the per-(sequence, head, split) kernel, which is faster
        // at batch 1 as measured so far
        const char* e = getenv("FORGE_ATTN");
        h->flat_attn = e && strcmp(e, "flat") == 0;
        for (int B = 1; B <= h->Bmax; ++B)
            if (h->flat_attn && forge_attn_flat_supported(B, h->H, h->Hkv, h->hd))
                partial_floats = std::max(partial_floats, (size_t)forge_attn_flat_partial_floats(B, h->H, h->hd, h->lmax));
    }
    h->partial = (float*)h->alloc(sizeof(float) * partial_floats);
    {
        const char* e = getenv("FORGE_PREQUANT");
        h->prequant = h->q4 && !(e && strcmp(e, "0") == 0);
        if (h->prequant) {
            h->pq_ctx = (uint8_t*)h->alloc((size_t)forge_pq_bytes(h->qd, 4));
            if (!h->pq_ctx) h->prequant = false;
            const char* es = getenv("FORGE_PREQUANT_S");
            if (h->prequant && !(es && strcmp(es, "0") == 0) && h->F % 128 == 0) {
                h->pq_s = (uint8_t*)h->alloc((size_t)forge_pq_bytes(h->F, 4));
                h->pq_s_on = h->pq_s != nullptr;
            }
            const char* en = getenv("FORGE_PREQUANT_NORM");
            if (h->prequant && !(en && strcmp(en, "0") == 0)) {
                h->pq_x = (uint8_t*)h->alloc((size_t)forge_pq_bytes(h->d, 4));
                h->pq_ssq = (float*)h->alloc(sizeof(float) * 4 * (h->d / 128));
                h->pq_norm = h->pq_x && h->pq_ssq;
            }
        }
    }
    h->bar = (unsigned long long*)h->alloc(16);
    h->epoch = (uint32_t*)h->alloc(16);
    {
        // default: captured multi-kernel graph; FORGE_DECODE_PATH=fused selects
        // the persistent single-kernel step
        const char* e = getenv("FORGE_DECODE_PATH");
        h->force_graph = (e && strcmp(e, "fused") == 0) ? 0 : 1;
    }
    h->counters = (uint32_t*)h->alloc(4 * (size_t)h->Bmax * h->Hkv);
    if (getenv("FORGE_GRAPH_TRACE")) {
        h->gtrace_cap = 5 * h->L + 2;
        const size_t n = (size_t)h->gtrace_cap * forge_sm_count() * 4;
        h->gtrace = (unsigned long long*)h->alloc(8 * n);
        if (h->gtrace) cudaMemset(h->gtrace, 0, 8 * n);
    }
    h->err = (uint32_t*)h->alloc(16);
    if (h->Bmax > 4) {  // batched GEMV path (int4 above 4 sequences, bf16 above 8); starts zeroed
        const size_t nb = (size_t)forge_gemv_b_scratch_bytes(std::max({h->d, h->qd, h->F}));
        h->bscratch = h->alloc(nb);
        if (h->bscratch && cudaMemset(h->bscratch, 0, nb) != cudaSuccess) h->bscratch = nullptr;
    }
    size_t st = std::max({(size_t)h->nqkv * d, (size_t)2 * h->F * d, (size_t)d * h->F, (size_t)d * h->qd,
                          (size_t)h->Vpad * d});
    h->stA = (uint16_t*)h->alloc(st * 2);
    h->stB = (uint16_t*)h->alloc(st * 2);
    h->codes = (uint8_t*)h->alloc(st / 2);
    h->scales = (uint16_t*)h->alloc(st / 128 * 2 + 16);
    if (rc || !h->emb || !h->head_w || !h->kc || !h->vc || !h->stA || !h->stB || !h->codes || !h->partial ||
        !h->hist || !h->logits || !h->scales || !h->bar || !h->epoch) {
        forge_b200_destroy(h);
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create: out of device memory");
    }
    if (cudaHostAlloc((void**)&h->h_tok, 4 * h->Bmax, cudaHostAllocDefault) != cudaSuccess) h->h_tok = nullptr;
    // RoPE tables in double (nn_lib.hexa:509-531), stored fp32 [lmax][hd/2];
    // rope_theta <= 0 turns the rotation off (cos 1, sin 0), the form of the
    // reference's single-layer decode check (tool/decode_eager_baseline.cu)
    if (m.rope_theta <= 0.f) {
        const size_t n = (size_t)h->lmax * (h->hd / 2);
        std::vector<float> c(n, 1.0f), s(n, 0.0f);
        cudaMemcpy(h->rope_cos, c.data(), n * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(h->rope_sin, s.data(), n * 4, cudaMemcpyHostToDevice);
    } else {
        const int half = h->hd / 2;
        std::vector<float> c((size_t)h->lmax * half), s((size_t)h->lmax * half);
        const double lnb = std::log((double)m.rope_theta);
        for (int p = 0; p < h->lmax; ++p)
            for (int i = 0; i < half; ++i) {
                const double ex = ((double)(2 * i) / (double)h->hd) * lnb;
                const double invf = 1.0 / std::exp(ex);
                const double ang = (double)p * invf;
                c[(size_t)p * half + i] = (float)std::cos(ang);
                s[(size_t)p * half + i] = (float)std::sin(ang);
            }
        cudaMemcpy(h->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(h->rope_sin, s.data(), s.size() * 4, cudaMemcpyHostToDevice);
    }
    cudaMemset(h->counters, 0, 4 * (size_t)h->Bmax * h->Hkv);
    cudaMemset(h->bar, 0, 16);
    cudaMemset(h->epoch, 0, 16);
    cudaMemset(h->amax, 0, 8 * h->Bmax);
    cudaMemset(h->err, 0, 16);
    cudaMemset(h->step, 0, 16);
    cudaMemset(h->pos, 0, 4 * h->Bmax);
    cudaMemset(h->tok, 0, 4 * h->Bmax);
    cudaMemset(h->kc, 0, h->kv_layer * h->L * 2);
    cudaMemset(h->vc, 0, h->kv_layer * h->L * 2);
    if (cudaDeviceSynchronize() != cudaSuccess) {
        forge_b200_destroy(h);
        return forge_fail(-1, "forge_b200_create: device initialisation failed");
    }
    if (T > 1 && (!h->logits_all || forge_tp_comm_init(&h->comm, nccl_id, R, T))) {
        forge_b200_destroy(h);
        return -1;
    }
    if (T > 1) {
        // residual all-reduces through peer memory unless FORGE_TP_ALLREDUCE=nccl
        const char* e = getenv("FORGE_TP_ALLREDUCE");
        if (!(e && strcmp(e, "nccl") == 0) && forge_tp_ar_init(h->comm, R, T, h->Bmax * h->d, h->stream, &h->ar)) {
            forge_b200_destroy(h);
            return -1;
        }
    }
    *out = h;
    return 0;
}
}  // namespace

FORGE_API int forge_b200_create(const ForgeModelDesc* desc, int device, ForgeB200** out) {
    if (desc && desc->tp_size > 1)
        return forge_fail(FORGE_REGIME_UNSUPPORTED, "forge_b200_create: tensor parallel handles use forge_b200_create_tp");
    return create_impl(desc, device, nullptr, out);
}

FORGE_API int forge_b200_create_tp(const ForgeModelDesc* desc, int device, const void* nccl_unique_id,
                                   ForgeB200** out) {
    if (!desc || !nccl_unique_id || desc->tp_size < 1)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create_tp: bad args");
    if (desc->tp_rank < 0 || desc->tp_rank >= desc->tp_size)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create_tp: rank %d outside 0..%d", desc->tp_rank,
                          desc->tp_size - 1);
    // an id that forge_b200_tp_unique_id never wrote (all zero bytes) would
    // leave every rank waiting in NCCL's bootstrap: refuse it up front
    const unsigned char* idb = static_cast<const unsigned char*>(nccl_unique_id);
    bool any = false;
    for (int i = 0; i < 128; ++i) any |= idb[i] != 0;
    if (desc->tp_size > 1 && !any)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create_tp: empty NCCL unique id (all zero bytes)");
    return create_impl(desc, device, nccl_unique_id, out);
}

FORGE_API void forge_b200_destroy(ForgeB200* h) {
    if (!h) return;
    cudaSetDevice(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    for (auto& kv : h->graphs) cudaGraphExecDestroy(kv.second);
    h->graphs.clear();
    if (h->ar) forge_tp_ar_destroy(h->ar);
    if (h->comm) forge_tp_comm_destroy(h->comm);  // after the graphs that hold its collectives
    for (void* p : h->allocs) cudaFree(p);
    for (void* p : {(void*)h->pre.x, (void*)h->pre.q, (void*)h->pre.ctx, (void*)h->pre.s, (void*)h->pre.partial,
                    (void*)h->pre.tok, (void*)h->pre.pos, (void*)h->pre.seq, (void*)h->pre.sel, (void*)h->pre.counters,
                    (void*)h->pre.qb, (void*)h->pre.ob})
        if (p) cudaFree(p);
    if (h->h_tok) cudaFreeHost(h->h_tok);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
}

FORGE_API void* forge_b200_stream(ForgeB200* h) { return h ? (void*)h->stream : nullptr; }

const ForgeModelDesc* forge_b200_desc_of(const ForgeB200* h) { return h ? &h->desc : nullptr; }

FORGE_API int forge_b200_load_layer(ForgeB200* h, int layer, const ForgeLayerWeights* w) {
    if (!h || !w || layer < 0 || layer >= h->L) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_load_layer: bad args");
    if (!w->wq || !w->wk || !w->wv || !w->wo || !w->wg || !w->wu || !w->wd || !w->g1 || !w->g2)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_load_layer: null weight pointer");
    cudaSetDevice(h->device);
    Src src[7];
    const uint16_t* ptrs[7] = {w->wq, w->wk, w->wv, w->wo, w->wg, w->wu, w->wd};
    for (int i = 0; i < 7; ++i) src[i] = Src{ptrs[i], 0, 0, 0.f};
    return load_layer_impl(h, layer, src, w->g1, w->g2, false) ? FORGE_INVALID_ARGS : 0;
}

FORGE_API int forge_b200_load_embedding(ForgeB200* h, const uint16_t* emb, const float* gF, const uint16_t* head) {
    if (!h || !emb || !gF) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_load_embedding: bad args");
    if (!h->desc.tied_head && !head) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_load_embedding: untied model needs a head");
    cudaSetDevice(h->device);
    Src e{emb, 0, 0, 0.f}, hd{head, 0, 0, 0.f};
    if (load_embed_impl(h, e, h->desc.tied_head ? nullptr : &hd, gF, false)) return FORGE_INVALID_ARGS;
    h->weights_ready = true;
    return 0;
}

FORGE_API int forge_b200_init_synthetic(ForgeB200* h, uint64_t seed, float std) {
    if (!h) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_init_synthetic: null handle");
    cudaSetDevice(h->device);
    for (int l = 0; l < h->L; ++l) {
        Src src[7];
        for (int i = 0; i < 7; ++i) src[i] = Src{nullptr, seed, (uint64_t)(2 + 7 * l + i) << 40, std};
        if (load_layer_impl(h, l, src, nullptr, nullptr, true)) return -1;
    }
    Src e{nullptr, seed, 0, std}, hd{nullptr, seed, (uint64_t)1 << 40, std};
    if (load_embed_impl(h, e, h->desc.tied_head ? nullptr : &hd, nullptr, true)) return -1;
    h->weights_ready = true;
    return 0;
}

/* The same with the std as a double, for FFIs that pass every float
 * argument as a double (hexa's @link extern fn). */
FORGE_API int forge_b200_get_desc(const ForgeB200* h, ForgeModelDesc* out) {
    if (!h || !out) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_get_desc: null argument");
    *out = h->desc;
    return 0;
}

FORGE_API int forge_b200_init_synthetic_d(ForgeB200* h, uint64_t seed, double std) {
    return forge_b200_init_synthetic(h, seed, (float)std);
}

FORGE_API int forge_b200_reset(ForgeB200* h) {
    if (!h) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_reset: null handle");
    cudaSetDevice(h->device);
    cudaMemsetAsync(h->pos, 0, 4 * h->Bmax, h->stream);
    cudaMemsetAsync(h->step, 0, 16, h->stream);
    cudaMemsetAsync(h->amax, 0, 8 * h->Bmax, h->stream);
    cudaMemsetAsync(h->bar, 0, 16, h->stream);
    cudaMemsetAsync(h->epoch, 0, 16, h->stream);
    cudaMemsetAsync(h->counters, 0, 4 * (size_t)h->Bmax * h->Hkv, h->stream);
    return cudaStreamSynchronize(h->stream) == cudaSuccess ? 0 : forge_fail(-1, "forge_b200_reset failed");
}

FORGE_API int forge_b200_fill_kv_synthetic(ForgeB200* h, uint64_t seed, int ctx_len, float std) {
    if (!h || ctx_len < 0 || ctx_len >= h->lmax) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_fill_kv_synthetic: bad args");
    cudaSetDevice(h->device);
    const int64_t n = (int64_t)h->kv_layer * h->L;
    if (forge_fill_normal_bf16(h->kc, n, seed, (uint64_t)1000 << 40, std, h->stream) ||
        forge_fill_normal_bf16(h->vc, n, seed, (uint64_t)1001 << 40, std, h->stream))
        return -1;
    k_set_i32<<<1, 256, 0, h->stream>>>(h->pos, h->Bmax, ctx_len);
    return cudaStreamSynchronize(h->stream) == cudaSuccess ? 0 : forge_fail(-1, "forge_b200_fill_kv_synthetic failed");
}

FORGE_API int forge_b200_set_positions(ForgeB200* h, const int32_t* pos, int batch) {
    if (!h || !pos || batch <= 0 || batch > h->Bmax) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_set_positions: bad args");
    for (int b = 0; b < batch; ++b)
        if (pos[b] < 0 || pos[b] >= h->lmax) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_set_positions: position out of range");
    cudaSetDevice(h->device);
    if (cudaMemcpy(h->pos, pos, 4 * batch, cudaMemcpyHostToDevice) != cudaSuccess) return forge_fail(-1, "H2D positions");
    return 0;
}

FORGE_API int forge_b200_get_kv(ForgeB200* h, int layer, int seq, uint16_t* k_out, uint16_t* v_out) {
    if (!h || layer < 0 || layer >= h->L || seq < 0 || seq >= h->Bmax || !k_out || !v_out)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_get_kv: bad args");
    cudaSetDevice(h->device);
    if (cudaStreamSynchronize(h->stream) != cudaSuccess) return forge_fail(-1, "forge_b200_get_kv: sync failed");
    const size_t per_seq = (size_t)h->Hkv * h->lmax * h->hd;
    const size_t off = (size_t)layer * h->kv_layer + (size_t)seq * per_seq;
    if (cudaMemcpy(k_out, h->kc + off, per_seq * 2, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(v_out, h->vc + off, per_seq * 2, cudaMemcpyDeviceToHost) != cudaSuccess)
        return forge_fail(-1, "forge_b200_get_kv: D2H failed");
    return 0;
}

FORGE_API int forge_b200_set_kv(ForgeB200* h, int layer, int seq, const uint16_t* k, const uint16_t* v, int n_pos) {
    if (!h || layer < 0 || layer >= h->L || seq < 0 || seq >= h->Bmax || !k || !v || n_pos < 0 || n_pos > h->lmax)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_set_kv: bad args");
    cudaSetDevice(h->device);
    if (cudaStreamSynchronize(h->stream) != cudaSuccess) return forge_fail(-1, "forge_b200_set_kv: sync failed");
    const size_t per_seq = (size_t)h->Hkv * h->lmax * h->hd;
    const size_t off = (size_t)layer * h->kv_layer + (size_t)seq * per_seq;
    const size_t row = (size_t)h->hd * 2, pitch = (size_t)h->lmax * row;
    // host [Hkv][n_pos][hd] -> cache [Hkv][lmax][hd]
    if (n_pos && (cudaMemcpy2D(h->kc + off, pitch, k, (size_t)n_pos * row, (size_t)n_pos * row, h->Hkv,
                               cudaMemcpyHostToDevice) != cudaSuccess ||
                  cudaMemcpy2D(h->vc + off, pitch, v, (size_t)n_pos * row, (size_t)n_pos * row, h->Hkv,
                               cudaMemcpyHostToDevice) != cudaSuccess))
        return forge_fail(-1, "forge_b200_set_kv: H2D failed");
    return 0;
}

FORGE_API int forge_b200_get_kv_rows(ForgeB200* h, int layer, int seq, uint16_t* k, uint16_t* v, int n_pos) {
    if (!h || layer < 0 || layer >= h->L || seq < 0 || seq >= h->Bmax || !k || !v || n_pos < 0 || n_pos > h->lmax)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_get_kv_rows: bad args");
    cudaSetDevice(h->device);
    if (cudaStreamSynchronize(h->stream) != cudaSuccess) return forge_fail(-1, "forge_b200_get_kv_rows: sync failed");
    const size_t per_seq = (size_t)h->Hkv * h->lmax * h->hd;
    const size_t off = (size_t)layer * h->kv_layer + (size_t)seq * per_seq;
    const size_t row = (size_t)h->hd * 2, pitch = (size_t)h->lmax * row;
    // cache [Hkv][lmax][hd] -> host [Hkv][n_pos][hd]
    if (n_pos && (cudaMemcpy2D(k, (size_t)n_pos * row, h->kc + off, pitch, (size_t)n_pos * row, h->Hkv,
                               cudaMemcpyDeviceToHost) != cudaSuccess ||
                  cudaMemcpy2D(v, (size_t)n_pos * row, h->vc + off, pitch, (size_t)n_pos * row, h->Hkv,
                               cudaMemcpyDeviceToHost) != cudaSuccess))
        return forge_fail(-1, "forge_b200_get_kv_rows: D2H failed");
    return 0;
}

// Enqueues one decode step: the fused persistent kernel when it fits, else
// the captured multi-kernel graph.
int enqueue_one(ForgeB200* h, int B) {
    if (const ForgeStepArgs* sa = fused_for(h, B)) return launch_fused(h, sa);
    cudaGraphExec_t g = graph_for(h, B);
    if (!g) return -1;
    return cudaGraphLaunch(g, h->stream) == cudaSuccess ? 0 : forge_fail(-1, "forge_b200: graph launch failed");
}

// Enqueues the copy of the last head's logits [batch][vocab] to the host
// (under tensor parallelism every rank holds one vocabulary slice: they are
// gathered first, and every rank calls this).
int enqueue_logits_copy(ForgeB200* h, int batch, float* logits) {
    if (!h->comm) {
        cudaMemcpy2DAsync(logits, sizeof(float) * h->V, h->logits, sizeof(float) * h->Vpad, sizeof(float) * h->V,
                          batch, cudaMemcpyDeviceToHost, h->stream);
        return 0;
    }
    const size_t per = (size_t)batch * h->Vpad;
    if (forge_tp_allgather_f32(h->comm, h->logits, h->logits_all, per, h->stream)) return -1;
    for (int r = 0; r < h->tp_size; ++r) {
        const int nv = std::max(0, std::min(h->Vpad, h->Vfull - r * h->Vpad));
        if (nv)
            cudaMemcpy2DAsync(logits + (size_t)r * h->Vpad, sizeof(float) * h->Vfull, h->logits_all + r * per,
                              sizeof(float) * h->Vpad, sizeof(float) * nv, batch, cudaMemcpyDeviceToHost, h->stream);
    }
    return 0;
}

FORGE_API int forge_b200_decode_step(ForgeB200* h, int batch, const int32_t* tokens, int32_t* next_tokens, float* logits) {
    if (int rc = check_ready(h, batch)) return rc;
    if (!tokens) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_decode_step: null tokens");
    int32_t* stage = h->h_tok;
    if (!stage) return forge_fail(-1, "forge_b200_decode_step: no pinned staging buffer");
    memcpy(stage, tokens, 4 * batch);
    cudaMemcpyAsync(h->tok, stage, 4 * batch, cudaMemcpyHostToDevice, h->stream);
    if (enqueue_one(h, batch)) return -1;
    if (next_tokens) cudaMemcpyAsync(stage, h->tok, 4 * batch, cudaMemcpyDeviceToHost, h->stream);
    if (logits && enqueue_logits_copy(h, batch, logits)) return -1;
    if (cudaStreamSynchronize(h->stream) != cudaSuccess)
        return forge_fail(-1, "forge_b200_decode_step: %s", cudaGetErrorString(cudaGetLastError()));
    if (next_tokens) memcpy(next_tokens, stage, 4 * batch);
    return read_err(h);
}

// One decode step whose next tokens are drawn by the reference sampler
// (self/ml/gpu_sampler.hexa:89-277) from the step's logits on the device;
// rng_state [batch] is read and advanced (host array).
FORGE_API int forge_b200_decode_step_sampled(ForgeB200* h, int batch, const int32_t* tokens, int32_t* next_tokens,
                                             double temperature, int top_k, double top_p, int64_t* rng_state) {
    if (int rc = check_ready(h, batch)) return rc;
    if (!tokens || !next_tokens || !rng_state)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_decode_step_sampled: null tokens or RNG state");
    if (h->comm)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_decode_step_sampled: not available under tensor parallelism");
    if (!h->samp_probs) {
        h->samp_probs = (float*)h->alloc(sizeof(float) * (size_t)h->Bmax * h->Vpad);
        h->samp_rng = (int64_t*)h->alloc(sizeof(int64_t) * (size_t)h->Bmax);
        if (!h->samp_probs || !h->samp_rng) return forge_fail(-1, "forge_b200_decode_step_sampled: allocation failed");
    }
    int32_t* stage = h->h_tok;
    if (!stage) return forge_fail(-1, "forge_b200_decode_step_sampled: no pinned staging buffer");
    memcpy(stage, tokens, 4 * batch);
    cudaMemcpyAsync(h->tok, stage, 4 * batch, cudaMemcpyHostToDevice, h->stream);
    cudaMemcpyAsync(h->samp_rng, rng_state, 8 * batch, cudaMemcpyHostToDevice, h->stream);
    if (enqueue_one(h, batch)) return -1;
    if (forge_sample_launch(h->logits, h->Vpad, batch, h->V, temperature, top_k, top_p, h->samp_rng, h->samp_probs,
                            h->Vpad, h->tok, h->stream))
        return -1;
    cudaMemcpyAsync(stage, h->tok, 4 * batch, cudaMemcpyDeviceToHost, h->stream);
    cudaMemcpyAsync(rng_state, h->samp_rng, 8 * batch, cudaMemcpyDeviceToHost, h->stream);
    if (cudaStreamSynchronize(h->stream) != cudaSuccess)
        return forge_fail(-1, "forge_b200_decode_step_sampled: %s", cudaGetErrorString(cudaGetLastError()));
    memcpy(next_tokens, stage, 4 * batch);
    return read_err(h);
}

namespace {
int64_t packed_i64(const void* args, int off) {
    int64_t v;
    memcpy(&v, static_cast<const char*>(args) + off, 8);
    return v;
}
double packed_f64(const void* args, int off) {
    double v;
    memcpy(&v, static_cast<const char*>(args) + off, 8);
    return v;
}
bool fits_i32(int64_t v) { return v >= INT32_MIN && v <= INT32_MAX; }
}  // namespace

FORGE_API int forge_b200_desc_from_packed(const void* args, ForgeModelDesc* d) {
    if (!args || !d) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_desc_from_packed: null argument");
    memset(d, 0, sizeof *d);
    int32_t* ints[] = {&d->n_layer, &d->d_model, &d->n_head, &d->n_kv_head, &d->head_dim, &d->ffn, &d->vocab};
    for (int i = 0; i < 7; ++i) {
        const int64_t v = packed_i64(args, 8 * i);
        if (!fits_i32(v)) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_desc_from_packed: field %d out of range", i);
        *ints[i] = (int32_t)v;
    }
    d->rms_eps = (float)packed_f64(args, 56);
    d->rope_theta = (float)packed_f64(args, 64);
    int32_t* rest[] = {&d->weight_kind, &d->tied_head, &d->max_batch, &d->max_ctx, &d->act_mode};
    for (int i = 0; i < 5; ++i) {
        const int64_t v = packed_i64(args, 72 + 8 * i);
        if (!fits_i32(v)) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_desc_from_packed: field %d out of range", 9 + i);
        *rest[i] = (int32_t)v;
    }
    d->tp_rank = 0;
    d->tp_size = 1;
    return 0;
}

FORGE_API int forge_b200_create_packed(const void* args) {
    ForgeModelDesc d;
    if (forge_b200_desc_from_packed(args, &d)) return FORGE_INVALID_ARGS;
    const int64_t device = packed_i64(args, 112);
    ForgeB200** out = reinterpret_cast<ForgeB200**>(static_cast<intptr_t>(packed_i64(args, 120)));
    if (!out || !fits_i32(device)) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_create_packed: bad device or result address");
    return forge_b200_create(&d, (int)device, out);
}

FORGE_API int forge_b200_decode_step_sampled_packed(const void* args) {
    if (!args) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_decode_step_sampled_packed: null argument");
    auto ptr = [&](int off) { return reinterpret_cast<void*>(static_cast<intptr_t>(packed_i64(args, off))); };
    const int64_t batch = packed_i64(args, 8), top_k = packed_i64(args, 40);
    if (!fits_i32(batch) || !fits_i32(top_k))
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_decode_step_sampled_packed: batch or top_k out of range");
    return forge_b200_decode_step_sampled(static_cast<ForgeB200*>(ptr(0)), (int)batch,
                                          static_cast<const int32_t*>(ptr(16)), static_cast<int32_t*>(ptr(24)),
                                          packed_f64(args, 32), (int)top_k, packed_f64(args, 48),
                                          static_cast<int64_t*>(ptr(56)));
}

FORGE_API int forge_b200_decode_device(ForgeB200* h, int batch, int n_steps) {
    if (int rc = check_ready(h, batch)) return rc;
    for (int i = 0; i < n_steps; ++i)
        if (enqueue_one(h, batch)) return -1;
    return 0;
}

namespace {
// Shortest prompt that takes the tensor-core attention in prefill
// (FORGE_PREFILL_FLASH_MIN; default 256).
int prefill_flash_min() {
    static const int v = [] {
        const char* e = getenv("FORGE_PREFILL_FLASH_MIN");
        const int x = e ? atoi(e) : 256;
        return x > 0 ? x : 256;
    }();
    return v;
}

// Grows the prefill buffers to R rows (outside any stream capture).
int prefill_reserve(ForgeB200* h, int64_t R) {
    auto& P = h->pre;
    if (R <= P.cap) return 0;
    cudaStreamSynchronize(h->stream);
    for (void* p : {(void*)P.x, (void*)P.q, (void*)P.ctx, (void*)P.s, (void*)P.partial, (void*)P.tok, (void*)P.pos,
                    (void*)P.seq, (void*)P.sel, (void*)P.counters})
        if (p) cudaFree(p);
    uint16_t *qb = P.qb, *ob = P.ob;
    const int64_t qb_cap = P.qb_cap;
    P = {};
    P.qb = qb;
    P.ob = ob;
    P.qb_cap = qb_cap;
    int64_t part = 0;  // split partials for any row count up to R
    for (int64_t r = 1; r <= R; ++r)
        part = std::max(part, r * forge_attn_pick_splits((int)r, h->Hkv, h->lmax));
    bool ok = cudaMalloc(&P.x, 4 * R * h->d) == cudaSuccess && cudaMalloc(&P.q, 4 * R * h->qd) == cudaSuccess &&
              cudaMalloc(&P.ctx, 4 * R * h->qd) == cudaSuccess && cudaMalloc(&P.s, 4 * R * h->F) == cudaSuccess &&
              cudaMalloc(&P.partial, 4 * part * h->H * (h->hd + 2)) == cudaSuccess &&
              cudaMalloc(&P.tok, 4 * R) == cudaSuccess && cudaMalloc(&P.pos, 4 * R) == cudaSuccess &&
              cudaMalloc(&P.seq, 4 * R) == cudaSuccess && cudaMalloc(&P.sel, 8 * (size_t)h->Bmax) == cudaSuccess &&
              cudaMalloc(&P.counters, 4 * R * h->Hkv) == cudaSuccess &&
              cudaMemset(P.counters, 0, 4 * R * h->Hkv) == cudaSuccess;
    if (ok && !h->bscratch) {  // the batched GEMV paths (more than 4 rows)
        const size_t nb = (size_t)forge_gemv_b_scratch_bytes(std::max({h->d, h->qd, h->F}));
        h->bscratch = h->alloc(nb);
        ok = h->bscratch && cudaMemset(h->bscratch, 0, nb) == cudaSuccess;
    }
    if (!ok) {
        cudaGetLastError();
        return forge_fail(-1, "forge_b200_prefill: out of device memory for %lld rows", (long long)R);
    }
    P.cap = R;
    return 0;
}

// All prompt positions of `batch` sequences through the model at once.
int prefill_impl(ForgeB200* h, int batch, const int32_t* prompt, int n, int exact_mode) {
    const int64_t R = (int64_t)batch * n;
    if (int rc = prefill_reserve(h, R)) return rc;
    auto& P = h->pre;
    std::vector<int32_t> tok(R), pos(R), seq(R);
    for (int b = 0; b < batch; ++b)
        for (int p = 0; p < n; ++p) {
            const int64_t r = (int64_t)b * n + p;
            tok[r] = prompt[r];
            pos[r] = p;
            seq[r] = b;
            if (tok[r] < 0 || tok[r] >= h->Vfull)
                return forge_fail(FORGE_INVALID_ARGS, "forge_b200_prefill: token %d outside the vocabulary", tok[r]);
        }
    cudaStream_t st = h->stream;
    if (cudaMemcpyAsync(P.tok, tok.data(), 4 * R, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(P.pos, pos.data(), 4 * R, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(P.seq, seq.data(), 4 * R, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return forge_fail(-1, "forge_b200_prefill: H2D of the prompt failed");
    // exact_mode: 1 hi/lo activations for bf16 weights at any row count,
    // 0 the model's own activation policy (bf16 activations above 4 rows)
    const RowMap rm{P.pos, P.seq, P.partial, P.counters, exact_mode == 1};
    // Long prompts take the tensor-core causal prefill for attention (bf16 Q,
    // P and O; K / V read in place from the cache); short ones, and shapes
    // it does not cover, the split flash-decode per row (fp32 Q and O).
    const int S = (n + 127) / 128 * 128;
    const bool flash = (h->hd == 128 || h->hd == 64) && n >= prefill_flash_min() && S <= h->lmax && h->H % h->Hkv == 0;
    if (flash) {
        const int64_t need = (int64_t)batch * h->H * S * h->hd;
        if (need > P.qb_cap) {
            cudaStreamSynchronize(st);
            if (P.qb) cudaFree(P.qb);
            if (P.ob) cudaFree(P.ob);
            P.qb = P.ob = nullptr;
            P.qb_cap = 0;
            if (cudaMalloc(&P.qb, 2 * need) != cudaSuccess || cudaMalloc(&P.ob, 2 * need) != cudaSuccess) {
                cudaGetLastError();
                return forge_fail(-1, "forge_b200_prefill: out of device memory for %lld attention rows", (long long)need);
            }
            P.qb_cap = need;
        }
        // cache rows n..S-1 of these sequences are read (masked) by the last
        // key block: zero them so that no stale value can reach the sums
        if (S > n)
            for (int l = 0; l < h->L; ++l)
                for (uint16_t* c : {h->kc + (size_t)l * h->kv_layer, h->vc + (size_t)l * h->kv_layer})
                    cudaMemset2DAsync(c + (size_t)n * h->hd, (size_t)h->lmax * h->hd * 2, 0, (size_t)(S - n) * h->hd * 2,
                                      (size_t)batch * h->Hkv, st);
    }
    const int cgrid = 4 * forge_sm_count();
    int rc = forge_embed_launch(h->emb, h->d, h->Vfull, P.tok, (int)R, P.x, h->err, st, false);
    for (int l = 0; l < h->L && !rc; ++l) {
        rc = enqueue_qkv(h, l, (int)R, P.x, P.q, true, &rm);
        if (!rc && flash) {
            k_rows_to_heads_bf16<<<cgrid, 256, 0, st>>>(P.q, batch, n, S, h->H, h->hd, P.qb);
            rc = forge_flash_prefill_kv(P.qb, h->kc + (size_t)l * h->kv_layer, h->vc + (size_t)l * h->kv_layer, P.ob,
                                        batch, h->H, h->Hkv, S, h->hd, h->lmax, (int64_t)h->Bmax * h->Hkv * h->lmax, st);
            if (!rc) k_heads_bf16_to_rows<<<cgrid, 256, 0, st>>>(P.ob, batch, n, S, h->H, h->hd, P.ctx);
        } else if (!rc) {
            rc = enqueue_attn(h, l, (int)R, P.q, P.ctx, false, &rm);
        }
        rc = rc || enqueue_oproj(h, l, (int)R, P.ctx, P.x, true, &rm) || enqueue_mlp(h, l, (int)R, P.x, true, &rm, P.s);
    }
    if (rc) return -1;
    // last position of every sequence: final norm, LM head, argmax; the
    // finaliser records the token as step n-1 and moves the positions to n
    if (enqueue_head(h, batch, P.x + (size_t)(n - 1) * h->d, true, n * h->d)) return -1;
    k_set_i32<<<1, 256, 0, st>>>(h->pos, batch, n - 1);
    k_set_i32<<<1, 1, 0, st>>>(h->step, 1, n - 1);
    return forge_argmax_finalize_launch(h->amax, batch, h->tok, h->hist, h->step, h->pos, h->hist_cap, st, false);
}

// R ragged rows (token, position, sequence) through the model, then the LM
// head and argmax of n_out of them; tokens into P.sel + Bmax.
int forward_rows_impl(ForgeB200* h, int R, const int32_t* tok, const int32_t* pos, const int32_t* seq, int n_out,
                      const int32_t* out_rows, int exact_mode) {
    std::vector<int64_t> keys(R);
    for (int r = 0; r < R; ++r) {
        if (tok[r] < 0 || tok[r] >= h->Vfull)
            return forge_fail(FORGE_INVALID_ARGS, "forge_b200_forward_rows: token %d outside the vocabulary", tok[r]);
        if (seq[r] < 0 || seq[r] >= h->Bmax || pos[r] < 0 || pos[r] >= h->lmax)
            return forge_fail(FORGE_INVALID_ARGS, "forge_b200_forward_rows: row %d: sequence %d / position %d out of range",
                              r, seq[r], pos[r]);
        keys[r] = (int64_t)seq[r] * h->lmax + pos[r];
    }
    std::sort(keys.begin(), keys.end());
    if (std::adjacent_find(keys.begin(), keys.end()) != keys.end())
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_forward_rows: two rows write the same cache position");
    for (int i = 0; i < n_out; ++i)
        if (out_rows[i] < 0 || out_rows[i] >= R)
            return forge_fail(FORGE_INVALID_ARGS, "forge_b200_forward_rows: output row %d outside 0..%d", out_rows[i], R - 1);
    if (int rc = prefill_reserve(h, R)) return rc;
    auto& P = h->pre;
    cudaStream_t st = h->stream;
    if (cudaMemcpyAsync(P.tok, tok, 4 * (size_t)R, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(P.pos, pos, 4 * (size_t)R, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(P.seq, seq, 4 * (size_t)R, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(P.sel, out_rows, 4 * (size_t)n_out, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return forge_fail(-1, "forge_b200_forward_rows: H2D of the rows failed");
    const RowMap rm{P.pos, P.seq, P.partial, P.counters, exact_mode == 1};
    int rc = forge_embed_launch(h->emb, h->d, h->Vfull, P.tok, R, P.x, h->err, st, false);
    for (int l = 0; l < h->L && !rc; ++l)
        rc = enqueue_qkv(h, l, R, P.x, P.q, true, &rm) || enqueue_attn(h, l, R, P.q, P.ctx, false, &rm) ||
             enqueue_oproj(h, l, R, P.ctx, P.x, true, &rm) || enqueue_mlp(h, l, R, P.x, true, &rm, P.s);
    if (rc) return -1;
    k_gather_rows<<<n_out, 256, 0, st>>>(P.x, P.sel, h->d, h->x);
    if (enqueue_head(h, n_out, h->x, false)) return -1;
    k_argmax_extract<<<1, 1024, 0, st>>>(h->amax, n_out, P.sel + h->Bmax);
    return cudaGetLastError() == cudaSuccess ? 0 : forge_fail(-1, "forge_b200_forward_rows: launch failed");
}
}  // namespace

FORGE_API int forge_b200_prefill(ForgeB200* h, int batch, const int32_t* prompt, int n_prompt, int exact,
                                 int32_t* next_tok, float* logits) {
    if (int rc = check_ready(h, batch)) return rc;
    if (!prompt || n_prompt <= 0 || n_prompt > h->lmax)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_prefill: bad prompt length %d", n_prompt);
    if (forge_b200_reset(h)) return -1;
    if (int rc = prefill_impl(h, batch, prompt, n_prompt, exact)) return rc;
    if (cudaStreamSynchronize(h->stream) != cudaSuccess)
        return forge_fail(-1, "forge_b200_prefill: %s", cudaGetErrorString(cudaGetLastError()));
    if (int e = read_err(h)) return e;
    if (forge_ops_check()) return -1;  // the tensor-core attention's error word
    if (next_tok && cudaMemcpy(next_tok, h->tok, 4 * (size_t)batch, cudaMemcpyDeviceToHost) != cudaSuccess)
        return forge_fail(-1, "forge_b200_prefill: D2H of the next tokens failed");
    if (logits) {
        if (enqueue_logits_copy(h, batch, logits)) return -1;
        if (cudaStreamSynchronize(h->stream) != cudaSuccess)
            return forge_fail(-1, "forge_b200_prefill: logits copy: %s", cudaGetErrorString(cudaGetLastError()));
    }
    return 0;
}

FORGE_API int forge_b200_forward_rows(ForgeB200* h, int n_rows, const int32_t* tok, const int32_t* pos,
                                      const int32_t* seq, int n_out, const int32_t* out_rows, int exact,
                                      int32_t* next_tok, float* logits) {
    if (int rc = check_ready(h, n_out)) return rc;
    if (n_rows <= 0 || !tok || !pos || !seq || !out_rows)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_forward_rows: no rows or a null array");
    if (int rc = forward_rows_impl(h, n_rows, tok, pos, seq, n_out, out_rows, exact)) return rc;
    if (next_tok)
        cudaMemcpyAsync(next_tok, h->pre.sel + h->Bmax, 4 * (size_t)n_out, cudaMemcpyDeviceToHost, h->stream);
    if (logits && enqueue_logits_copy(h, n_out, logits)) return -1;
    if (cudaStreamSynchronize(h->stream) != cudaSuccess)
        return forge_fail(-1, "forge_b200_forward_rows: %s", cudaGetErrorString(cudaGetLastError()));
    return read_err(h);
}

FORGE_API int forge_b200_generate(ForgeB200* h, int batch, const int32_t* prompt, int n_prompt, int n_gen, int32_t* out) {
    if (int rc = check_ready(h, batch)) return rc;
    if (!prompt || !out || n_prompt <= 0 || n_gen <= 0 || n_prompt + n_gen - 1 > h->lmax)
        return forge_fail(FORGE_INVALID_ARGS, "forge_b200_generate: bad prompt/generation length");
    if (forge_b200_reset(h)) return -1;
    // the whole prompt in one pass (hi/lo activations unless the model asks
    // for bf16 ones), then one decode step per further token
    int rc = prefill_impl(h, batch, prompt, n_prompt, h->desc.act_mode == 2 ? 0 : 1);
    for (int i = 1; i < n_gen && !rc; ++i) rc = enqueue_one(h, batch);
    if (cudaStreamSynchronize(h->stream) != cudaSuccess)
        rc = forge_fail(-1, "forge_b200_generate: %s", cudaGetErrorString(cudaGetLastError()));
    if (rc) return rc;
    if (int e = read_err(h)) return e;
    if (forge_ops_check()) return -1;
    std::vector<int32_t> hist((size_t)n_gen * batch);
    if (cudaMemcpy2D(hist.data(), 4 * batch, h->hist + (size_t)(n_prompt - 1) * batch, 4 * batch, 4 * batch, n_gen,
                     cudaMemcpyDeviceToHost) != cudaSuccess)
        return forge_fail(-1, "forge_b200_generate: D2H history failed");
    for (int i = 0; i < n_gen; ++i)
        for (int b = 0; b < batch; ++b) out[(size_t)b * n_gen + i] = hist[(size_t)i * batch + b];
    return 0;
}

FORGE_API int forge_b200_sync(ForgeB200* h) {
    if (!h) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_sync: null handle");
    cudaSetDevice(h->device);
    if (cudaStreamSynchronize(h->stream) != cudaSuccess)
        return forge_fail(-1, "forge_b200_sync: %s", cudaGetErrorString(cudaGetLastError()));
    return read_err(h);
}

// 1 when decode steps at this batch size run as the single fused kernel.
FORGE_API int forge_b200_uses_fused_step(ForgeB200* h, int batch) {
    if (!h || batch <= 0 || batch > h->Bmax) return -1;
    cudaSetDevice(h->device);
    return fused_for(h, batch) ? 1 : 0;
}

// Copies the last fused step's timeline: [grid][nphases][4] globaltimer ns
// (phase entry, barrier passed, -, phase done). Returns nphases or -1.
FORGE_API int forge_b200_step_trace(ForgeB200* h, unsigned long long* out, int cap) {
    if (!h || !h->trace) return -1;
    const size_t n = (size_t)4 * h->trace_n * forge_sm_count();
    if ((size_t)cap < n) return -1;
    if (cudaMemcpy(out, h->trace, n * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return h->trace_n;
}

FORGE_API int64_t forge_b200_step_bytes(ForgeB200* h, int batch, int ctx_len) {
    if (!h) return -1;
    const bool q4 = h->q4;
    auto mat = [&](int64_t N, int64_t K) { return (int64_t)tile_bytes(q4, N, K) + (int64_t)scale_bytes(q4, N, K); };
    int64_t per_layer = mat(h->nqkv, h->d) + mat(h->d, h->qd) + mat(2 * h->F, h->d) + mat(h->d, h->F) + 8 * h->d;
    int64_t bytes = per_layer * h->L + (int64_t)h->Vpad * h->d * 2 + 4 * h->d + (int64_t)batch * h->d * 2;
    // KV: read positions 0..ctx (ctx+1 rows incl. the new one), write one row, K and V, every layer
    bytes += (int64_t)batch * h->L * 2 * h->Hkv * h->hd * 2 * ((int64_t)ctx_len + 1 + 1);
    return bytes;
}

FORGE_API int forge_b200_launches_per_step(ForgeB200* h, int batch) {
    if (!h || batch <= 0) return -1;
    if (fused_for(h, batch)) return 1;
    const bool split = h->split_for(batch);
    auto launches = [&](int K) { return forge_gemv_launch_count(K, batch, split, h->q4, h->bscratch != nullptr); };
    int per_layer = launches(h->d) * 2 + launches(h->qd) + launches(h->F) + 1;
    if (h->comm && !tp_fused(h, batch) && tp_oneshot(h, batch)) per_layer += 2;  // the peer-memory all-reduces
    if (h->pq_s_on && batch <= 4 && forge_gemv_launch_count(h->F, batch, split, true, false) == 1)
        per_layer += 1;  // the staging of s
    const int norm_stages = pq_x_on(h, batch) && !pq_by_ar(h, batch) ? 2 * h->L - 1 : 0;  // x staged after O / down
    return 1 + h->L * per_layer + norm_stages + forge_gemv_launch_count(h->d, batch, split, false, h->bscratch != nullptr) +
           1;
}
int64_t forge_b200_width(const ForgeB200* h, int which) {
    if (!h) return 0;
    return which == 0 ? h->d : which == 1 ? h->qd : h->V;  // under tensor parallelism: this rank's slice
}

// ---- block-level entries (the v2 fused families) ------------------------------
// Each runs one block of one layer on the handle's stream, on device arrays
// the caller owns, at the handle's current positions; they are the pieces
// forge_b200_decode_step chains, with the same kernels and arguments.
namespace {
int check_block(ForgeB200* h, int layer, int B) {
    if (int rc = check_ready(h, B)) return rc;
    if (layer < 0 || layer >= h->L) return forge_fail(FORGE_INVALID_ARGS, "forge_b200: layer %d outside 0..%d", layer, h->L - 1);
    return 0;
}
}  // namespace

FORGE_API int forge_b200_qkv_rope(ForgeB200* h, int layer, int batch, const float* x, float* q) {
    if (int rc = check_block(h, layer, batch)) return rc;
    if (!x || !q) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_qkv_rope: null array");
    return enqueue_qkv(h, layer, batch, x, q, false);
}

FORGE_API int forge_b200_attention(ForgeB200* h, int layer, int batch, const float* q, float* ctx) {
    if (int rc = check_block(h, layer, batch)) return rc;
    if (!q || !ctx) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_attention: null array");
    return enqueue_attn(h, layer, batch, q, ctx, false);
}

FORGE_API int forge_b200_o_proj(ForgeB200* h, int layer, int batch, const float* ctx, float* x) {
    if (int rc = check_block(h, layer, batch)) return rc;
    if (!ctx || !x) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_o_proj: null array");
    return enqueue_oproj(h, layer, batch, ctx, x, false);
}

FORGE_API int forge_b200_mlp(ForgeB200* h, int layer, int batch, const float* x, float* y) {
    if (int rc = check_block(h, layer, batch)) return rc;
    if (!x || !y) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_mlp: null array");
    if (x != y) {
        cudaError_t e = cudaMemcpyAsync(y, x, (size_t)batch * h->d * 4, cudaMemcpyDeviceToDevice, h->stream);
        if (e != cudaSuccess) return forge_fail(-1, "forge_b200_mlp: copy: %s", cudaGetErrorString(e));
    }
    return enqueue_mlp(h, layer, batch, y, false);
}

FORGE_API int forge_b200_lm_head(ForgeB200* h, int batch, const float* x, int32_t* tok, float* logits) {
    if (int rc = check_ready(h, batch)) return rc;
    if (!x || !tok) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_lm_head: null array");
    if (enqueue_head(h, batch, x, false)) return -1;
    k_argmax_extract<<<1, 1024, 0, h->stream>>>(h->amax, batch, tok);
    if (int rc = forge_check_launch("argmax extract")) return rc;
    if (logits) {
        cudaError_t e = cudaMemcpy2DAsync(logits, (size_t)h->V * 4, h->logits, (size_t)h->Vpad * 4, (size_t)h->V * 4,
                                          batch, cudaMemcpyDeviceToDevice, h->stream);
        if (e != cudaSuccess) return forge_fail(-1, "forge_b200_lm_head: logits copy: %s", cudaGetErrorString(e));
    }
    return 0;
}

FORGE_API int forge_b200_embed(ForgeB200* h, int batch, const int32_t* tok, float* x) {
    if (int rc = check_ready(h, batch)) return rc;
    if (!tok || !x) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_embed: null array");
    return forge_embed_launch(h->emb, h->d, h->Vfull, tok, batch, x, h->err, h->stream, false);
}

FORGE_API int forge_b200_advance(ForgeB200* h, int batch) {
    if (int rc = check_ready(h, batch)) return rc;
    k_add_i32<<<1, 256, 0, h->stream>>>(h->pos, batch, 1);
    return forge_check_launch("advance positions");
}
}  // extern "C"

