/* forge_oracle.c — CPU oracle (test infrastructure only; see forge_oracle.h).
 *
 * Every function states the reference file:line it restates. Arithmetic is
 * f64 unless a flag asks for a device storage rounding (bf16 KV cache,
 * bf16 GEMV inputs); the device kernels are checked against this file.
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off).
 */
#include "forge_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---------------------------------------------------------------- bf16 --
 * RNE f32 -> bf16 bit pattern: quiet NaN keeps a payload bit, otherwise add
 * 0x7FFF + lsb and truncate (runtime_bf16_emit.hexa:264-277). */
uint16_t or_f32_to_bf16(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    if (((bits >> 23) & 0xFF) == 0xFF && (bits & 0x7FFFFF) != 0)
        return (uint16_t)((bits >> 16) | 0x0040);
    uint32_t lsb = (bits >> 16) & 1u;
    return (uint16_t)((bits + 0x7FFFu + lsb) >> 16);
}
/* bf16 -> f32 widening is exact (runtime_bf16_emit.hexa:280-286). */
float or_bf16_to_f32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float v;
    memcpy(&v, &bits, 4);
    return v;
}
void or_f32_to_bf16_n(const float* s, uint16_t* d, int64_t n) {
    for (int64_t i = 0; i < n; i++) d[i] = or_f32_to_bf16(s[i]);
}
void or_bf16_to_f32_n(const uint16_t* s, float* d, int64_t n) {
    for (int64_t i = 0; i < n; i++) d[i] = or_bf16_to_f32(s[i]);
}
static double rnd_bf16(double x) { return (double)or_bf16_to_f32(or_f32_to_bf16((float)x)); }

/* ------------------------------------------------------- flame LCG fill --
 * tensor_lib.hexa:67-88: st = st*6364136223846793005 + 1442695040888963407
 * (int64, wrapping), m = st % 2147483647 (C remainder), |m|; value
 * (m / 2147483647.0 * 2 - 1) * scale. */
void or_flame_fill_lcg(double* t, int64_t n, int64_t seed, double scale) {
    int64_t st = seed;
    for (int64_t i = 0; i < n; i++) {
        uint64_t s = (uint64_t)st * 6364136223846793005ULL + 1442695040888963407ULL;
        int64_t m = (int64_t)s % 2147483647LL;
        if (m < 0) m = -m;
        st = m;
        double f = (double)m / 2147483647.0;
        t[i] = (f * 2.0 - 1.0) * scale;
    }
}

/* ------------------------------------------------------------ quant_lib --
 * _q_round: round half away from zero via trunc(|x| + 0.5) (quant_lib.hexa:33-36). */
static double q_round(double x) {
    if (x >= 0.0) return (double)(int64_t)(x + 0.5);
    return 0.0 - (double)(int64_t)((0.0 - x) + 0.5);
}
/* nn_int4_quant_fwd (quant_lib.hexa:41-74): per-output-channel s = max|W|/7
 * (0 -> 1), q = clamp(round(W/s), -7, 7), Wq = q*s, mask = in-range. */
void or_int4_quant_fwd(const double* w, double* wq, double* scale, double* ql,
                       double* mask, int cout, int rest) {
    for (int co = 0; co < cout; co++) {
        double mx = 0.0;
        for (int j = 0; j < rest; j++) {
            double a = fabs(w[(int64_t)co * rest + j]);
            if (a > mx) mx = a;
        }
        double s = mx > 0.0 ? mx / 7.0 : 1.0;
        scale[co] = s;
        for (int j = 0; j < rest; j++) {
            int64_t idx = (int64_t)co * rest + j;
            double q = q_round(w[idx] / s);
            double in = 1.0;
            if (q > 7.0) { q = 7.0; in = 0.0; }
            if (q < -7.0) { q = -7.0; in = 0.0; }
            ql[idx] = q;
            mask[idx] = in;
            wq[idx] = q * s;
        }
    }
}
/* _q_code (quant_lib.hexa:103-112): code = clamp(round(w/s)) + zero. */
static int q_code(double w, double s, int zero) {
    int64_t q = (int64_t)q_round(w / s);
    if (q > 7) q = 7;
    if (q < -7) q = -7;
    return (int)q + zero;
}
/* nn_int4_pack (quant_lib.hexa:114-129): even index -> low nibble. */
void or_int4_pack(const double* w, uint8_t* packed, int n, double s, int zero) {
    for (int i = 0; i < n; i += 2) {
        int b = q_code(w[i], s, zero);
        if (i + 1 < n) b |= q_code(w[i + 1], s, zero) << 4;
        packed[i / 2] = (uint8_t)b;
    }
}
/* nn_int4_unpack (quant_lib.hexa:131-141): (code - zero) * s. */
void or_int4_unpack(const uint8_t* packed, double* out, int n, double s, int zero) {
    for (int i = 0; i < n; i++) {
        int b = packed[i / 2];
        int code = (i & 1) ? ((b >> 4) & 15) : (b & 15);
        out[i] = (double)(code - zero) * s;
    }
}

/* ------------------------------------------------------- group-128 int4 --
 * Strict generalisation of quant_lib to groups of `group` weights along the
 * input dim with a bf16 scale: s = bf16_rne(f32(max|W_g|) / 7) (0 -> 1),
 * q = clamp(_q_round(W / s), -7, 7) in f64, code = q + 7, even k low nibble.
 * With group == K and the f64 scale this is exactly nn_int4_quant_fwd+pack. */
int or_q4g_quantize_bf16(const uint16_t* w, int64_t rows, int64_t K, int group,
                         uint8_t* codes, uint16_t* scales) {
    if (rows <= 0 || K <= 0 || group <= 0 || (K % group) != 0 || (group & 1)) return -1;
    int64_t G = K / group;
#pragma omp parallel for schedule(static) if (rows * K > (1 << 18))
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t g = 0; g < G; g++) {
            const uint16_t* wg = w + r * K + g * group;
            float mx = 0.0f;
            for (int j = 0; j < group; j++) {
                float a = fabsf(or_bf16_to_f32(wg[j]));
                if (a > mx) mx = a;
            }
            uint16_t sb = or_f32_to_bf16(mx / 7.0f);
            if (mx == 0.0f || (sb & 0x7FFF) == 0) sb = 0x3F80; /* 1.0 sentinel */
            scales[r * G + g] = sb;
            double s = (double)or_bf16_to_f32(sb);
            uint8_t* cp = codes + (r * K + g * group) / 2;
            for (int j = 0; j < group; j += 2) {
                int lo = q_code((double)or_bf16_to_f32(wg[j]), s, 7);
                int hi = q_code((double)or_bf16_to_f32(wg[j + 1]), s, 7);
                cp[j / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
    return 0;
}
int or_q4g_dequant(const uint8_t* codes, const uint16_t* scales, int64_t rows,
                   int64_t K, int group, float* out) {
    if (rows <= 0 || K <= 0 || group <= 0 || (K % group) != 0) return -1;
    int64_t G = K / group;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t k = 0; k < K; k++) {
            int b = codes[(r * K + k) / 2];
            int code = (k & 1) ? ((b >> 4) & 15) : (b & 15);
            out[r * K + k] = (float)(code - 7) * or_bf16_to_f32(scales[r * G + k / group]);
        }
    return 0;
}

/* ------------------------------------------------------ synthetic data --
 * Counter-based N(0,1): a 64-bit splitmix-style hash of (seed, index) gives
 * two 32-bit uniforms; Box–Muller with a series ln and cos written here from
 * their Taylor/atanh expansions so that host and device produce the same
 * bits (no libm; every op is one IEEE +,-,*,/,sqrt; built without FMA
 * contraction). */
static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
static double ser_ln(double u) { /* u in (0, 1] */
    uint64_t bits;
    memcpy(&bits, &u, 8);
    int e = (int)((bits >> 52) & 0x7FF) - 1023;
    uint64_t mb = (bits & 0x000FFFFFFFFFFFFFULL) | 0x3FF0000000000000ULL;
    double m;
    memcpy(&m, &mb, 8);
    if (m > 1.4142135623730951) { m = m * 0.5; e = e + 1; }
    double s = (m - 1.0) / (m + 1.0);
    double s2 = s * s;
    double p = 1.0 / 23.0;
    p = p * s2 + 1.0 / 21.0;
    p = p * s2 + 1.0 / 19.0;
    p = p * s2 + 1.0 / 17.0;
    p = p * s2 + 1.0 / 15.0;
    p = p * s2 + 1.0 / 13.0;
    p = p * s2 + 1.0 / 11.0;
    p = p * s2 + 1.0 / 9.0;
    p = p * s2 + 1.0 / 7.0;
    p = p * s2 + 1.0 / 5.0;
    p = p * s2 + 1.0 / 3.0;
    p = p * s2 + 1.0;
    double lnm = (2.0 * s) * p;
    return (double)e * 0.6931471805599453 + lnm;
}
static double ser_cos(double x) { /* |x| <= pi/4 */
    double x2 = x * x;
    double p = 1.0 / 2432902008176640000.0;
    p = p * x2 - 1.0 / 6402373705728000.0;
    p = p * x2 + 1.0 / 20922789888000.0;
    p = p * x2 - 1.0 / 87178291200.0;
    p = p * x2 + 1.0 / 479001600.0;
    p = p * x2 - 1.0 / 3628800.0;
    p = p * x2 + 1.0 / 40320.0;
    p = p * x2 - 1.0 / 720.0;
    p = p * x2 + 1.0 / 24.0;
    p = p * x2 - 1.0 / 2.0;
    p = p * x2 + 1.0;
    return p;
}
static double ser_sin(double x) { /* |x| <= pi/4 */
    double x2 = x * x;
    double p = 1.0 / 51090942171709440000.0;
    p = p * x2 - 1.0 / 121645100408832000.0;
    p = p * x2 + 1.0 / 355687428096000.0;
    p = p * x2 - 1.0 / 1307674368000.0;
    p = p * x2 + 1.0 / 6227020800.0;
    p = p * x2 - 1.0 / 39916800.0;
    p = p * x2 + 1.0 / 362880.0;
    p = p * x2 - 1.0 / 5040.0;
    p = p * x2 + 1.0 / 120.0;
    p = p * x2 - 1.0 / 6.0;
    p = p * x2 + 1.0;
    return x * p;
}
static double ser_cos2pi(double u) { /* u in [0, 1) */
    const double two_pi = 6.283185307179586;
    double sign = 1.0;
    if (u > 0.5) u = 1.0 - u;
    if (u > 0.25) { u = 0.5 - u; sign = -1.0; }
    double r;
    if (u > 0.125) r = ser_sin((0.25 - u) * two_pi);
    else r = ser_cos(u * two_pi);
    return sign * r;
}
double or_normal_at(uint64_t seed, uint64_t idx) {
    uint64_t z = mix64(seed * 0x9E3779B97F4A7C15ULL + idx * 0xD1B54A32D192ED03ULL +
                       0x632BE59BD9B4E019ULL);
    uint32_t a = (uint32_t)(z >> 32), b = (uint32_t)z;
    double u1 = ((double)a + 1.0) * (1.0 / 4294967296.0);
    double u2 = (double)b * (1.0 / 4294967296.0);
    double r = sqrt(-2.0 * ser_ln(u1));
    return r * ser_cos2pi(u2);
}
void or_fill_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t offset, float std) {
    double sd = (double)std;
#pragma omp parallel for schedule(static) if (n > (1 << 16))
    for (int64_t i = 0; i < n; i++)
        out[i] = or_f32_to_bf16((float)(sd * or_normal_at(seed, offset + (uint64_t)i)));
}

/* RoPE tables (nn_lib.hexa:509-531): invf_i = 1/exp((2i/hd) ln theta),
 * ang = p*invf_i; the reference's d5 Taylor sin/cos is replaced by libm
 * (difference ~1e-16 before the f32 store). Stored [lmax][hd/2]. */
void or_rope_table(float* cos_t, float* sin_t, int lmax, int hd, double theta) {
    int half = hd / 2;
    double lnb = log(theta);
    for (int p = 0; p < lmax; p++)
        for (int i = 0; i < half; i++) {
            double ex = ((double)(2 * i) / (double)hd) * lnb;
            double invf = 1.0 / exp(ex);
            double ang = (double)p * invf;
            cos_t[(int64_t)p * half + i] = (float)cos(ang);
            sin_t[(int64_t)p * half + i] = (float)sin(ang);
        }
}

/* ------------------------------------------------------------ model ---- */
static double mat_at(const OrMat* m, int64_t r, int64_t c) {
    switch (m->kind) {
    case OR_MAT_F32: return (double)((const float*)m->w)[r * m->cols + c];
    case OR_MAT_BF16: return (double)or_bf16_to_f32(((const uint16_t*)m->w)[r * m->cols + c]);
    default: {
        const uint8_t* cd = (const uint8_t*)m->w;
        int b = cd[(r * m->cols + c) / 2];
        int code = (c & 1) ? ((b >> 4) & 15) : (b & 15);
        int64_t G = m->cols / m->group;
        return (double)(code - 7) * (double)or_bf16_to_f32(m->scales[r * G + c / m->group]);
    }
    }
}
/* y = W x with f64 accumulation; q4 rows accumulate sum(q*x) per group and
 * scale once per group (same algebra as the device). */
static double row_dot(const OrMat* m, int64_t r, const double* x) {
    int64_t K = m->cols;
    double acc = 0.0;
    if (m->kind == OR_MAT_F32) {
        const float* w = (const float*)m->w + r * K;
        for (int64_t c = 0; c < K; c++) acc += (double)w[c] * x[c];
    } else if (m->kind == OR_MAT_BF16) {
        const uint16_t* w = (const uint16_t*)m->w + r * K;
        for (int64_t c = 0; c < K; c++) acc += (double)or_bf16_to_f32(w[c]) * x[c];
    } else {
        const uint8_t* cd = (const uint8_t*)m->w + r * K / 2;
        int64_t G = K / m->group;
        for (int64_t g = 0; g < G; g++) {
            double part = 0.0;
            for (int64_t c = g * m->group; c < (g + 1) * m->group; c += 2) {
                int b = cd[c / 2];
                part += (double)((b & 15) - 7) * x[c] + (double)(((b >> 4) & 15) - 7) * x[c + 1];
            }
            acc += part * (double)or_bf16_to_f32(m->scales[r * G + g]);
        }
    }
    return acc;
}
static void gemv(const OrMat* m, const double* x_in, double* y, int act_bf16) {
    const double* x = x_in;
    double* xr = NULL;
    if (act_bf16) {
        xr = (double*)malloc(sizeof(double) * (size_t)m->cols);
        for (int64_t c = 0; c < m->cols; c++) xr[c] = rnd_bf16(x_in[c]);
        x = xr;
    }
    int64_t R = m->rows;
#pragma omp parallel for schedule(static) if (R * m->cols > (1 << 16))
    for (int64_t r = 0; r < R; r++) y[r] = row_dot(m, r, x);
    free(xr);
}
/* nn_rmsnorm_fwd (nn_lib.hexa:150-171): y = g * (x * 1/sqrt(mean(x^2)+eps)). */
static void rmsnorm(const double* x, const float* g, double* y, int d, float eps) {
    double ms = 0.0;
    for (int i = 0; i < d; i++) ms += x[i] * x[i];
    ms = ms / (double)d;
    double inv = 1.0 / sqrt(ms + (double)eps);
    for (int i = 0; i < d; i++) y[i] = (double)g[i] * (x[i] * inv);
}
/* rotate-half RoPE (nn_lib.hexa:541-562) on one head vector at position p. */
static void rope(double* v, int hd, const float* ct, const float* st, int p) {
    int h = hd / 2;
    for (int c = 0; c < h; c++) {
        double cs = ct[(int64_t)p * h + c], sn = st[(int64_t)p * h + c];
        double a = v[c], b = v[c + h];
        v[c] = a * cs - b * sn;
        v[c + h] = b * cs + a * sn;
    }
}
static double silu(double a) { return a / (1.0 + exp(-a)); }

int or_decode_step(const OrModel* m, float* kc, float* vc, int lmax, int B,
                   const int32_t* tok, const int32_t* pos, int flags,
                   float* logits, int32_t* argmax, double* hidden_out) {
    const int d = m->d, H = m->n_head, Hkv = m->n_kv, hd = m->hd, F = m->ffn, V = m->vocab;
    if (d <= 0 || H <= 0 || Hkv <= 0 || (H % Hkv) || (hd & 1) || B <= 0) return -1;
    const int qd = H * hd, kvd = Hkv * hd, rep = H / Hkv;
    const int act = (flags & OR_ACT_BF16) != 0, kvr = (flags & OR_KV_BF16) != 0;
    int maxp = 0;
    for (int b = 0; b < B; b++) {
        if (pos[b] < 0 || pos[b] >= lmax || tok[b] < 0 || tok[b] >= V) return -1;
        if (pos[b] > maxp) maxp = pos[b];
    }
    float* ct = (float*)malloc(sizeof(float) * (size_t)(maxp + 1) * (hd / 2));
    float* st = (float*)malloc(sizeof(float) * (size_t)(maxp + 1) * (hd / 2));
    or_rope_table(ct, st, maxp + 1, hd, (double)m->theta);
    double* x = (double*)malloc(sizeof(double) * d);
    double* r = (double*)malloc(sizeof(double) * (d > F ? d : F));
    double* q = (double*)malloc(sizeof(double) * qd);
    double* k = (double*)malloc(sizeof(double) * kvd);
    double* v = (double*)malloc(sizeof(double) * kvd);
    double* ctx = (double*)malloc(sizeof(double) * qd);
    double* o = (double*)malloc(sizeof(double) * d);
    double* a = (double*)malloc(sizeof(double) * F);
    double* u = (double*)malloc(sizeof(double) * F);
    double* sc = (double*)malloc(sizeof(double) * (size_t)(maxp + 1));
    double* lg = (double*)malloc(sizeof(double) * V);
    const double scale = 1.0 / sqrt((double)hd);
    for (int b = 0; b < B; b++) {
        const int p = pos[b];
        for (int c = 0; c < d; c++) x[c] = mat_at(&m->emb, tok[b], c); /* nn_embedding_fwd */
        for (int l = 0; l < m->n_layer; l++) {
            const OrLayer* L = &m->layers[l];
            rmsnorm(x, L->g1, r, d, m->eps);
            gemv(&L->wq, r, q, act);
            gemv(&L->wk, r, k, act);
            gemv(&L->wv, r, v, act);
            if (!(flags & OR_NO_ROPE)) {
                for (int h = 0; h < H; h++) rope(q + (int64_t)h * hd, hd, ct, st, p);
                for (int h = 0; h < Hkv; h++) rope(k + (int64_t)h * hd, hd, ct, st, p);
            }
            for (int h = 0; h < Hkv; h++) {
                size_t base = ((((size_t)l * B + b) * Hkv + h) * lmax + p) * hd;
                for (int c = 0; c < hd; c++) {
                    double kk = k[h * hd + c], vv = v[h * hd + c];
                    kc[base + c] = kvr ? (float)rnd_bf16(kk) : (float)kk;
                    vc[base + c] = kvr ? (float)rnd_bf16(vv) : (float)vv;
                }
            }
            /* attention core for one query (nn_lib.hexa:221-278, row i = p) */
            for (int h = 0; h < H; h++) {
                int kvh = h / rep;
                size_t hb = (((size_t)l * B + b) * Hkv + kvh) * lmax * hd;
                double mx = -INFINITY;
                for (int j = 0; j <= p; j++) {
                    double dot = 0.0;
                    const float* kr = kc + hb + (size_t)j * hd;
                    for (int c = 0; c < hd; c++) dot += q[h * hd + c] * (double)kr[c];
                    sc[j] = dot * scale;
                    if (sc[j] > mx) mx = sc[j];
                }
                double tot = 0.0;
                for (int j = 0; j <= p; j++) { sc[j] = exp(sc[j] - mx); tot += sc[j]; }
                for (int c = 0; c < hd; c++) {
                    double acc = 0.0;
                    for (int j = 0; j <= p; j++) acc += sc[j] * (double)vc[hb + (size_t)j * hd + c];
                    ctx[h * hd + c] = acc / tot;
                }
            }
            gemv(&L->wo, ctx, o, act);
            for (int c = 0; c < d; c++) x[c] += o[c];            /* residual 1 */
            rmsnorm(x, L->g2, r, d, m->eps);
            gemv(&L->wg, r, a, act);
            gemv(&L->wu, r, u, act);
            for (int f = 0; f < F; f++) a[f] = silu(a[f]) * u[f];  /* nn_swiglu_fwd */
            gemv(&L->wd, a, o, act);
            for (int c = 0; c < d; c++) x[c] += o[c];            /* residual 2 */
        }
        if (hidden_out) memcpy(hidden_out + (size_t)b * d, x, sizeof(double) * d);
        rmsnorm(x, m->gF, r, d, m->eps);                          /* final norm */
        gemv(&m->head, r, lg, act);                               /* LM head   */
        int best = 0;
        for (int kk = 1; kk < V; kk++) if (lg[kk] > lg[best]) best = kk;
        if (argmax) argmax[b] = best;
        if (logits) for (int kk = 0; kk < V; kk++) logits[(size_t)b * V + kk] = (float)lg[kk];
    }
    free(ct); free(st); free(x); free(r); free(q); free(k); free(v); free(ctx);
    free(o); free(a); free(u); free(sc); free(lg);
    return 0;
}

/* Full recompute (decoder_lib.hexa:93-208 composed with
 * decoder_block_lib.hexa:217-508): every position through every block, causal
 * GQA attention with the full P matrix, final norm + head on the last row. */
int or_full_forward(const OrModel* m, const int32_t* ids, int T, double* logits) {
    const int d = m->d, H = m->n_head, Hkv = m->n_kv, hd = m->hd, F = m->ffn, V = m->vocab;
    if (T <= 0) return -1;
    const int qd = H * hd, kvd = Hkv * hd, rep = H / Hkv;
    float* ct = (float*)malloc(sizeof(float) * (size_t)T * (hd / 2));
    float* st = (float*)malloc(sizeof(float) * (size_t)T * (hd / 2));
    or_rope_table(ct, st, T, hd, (double)m->theta);
    double* X = (double*)malloc(sizeof(double) * (size_t)T * d);
    double* R = (double*)malloc(sizeof(double) * (size_t)T * (d > F ? d : F));
    double* Q = (double*)malloc(sizeof(double) * (size_t)T * qd);
    double* K = (double*)malloc(sizeof(double) * (size_t)T * kvd);
    double* Vv = (double*)malloc(sizeof(double) * (size_t)T * kvd);
    double* C = (double*)malloc(sizeof(double) * (size_t)T * qd);
    double* O = (double*)malloc(sizeof(double) * d);
    double* A = (double*)malloc(sizeof(double) * F);
    double* U = (double*)malloc(sizeof(double) * F);
    double* P = (double*)malloc(sizeof(double) * (size_t)T);
    const double scale = 1.0 / sqrt((double)hd);
    for (int t = 0; t < T; t++)
        for (int c = 0; c < d; c++) X[(size_t)t * d + c] = mat_at(&m->emb, ids[t], c);
    for (int l = 0; l < m->n_layer; l++) {
        const OrLayer* L = &m->layers[l];
        for (int t = 0; t < T; t++) {
            rmsnorm(X + (size_t)t * d, L->g1, R, d, m->eps);
            gemv(&L->wq, R, Q + (size_t)t * qd, 0);
            gemv(&L->wk, R, K + (size_t)t * kvd, 0);
            gemv(&L->wv, R, Vv + (size_t)t * kvd, 0);
            for (int h = 0; h < H; h++) rope(Q + (size_t)t * qd + h * hd, hd, ct, st, t);
            for (int h = 0; h < Hkv; h++) rope(K + (size_t)t * kvd + h * hd, hd, ct, st, t);
        }
        for (int h = 0; h < H; h++) {
            int kvh = h / rep;
            for (int i = 0; i < T; i++) {
                double mx = -INFINITY;
                for (int j = 0; j <= i; j++) {
                    double dot = 0.0;
                    for (int c = 0; c < hd; c++)
                        dot += Q[(size_t)i * qd + h * hd + c] * K[(size_t)j * kvd + kvh * hd + c];
                    P[j] = dot * scale;
                    if (P[j] > mx) mx = P[j];
                }
                double tot = 0.0;
                for (int j = 0; j <= i; j++) { P[j] = exp(P[j] - mx); tot += P[j]; }
                for (int c = 0; c < hd; c++) {
                    double acc = 0.0;
                    for (int j = 0; j <= i; j++) acc += (P[j] / tot) * Vv[(size_t)j * kvd + kvh * hd + c];
                    C[(size_t)i * qd + h * hd + c] = acc;
                }
            }
        }
        for (int t = 0; t < T; t++) {
            double* x = X + (size_t)t * d;
            gemv(&L->wo, C + (size_t)t * qd, O, 0);
            for (int c = 0; c < d; c++) x[c] += O[c];
            rmsnorm(x, L->g2, R, d, m->eps);
            gemv(&L->wg, R, A, 0);
            gemv(&L->wu, R, U, 0);
            for (int f = 0; f < F; f++) A[f] = silu(A[f]) * U[f];
            gemv(&L->wd, A, O, 0);
            for (int c = 0; c < d; c++) x[c] += O[c];
        }
    }
    rmsnorm(X + (size_t)(T - 1) * d, m->gF, R, d, m->eps);
    gemv(&m->head, R, logits, 0);
    (void)V;
    free(ct); free(st); free(X); free(R); free(Q); free(K); free(Vv); free(C);
    free(O); free(A); free(U); free(P);
    return 0;
}

int or_greedy(const OrModel* m, int lmax, const int32_t* prompt, int n_prompt,
              int n_gen, int flags, int32_t* out_ids, float* margins) {
    if (n_prompt <= 0 || n_prompt + n_gen > lmax + 1) return -1;
    size_t kvn = (size_t)m->n_layer * m->n_kv * lmax * m->hd;
    float* kc = (float*)calloc(kvn, sizeof(float));
    float* vc = (float*)calloc(kvn, sizeof(float));
    float* lg = (float*)malloc(sizeof(float) * m->vocab);
    int32_t tok = prompt[0], am = 0;
    int gen = 0;
    for (int p = 0; p < n_prompt + n_gen - 1; p++) {
        tok = p < n_prompt ? prompt[p] : out_ids[p - n_prompt];
        int32_t pp = p;
        if (or_decode_step(m, kc, vc, lmax, 1, &tok, &pp, flags, lg, &am, NULL)) break;
        if (p >= n_prompt - 1) {
            out_ids[gen] = am;
            if (margins) {
                float t1 = lg[am], t2 = -INFINITY;
                for (int k = 0; k < m->vocab; k++) if (k != am && lg[k] > t2) t2 = lg[k];
                margins[gen] = t1 - t2;
            }
            gen++;
        }
    }
    free(kc); free(vc); free(lg);
    return gen == n_gen ? 0 : -1;
}

/* flash_decode.hexa:14-27: per-chunk (m, l, O) partials, LSE merge. */
void or_flash_decode_single(const float* q, const float* K, const float* V, int L,
                            int hd, int chunk, double* out) {
    const double scale = 1.0 / sqrt((double)hd);
    int nc = (L + chunk - 1) / chunk;
    double* m = (double*)malloc(sizeof(double) * nc);
    double* l = (double*)malloc(sizeof(double) * nc);
    double* O = (double*)calloc((size_t)nc * hd, sizeof(double));
    for (int c = 0; c < nc; c++) {
        int j0 = c * chunk, j1 = j0 + chunk < L ? j0 + chunk : L;
        double mx = -INFINITY;
        for (int j = j0; j < j1; j++) {
            double s = 0.0;
            for (int e = 0; e < hd; e++) s += (double)q[e] * K[(size_t)j * hd + e];
            s *= scale;
            if (s > mx) mx = s;
        }
        double lsum = 0.0;
        for (int j = j0; j < j1; j++) {
            double s = 0.0;
            for (int e = 0; e < hd; e++) s += (double)q[e] * K[(size_t)j * hd + e];
            double p = exp(s * scale - mx);
            lsum += p;
            for (int e = 0; e < hd; e++) O[(size_t)c * hd + e] += p * V[(size_t)j * hd + e];
        }
        m[c] = mx; l[c] = lsum;
    }
    double mg = -INFINITY;
    for (int c = 0; c < nc; c++) if (m[c] > mg) mg = m[c];
    double lg = 0.0;
    for (int c = 0; c < nc; c++) lg += exp(m[c] - mg) * l[c];
    for (int e = 0; e < hd; e++) {
        double acc = 0.0;
        for (int c = 0; c < nc; c++) acc += exp(m[c] - mg) * O[(size_t)c * hd + e];
        out[e] = acc / lg;
    }
    free(m); free(l); free(O);
}

void or_matmul_f64(const double* A, const double* B, double* C, int M, int K, int N) {
    for (int i = 0; i < M; i++)
        for (int j = 0; j < N; j++) {
            double acc = 0.0;
            for (int k = 0; k < K; k++) acc += A[(size_t)i * K + k] * B[(size_t)k * N + j];
            C[(size_t)i * N + j] = acc;
        }
}

void or_ref_lcg_f32(uint32_t* state, float* out, int64_t n) {
    uint32_t st = *state;
    for (int64_t i = 0; i < n; ++i) {
        st = st * 1664525u + 1013904223u;
        out[i] = ((float)(st >> 8) / (float)(1u << 24)) - 0.5f;
    }
    *state = st;
}

/* ------------------------------------------------------------- sampler --
 * self/ml/gpu_sampler.hexa: RNG at :57-65, argmax at :70-85, the pipeline at
 * :89-277. The host buffer of the reference holds f32 (deref_f32 /
 * write_f32); hexa floats are f64. */
double or_sampler_rand(int64_t* state) {
    int64_t x = *state;
    x = x ^ (int64_t)((uint64_t)x * 8192u);
    x = x ^ (x / 131072);
    x = x ^ (int64_t)((uint64_t)x * 32u);
    if (x < 0) x = (int64_t)(0u - (uint64_t)x);
    *state = x;
    return (double)(x % 1000000) / 1000000.0;
}

static int or_argmax_first(const float* v, int n) {
    int best = 0;
    double bv = v[0];
    for (int i = 1; i < n; ++i)
        if ((double)v[i] > bv) { bv = v[i]; best = i; }
    return best;
}

int or_sample_token(const float* logits, int V, double temperature, int top_k, double top_p,
                    int64_t* rng_state, float* probs) {
    if (V <= 0) return -1;
    if (temperature <= 0.0) return or_argmax_first(logits, V);
    float* h = (float*)malloc(sizeof(float) * (size_t)V);
    const double inv_t = 1.0 / temperature;
    for (int i = 0; i < V; ++i) h[i] = (float)((double)logits[i] * inv_t);
    double mx = h[0];
    for (int i = 1; i < V; ++i)
        if ((double)h[i] > mx) mx = h[i];
    double sum_e = 0.0;
    for (int i = 0; i < V; ++i) {
        const double e = exp((double)h[i] - mx);
        h[i] = (float)e;
        sum_e = sum_e + e;
    }
    const double inv_sum = 1.0 / sum_e;
    for (int i = 0; i < V; ++i) h[i] = (float)((double)h[i] * inv_sum);
    if (top_k > 0 && top_k < V) {
        float* sb = (float*)malloc(sizeof(float) * (size_t)V);
        memcpy(sb, h, sizeof(float) * (size_t)V);
        for (int j = 0; j < top_k; ++j) {  /* partial selection sort */
            int best = j;
            for (int m = j + 1; m < V; ++m)
                if ((double)sb[m] > (double)sb[best]) best = m;
            if (best != j) { float t = sb[j]; sb[j] = sb[best]; sb[best] = t; }
        }
        const double thr = sb[top_k - 1];
        free(sb);
        double sum_k = 0.0;
        for (int i = 0; i < V; ++i) {
            if ((double)h[i] < thr) h[i] = 0.0f;
            else sum_k = sum_k + (double)h[i];
        }
        if (sum_k > 0.0) {
            const double inv_k = 1.0 / sum_k;
            for (int i = 0; i < V; ++i) h[i] = (float)((double)h[i] * inv_k);
        }
    }
    if (top_p < 1.0 && top_p > 0.0) {
        int* idx = (int*)malloc(sizeof(int) * (size_t)V);
        double* val = (double*)malloc(sizeof(double) * (size_t)V);
        int nn = 0;
        for (int i = 0; i < V; ++i)
            if ((double)h[i] > 0.0) { idx[nn] = i; val[nn] = h[i]; ++nn; }
        for (int ii = 0; ii < nn; ++ii) {  /* selection sort, descending, with swaps */
            int best = ii;
            for (int jj = ii + 1; jj < nn; ++jj)
                if (val[jj] > val[best]) best = jj;
            if (best != ii) {
                int ti = idx[ii]; idx[ii] = idx[best]; idx[best] = ti;
                double tv = val[ii]; val[ii] = val[best]; val[best] = tv;
            }
        }
        for (int i = 0; i < V; ++i) h[i] = 0.0f;
        double cum = 0.0, sum_p = 0.0;
        for (int i = 0; i < nn; ++i) {
            h[idx[i]] = (float)val[i];
            sum_p = sum_p + val[i];
            cum = cum + val[i];
            if (cum >= top_p) break;
        }
        if (sum_p > 0.0) {
            const double inv_p = 1.0 / sum_p;
            for (int i = 0; i < V; ++i) h[i] = (float)((double)h[i] * inv_p);
        }
        free(idx);
        free(val);
    }
    const double r = or_sampler_rand(rng_state);
    double cum = 0.0;
    int chosen = V - 1;
    for (int i = 0; i < V; ++i) {
        cum = cum + (double)h[i];
        if (cum > r) { chosen = i; break; }
    }
    if (probs) memcpy(probs, h, sizeof(float) * (size_t)V);
    free(h);
    return chosen;
}

/* ------------------------------------------------ training-side families */
double or_dt_exp(double x) {
    int r = 0;
    double xr = x;
    while ((xr > 0.0 ? xr : 0.0 - xr) > 0.25) { xr = xr / 2.0; r++; }
    double term = 1.0, acc = 1.0;
    for (int k = 1; k < 12; k++) { term = term * xr / (double)k; acc = acc + term; }
    for (int i = 0; i < r; i++) acc = acc * acc;
    return acc;
}

double or_attn_scale(int64_t hd) {
    double x = (double)hd, g = x > 1.0 ? x : 1.0;
    for (int i = 0; i < 24; i++) g = 0.5 * (g + x / g);
    return 1.0 / g;
}

void or_train_rmsnorm_rows(const double* x, int64_t R, int64_t C, double eps, double* y) {
    for (int64_t r = 0; r < R; r++) {
        double ss = 0.0;
        for (int64_t j = 0; j < C; j++) ss += x[r * C + j] * x[r * C + j];
        double inv = 1.0 / sqrt(ss / (double)C + eps);
        for (int64_t j = 0; j < C; j++) y[r * C + j] = x[r * C + j] * inv;
    }
}

void or_train_rmsnorm_bwd_rows(const double* x, const double* dxn, int64_t R, int64_t C, double* dx) {
    for (int64_t r = 0; r < R; r++) {
        const double* xr = x + r * C;
        const double* dr = dxn + r * C;
        double ss = 0.0, dot = 0.0;
        for (int64_t j = 0; j < C; j++) ss += xr[j] * xr[j];
        for (int64_t j = 0; j < C; j++) dot += dr[j] * xr[j];
        double inv = 1.0 / sqrt(ss / (double)C + 1e-6);
        double coef = (inv * inv * inv) / (double)C;
        for (int64_t i = 0; i < C; i++) dx[r * C + i] = inv * dr[i] - coef * xr[i] * dot;
    }
}

void or_train_adamw(double* w, double* m, double* v, const double* g, int64_t n, double lr, double b1, double b2,
                    double eps, double wd, int64_t step_t, double* out) {
    double b1t = 1.0, b2t = 1.0;
    for (int64_t e = 0; e < step_t; e++) { b1t *= b1; b2t *= b2; }
    const double c1 = 1.0 - b1t, c2 = 1.0 - b2t;
    for (int64_t i = 0; i < n; i++) {
        double gi = g[i], wi0 = w[i];
        double mi = b1 * m[i] + (1.0 - b1) * gi;
        double vi = b2 * v[i] + (1.0 - b2) * gi * gi;
        double mhat = mi / c1, vhat = vi / c2;
        double denom = sqrt(vhat) + eps;
        double wi = wi0 - lr * wd * wi0 - lr * mhat / denom;
        m[i] = mi;
        v[i] = vi;
        out[i] = wi;
    }
}

void or_train_rope(const double* t, const double* c, const double* s, int64_t T, int64_t nheads, int64_t hd, int bwd,
                   double* out) {
    const int64_t half = hd / 2, total = T * nheads * hd;
    for (int64_t i = 0; i < total; i++) {
        int64_t col = i % hd, row = i - col, tt = i / (nheads * hd), bse = tt * hd;
        if (!bwd) {
            double rh = col < half ? 0.0 - t[row + half + col] : t[row + col - half];
            out[i] = t[row + col] * c[bse + col] + rh * s[bse + col];
        } else {
            double gs = col < half ? t[row + half + col] * s[bse + half + col]
                                   : 0.0 - t[row + col - half] * s[bse + col - half];
            out[i] = t[row + col] * c[bse + col] + gs;
        }
    }
}

void or_train_silu(const double* a, const double* b, int64_t n, int mode, double* out) {
    for (int64_t i = 0; i < n; i++) {
        double x = a[i];
        if (mode == 0) {
            out[i] = x * (1.0 / (1.0 + exp(-x)));
        } else if (mode == 1) {
            double sg = 1.0 / (1.0 + exp(-x));
            out[i] = sg * (1.0 + x * (1.0 - sg));
        } else {
            double sig = 1.0 / (1.0 + or_dt_exp(0.0 - x));
            out[i] = (x * sig) * b[i];
        }
    }
}

void or_train_attn_fwd(const double* q, const double* k, const double* v, int64_t T, int64_t nh, int64_t nkv,
                       int64_t hd, double* p, double* ctx) {
    const int64_t n_rep = nh / nkv, d = nh * hd;
    const double scale = or_attn_scale(hd);
    for (int64_t hh = 0; hh < nh; hh++)
        for (int64_t i = 0; i < T; i++) {
            int64_t kvh = hh / n_rep, L = i + 1;
            double* pr = p + (hh * T + i) * T;
            for (int64_t j = 0; j < T; j++) pr[j] = 0.0;
            for (int64_t j = 0; j < L; j++) {
                double dot = 0.0;
                for (int64_t cc = 0; cc < hd; cc++) dot += q[(i * nh + hh) * hd + cc] * k[(j * nkv + kvh) * hd + cc];
                pr[j] = dot * scale;
            }
            double mx = pr[0];
            for (int64_t j = 1; j < L; j++) if (pr[j] > mx) mx = pr[j];
            double tot = 0.0;
            for (int64_t j = 0; j < L; j++) { pr[j] = or_dt_exp(pr[j] - mx); tot += pr[j]; }
            for (int64_t j = 0; j < L; j++) pr[j] = pr[j] / tot;
            for (int64_t c2 = 0; c2 < hd; c2++) {
                double acc = 0.0;
                for (int64_t j = 0; j < L; j++) acc += pr[j] * v[(j * nkv + kvh) * hd + c2];
                ctx[i * d + hh * hd + c2] = acc;
            }
        }
}

void or_train_attn_bwd(const double* q, const double* k, const double* v, const double* p, const double* dctx,
                       int64_t T, int64_t nh, int64_t nkv, int64_t hd, double* dq, double* dk, double* dv) {
    const int64_t n_rep = nh / nkv, d = nh * hd;
    const double scale = or_attn_scale(hd);
    double* ds = (double*)calloc((size_t)(nh * T * T), sizeof(double));
    for (int64_t hh = 0; hh < nh; hh++)
        for (int64_t i = 0; i < T; i++) {
            int64_t kvh = hh / n_rep;
            double* dr = ds + (hh * T + i) * T;
            const double* pr = p + (hh * T + i) * T;
            for (int64_t j = 0; j <= i; j++) {
                double acc = 0.0;
                for (int64_t cc = 0; cc < hd; cc++) acc += dctx[i * d + hh * hd + cc] * v[(j * nkv + kvh) * hd + cc];
                dr[j] = acc;
            }
            double sdot = 0.0;
            for (int64_t j = 0; j <= i; j++) sdot += pr[j] * dr[j];
            for (int64_t j = 0; j <= i; j++) dr[j] = (pr[j] * (dr[j] - sdot)) * scale;
            for (int64_t c2 = 0; c2 < hd; c2++) {
                double acc = 0.0;
                for (int64_t j = 0; j <= i; j++) acc += dr[j] * k[(j * nkv + kvh) * hd + c2];
                dq[(i * nh + hh) * hd + c2] = acc;
            }
        }
    for (int64_t j = 0; j < T; j++)
        for (int64_t kvh = 0; kvh < nkv; kvh++)
            for (int64_t cc = 0; cc < hd; cc++) {
                double av = 0.0, ak = 0.0;
                for (int64_t hh = kvh * n_rep; hh < (kvh + 1) * n_rep; hh++)
                    for (int64_t i = j; i < T; i++) {
                        av += p[(hh * T + i) * T + j] * dctx[i * d + hh * hd + cc];
                        ak += ds[(hh * T + i) * T + j] * q[(i * nh + hh) * hd + cc];
                    }
                dv[(j * nkv + kvh) * hd + cc] = av;
                dk[(j * nkv + kvh) * hd + cc] = ak;
            }
    free(ds);
}
