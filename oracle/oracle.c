/*
 * CPU oracle for the strict speculative decode path.  TEST INFRASTRUCTURE
 * ONLY: see oracle.h for what is restated from where, and for the parity
 * status of each part.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct __attribute__((packed)) {
    uint16_t d;
    int8_t qs[32];
} blk_q8;

_Static_assert(sizeof(blk_q8) == 34, "q8_0 block is 34 bytes");

static inline float h2f(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}
static inline uint16_t f2h(float f) {
    _Float16 v = (_Float16)f; /* IEEE round to nearest even */
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}
static inline float round_f16(float f) { return h2f(f2h(f)); }

/* ------------------------------------------------------------ exp, sin, cos
 * Own implementations; the library is built with -ffp-contract=off, so only
 * the fmaf calls written here are fused, and the CUDA kernels evaluate the
 * same sequence, so both sides return identical floats.
 * exp: float arithmetic throughout.  n = rint(x log2 e); Cody-Waite reduction
 * r = x - n ln2 with ln2 split into a 16-bit head (0x3F317200) and a tail,
 * each step one fmaf; e^r by the Taylor polynomial to r^7 in Horner form
 * (fmaf per step, coefficients the floats nearest 1/k!); then exact scaling
 * by 2^n (two factors, so a subnormal result is rounded once).
 * Within 1 ulp of the true value (|r| <= 0.347: truncation 5e-9 relative).
 * sin/cos: Cody-Waite reduction by pi/2 and Taylor series in double, every
 * operation rounded separately; the double result is within a few 1e-16
 * relative of the true value, so the float result is the correctly rounded
 * one except in rare near-tie cases. */
#define MTB_PIO2_1 1.5707963267341256       /* pi/2 to 33 bits */
#define MTB_PIO2_2 6.077100506303966e-11    /* next 33 bits */
#define MTB_PIO2_3 2.0222662487959506e-21   /* remainder */
#define MTB_TWO_OVER_PI 0.6366197723675814

static inline float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float exp_own(float x) {
    /* x is clamped for the arithmetic and the special cases are selected at
     * the end; 2^n is applied as (p * 2^a) * 2^b with (a, b) = (n, 0),
     * (1, 127) for n = 128, (n + 64, -64) for n < -126. */
    const float xc = fminf(fmaxf(x, -103.972084f), 88.7228317f);
    const float n = rintf(xc * 1.44269502f);
    float r = fmaf(n, -0.693145752f, xc);
    r = fmaf(n, -1.42860677e-6f, r);
    float p = 1.98412701e-4f;
    p = fmaf(p, r, 1.38888892e-3f);
    p = fmaf(p, r, 8.33333377e-3f);
    p = fmaf(p, r, 4.16666679e-2f);
    p = fmaf(p, r, 1.66666672e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = (int)n;
    const int ea = ni > 127 ? 1 : (ni < -126 ? ni + 64 : ni);
    const int eb = ni > 127 ? 127 : (ni < -126 ? -64 : 0);
    const float y = (p * bits_f32((uint32_t)(ea + 127) << 23)) * bits_f32((uint32_t)(eb + 127) << 23);
    if (x != x) return x;
    if (x > 88.7228317f) return INFINITY;   /* the largest x with a finite result */
    if (x < -103.972084f) return 0.0f;      /* e^x below half the smallest subnormal */
    return y;
}

float orc_expf(float x) { return exp_own(x); }

void orc_sincosf(float x, float* s_out, float* c_out) {
    const double xd = (double)x;
    const double k = rint(xd * MTB_TWO_OVER_PI);
    const double r = ((xd - k * MTB_PIO2_1) - k * MTB_PIO2_2) - k * MTB_PIO2_3;
    const double r2 = r * r;
    /* sin r = r - r^3/3! + ... (to r^19), cos r = 1 - r^2/2! + ... (to r^20) */
    double ps = -1.0 / 121645100408832000.0;
    ps = ps * r2 + 1.0 / 355687428096000.0;
    ps = ps * r2 - 1.0 / 1307674368000.0;
    ps = ps * r2 + 1.0 / 6227020800.0;
    ps = ps * r2 - 1.0 / 39916800.0;
    ps = ps * r2 + 1.0 / 362880.0;
    ps = ps * r2 - 1.0 / 5040.0;
    ps = ps * r2 + 1.0 / 120.0;
    ps = ps * r2 - 1.0 / 6.0;
    ps = ps * r2 + 1.0;
    const double sv = ps * r;
    double pc = 1.0 / 2432902008176640000.0;
    pc = pc * r2 - 1.0 / 6402373705728000.0;
    pc = pc * r2 + 1.0 / 20922789888000.0;
    pc = pc * r2 - 1.0 / 87178291200.0;
    pc = pc * r2 + 1.0 / 479001600.0;
    pc = pc * r2 - 1.0 / 3628800.0;
    pc = pc * r2 + 1.0 / 40320.0;
    pc = pc * r2 - 1.0 / 720.0;
    pc = pc * r2 + 1.0 / 24.0;
    pc = pc * r2 - 0.5;
    pc = pc * r2 + 1.0;
    const double cv = pc;
    const long long q = ((long long)k % 4 + 4) % 4;
    double so, co;
    if (q == 0) { so = sv; co = cv; }
    else if (q == 1) { so = cv; co = -sv; }
    else if (q == 2) { so = -sv; co = -cv; }
    else { so = -cv; co = sv; }
    *s_out = (float)so;
    *c_out = (float)co;
}

/* Sum of float squares in double in the CUDA kernels' order: `threads`
 * strided partial sums (each sequential from 0.0), a xor-butterfly inside
 * each group of 32 (pairs i, i+16, then i, i+8, ... ), then the group totals
 * added in order.  Addition is commutative, so only the tree shape matters. */
static double sum_squares_tree(const float* x, int n, int threads) {
    double part[1024];
    for (int i = 0; i < threads; ++i) {
        double acc = 0.0;
        for (int j = i; j < n; j += threads) acc += (double)(x[j] * x[j]);
        part[i] = acc;
    }
    double tot = 0.0;
    for (int w = 0; w < threads / 32; ++w) {
        double* v = part + 32 * w;
        for (int off = 16; off > 0; off >>= 1)
            for (int i = 0; i < off; ++i) v[i] = v[i] + v[i + off];
        tot += v[0];
    }
    return tot;
}

/* The hidden-row sum of squares, in the kernels' tree (row_rms_scale and
 * block_sum_squares): element squares (float products, widened to double);
 * each 32-element block summed pairwise over adjacent pairs,
 * ((s0 + s1) + (s2 + s3)) + ...; lane l's partial the blocks l, l + 32, ...
 * added in order from 0; the 32 partials combined by one xor butterfly. */
static double sum_squares_blocks(const float* x, int n) {
    double part[32];
    for (int l = 0; l < 32; ++l) part[l] = 0.0;
    for (int b = 0; b < n / 32; ++b) {
        double u[16];
        const float* v = x + 32 * b;
        for (int i = 0; i < 16; ++i) u[i] = (double)(v[2 * i] * v[2 * i]) + (double)(v[2 * i + 1] * v[2 * i + 1]);
        for (int w = 8; w >= 1; w >>= 1)
            for (int i = 0; i < w; ++i) u[i] = u[2 * i] + u[2 * i + 1];
        part[b % 32] += u[0];
    }
    for (int off = 16; off > 0; off >>= 1)
        for (int i = 0; i < off; ++i) part[i] = part[i] + part[i + off];
    return part[0];
}

/* Float xor-butterfly total of 32 values (the kernels' warp sum). */
static float warp_tree_sum(float* v) {
    for (int off = 16; off > 0; off >>= 1)
        for (int i = 0; i < off; ++i) v[i] = v[i] + v[i + off];
    return v[0];
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------ q8_0 */

/* ggml x86 SIMD from_float for Q8_0 (the activation conversion that ggml's CPU
 * mul_mat applies to src1 before every q8_0 dot, called by the reference at
 * src/cpu_projection.cpp:25 and src/cpu_activation.cpp:30). */
void orc_quantize_act_q8(const float* x, int64_t k, void* out_blocks) {
    blk_q8* y = (blk_q8*)out_blocks;
    for (int64_t i = 0; i < k / 32; ++i) {
        const float* v = x + i * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = amax / 127.f;
        y[i].d = f2h(d);
        const float id = (amax != 0.0f) ? 127.f / amax : 0.0f;
        for (int j = 0; j < 32; ++j) y[i].qs[j] = (int8_t)nearbyintf(v[j] * id);
    }
}

/* quantize_row_q8_0_ref: the weight quantiser (gguf.quantize in the
 * reference converter, scripts/convert_moss_transcribe_to_gguf.py:360). */
void orc_quantize_ref_q8(const float* x, int64_t k, void* out_blocks) {
    blk_q8* y = (blk_q8*)out_blocks;
    for (int64_t i = 0; i < k / 32; ++i) {
        const float* v = x + i * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = amax / 127.f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = f2h(d);
        for (int j = 0; j < 32; ++j) y[i].qs[j] = (int8_t)roundf(v[j] * id);
    }
}

/* q8_0 x q8_0 dot: exact integer sum per 32-block, times d_w*d_x (an exact
 * product of two fp16 values), accumulated with one fmaf per block in
 * ascending block order inside each 256-element slice; the slice partials
 * are then added in ascending order.  ggml's x86 path spreads each block over
 * eight lanes instead; the evaluation order here is the one this oracle and
 * the CUDA kernels share (a difference of float rounding order only). */
/* Exact int32 sum of the 32 products of one block pair.  With AVX-512 VNNI
 * (the -march=native build on such a host) it is one u8 x s8 dot of |w| and
 * sign(w) * x, as ggml's x86 path forms it; integer sums are exact, so the
 * result is the scalar loop's. */
#if defined(__AVX512VNNI__) && defined(__AVX512VL__)
#include <immintrin.h>
static inline int block_isum(const int8_t* w, const int8_t* x) {
    const __m256i wv = _mm256_loadu_si256((const __m256i*)w);
    const __m256i xv = _mm256_loadu_si256((const __m256i*)x);
    const __m256i p = _mm256_dpbusd_epi32(_mm256_setzero_si256(), _mm256_sign_epi8(wv, wv), _mm256_sign_epi8(xv, wv));
    __m128i h = _mm_add_epi32(_mm256_castsi256_si128(p), _mm256_extracti128_si256(p, 1));
    h = _mm_add_epi32(h, _mm_shuffle_epi32(h, 0x4e));
    h = _mm_add_epi32(h, _mm_shuffle_epi32(h, 0xb1));
    return _mm_cvtsi128_si32(h);
}
#else
static inline int block_isum(const int8_t* w, const int8_t* x) {
    int isum = 0;
    for (int j = 0; j < 32; ++j) isum += w[j] * x[j];
    return isum;
}
#endif

#if defined(__AVX512VNNI__) && defined(__AVX512VL__)
#define ORC_HAVE_DOT_X8 1
/* dot_q8 of one weight row with 8 activation rows at once (lane t = row t, the
 * rows x_stride blocks apart): per block the 8 exact integer sums (u8 x s8
 * dots of |w| and sign(w) * x, then a horizontal-add tree), and lane by lane
 * the same fmaf(isum, d_w * d_x, acc) per block and slice sums as dot_q8, so
 * every lane equals dot_q8's result bit for bit (the native build only). */
static inline void dot_q8_x8(const blk_q8* w, const blk_q8* x, size_t x_stride, int nb, float* out) {
    __m256 total = _mm256_setzero_ps();
    for (int s0 = 0; s0 < nb; s0 += 8) {
        __m256 acc = _mm256_setzero_ps();
        for (int b = s0; b < s0 + 8 && b < nb; ++b) {
            const __m256i wv = _mm256_loadu_si256((const __m256i*)w[b].qs);
            const __m256i wabs = _mm256_sign_epi8(wv, wv);
            __m256i p[8];
            float dx[8];
            for (int t = 0; t < 8; ++t) {
                const blk_q8* xb = x + (size_t)t * x_stride + b;
                const __m256i xv = _mm256_loadu_si256((const __m256i*)xb->qs);
                p[t] = _mm256_dpbusd_epi32(_mm256_setzero_si256(), wabs, _mm256_sign_epi8(xv, wv));
                dx[t] = h2f(xb->d);
            }
            const __m256i s01 = _mm256_hadd_epi32(p[0], p[1]), s23 = _mm256_hadd_epi32(p[2], p[3]);
            const __m256i s45 = _mm256_hadd_epi32(p[4], p[5]), s67 = _mm256_hadd_epi32(p[6], p[7]);
            const __m256i q0 = _mm256_hadd_epi32(s01, s23), q1 = _mm256_hadd_epi32(s45, s67);
            const __m256i isum = _mm256_add_epi32(_mm256_permute2x128_si256(q0, q1, 0x20),
                                                  _mm256_permute2x128_si256(q0, q1, 0x31));
            const __m256 d = _mm256_mul_ps(_mm256_set1_ps(h2f(w[b].d)), _mm256_loadu_ps(dx));
            acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(isum), d, acc);
        }
        total = _mm256_add_ps(total, acc);
    }
    _mm256_storeu_ps(out, total);
}
#endif

static inline float dot_q8(const blk_q8* w, const blk_q8* x, int nb) {
    float total = 0.0f;
    for (int s0 = 0; s0 < nb; s0 += 8) {
        float acc = 0.0f;
        for (int b = s0; b < s0 + 8 && b < nb; ++b) {
            const float d = h2f(w[b].d) * h2f(x[b].d);
            acc = fmaf((float)block_isum(w[b].qs, x[b].qs), d, acc);
        }
        total = total + acc;
    }
    return total;
}

/* ggml_mul_mat(W q8_0 [n_rows x k], x f32 [T x k]) -> y [T x n_rows]. */
void orc_mul_mat_q8(const void* w_blocks, int n_rows, int k, const float* x, int T, float* y) {
    const int nb = k / 32;
    blk_q8* xq = (blk_q8*)malloc(sizeof(blk_q8) * (size_t)nb * (size_t)T);
    for (int t = 0; t < T; ++t) orc_quantize_act_q8(x + (size_t)t * k, k, xq + (size_t)t * nb);
    const blk_q8* w = (const blk_q8*)w_blocks;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < n_rows; ++n) {
        const blk_q8* row = w + (size_t)n * nb;
        int t = 0;
#ifdef ORC_HAVE_DOT_X8
        for (; t + 8 <= T; t += 8) {
            float o8[8];
            dot_q8_x8(row, xq + (size_t)t * nb, (size_t)nb, nb, o8);
            for (int u = 0; u < 8; ++u) y[(size_t)(t + u) * n_rows + n] = o8[u];
        }
#endif
        for (; t < T; ++t) y[(size_t)t * n_rows + n] = dot_q8(row, xq + (size_t)t * nb, nb);
    }
    free(xq);
}

/* ------------------------------------------------------------------ f16 */

/* F16 weights (configs[2] of the benchmark): ggml's mul_mat with an F16 src0
 * converts src1 to F16 (its vec_dot_type) and accumulates the F16 x F16
 * products in f32.  The products of two fp16 values are exact in f32; the
 * order of the sums is the one this oracle and the CUDA kernels share: each
 * 32-element block one fmaf chain from 0 in ascending order, the blocks of a
 * 256-element slice added in ascending order, then the slices in ascending
 * order (the q8_0 dot's slice structure, with the block sum in place of the
 * integer block sum x scale). */
static inline float dot_f16(const uint16_t* w, const uint16_t* xh, int k) {
    float total = 0.0f;
    for (int s0 = 0; s0 < k; s0 += 256) {
        float acc = 0.0f;
        for (int b = s0; b < s0 + 256 && b < k; b += 32) {
            float bs = 0.0f;
            for (int j = 0; j < 32; ++j) bs = fmaf(h2f(xh[b + j]), h2f(w[b + j]), bs);
            acc = acc + bs;
        }
        total = total + acc;
    }
    return total;
}

/* ggml_mul_mat(W f16 [n_rows x k], x f32 [T x k]) -> y [T x n_rows]; x is
 * rounded to fp16 first (round to nearest even). */
void orc_mul_mat_f16(const void* w_half, int n_rows, int k, const float* x, int T, float* y) {
    uint16_t* xh = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)k * (size_t)T);
    for (size_t i = 0; i < (size_t)k * (size_t)T; ++i) xh[i] = f2h(x[i]);
    const uint16_t* w = (const uint16_t*)w_half;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < n_rows; ++n) {
        const uint16_t* row = w + (size_t)n * k;
        for (int t = 0; t < T; ++t) y[(size_t)t * n_rows + n] = dot_f16(row, xh + (size_t)t * k, k);
    }
    free(xh);
}

/* ------------------------------------------------------------- model */

typedef struct {
    const void *wq, *wk, *wv, *wo, *wgate, *wup, *wdown;
    const float *attn_norm, *q_norm, *k_norm, *ffn_norm;
} orc_layer;

struct orc_model {
    int hidden, n_layers, n_heads, n_kv, head_dim, ffn, vocab;
    int wtype;  /* ORC_Q8_0 or ORC_F16: token_embd and every projection (set by the first of them) */
    float eps, theta;
    const void* token_embd;
    const float* output_norm;
    orc_layer* layers;
};

orc_model* orc_model_create(int hidden, int n_layers, int n_heads, int n_kv_heads, int head_dim,
                            int ffn, int vocab, float rms_eps, float rope_theta) {
    if (hidden <= 0 || hidden % 32 || n_layers <= 0 || n_heads <= 0 || n_kv_heads <= 0 ||
        n_heads % n_kv_heads || head_dim <= 0 || head_dim % 2 || ffn <= 0 || ffn % 32 || vocab <= 0)
        return NULL;
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->hidden = hidden;
    m->n_layers = n_layers;
    m->n_heads = n_heads;
    m->n_kv = n_kv_heads;
    m->head_dim = head_dim;
    m->ffn = ffn;
    m->vocab = vocab;
    m->eps = rms_eps;
    m->theta = rope_theta;
    m->layers = (orc_layer*)calloc((size_t)n_layers, sizeof(orc_layer));
    return m;
}

void orc_model_free(orc_model* m) {
    if (!m) return;
    free(m->layers);
    free(m);
}

int orc_model_set_tensor(orc_model* m, const char* name, const void* data, int type) {
    if (!m || !name || !data) return -1;
    if (!strcmp(name, "token_embd.weight")) {
        if ((type != ORC_Q8_0 && type != ORC_F16) || (m->wtype && type != m->wtype)) return -2;
        m->wtype = type;
        m->token_embd = data;
        return 0;
    }
    if (!strcmp(name, "qwen3.output_norm.weight")) {
        if (type != ORC_F32) return -2;
        m->output_norm = (const float*)data;
        return 0;
    }
    int layer = -1, used = 0;
    char field[64];
    if (sscanf(name, "qwen3.blk.%d.%63s%n", &layer, field, &used) != 2 || layer < 0 ||
        layer >= m->n_layers)
        return -3;
    orc_layer* L = &m->layers[layer];
    struct { const char* n; const void** q; const float** f; } map[] = {
        {"attn_q.weight", &L->wq, NULL},       {"attn_k.weight", &L->wk, NULL},
        {"attn_v.weight", &L->wv, NULL},       {"attn_o.weight", &L->wo, NULL},
        {"ffn_gate.weight", &L->wgate, NULL},  {"ffn_up.weight", &L->wup, NULL},
        {"ffn_down.weight", &L->wdown, NULL},  {"attn_norm.weight", NULL, &L->attn_norm},
        {"attn_q_norm.weight", NULL, &L->q_norm}, {"attn_k_norm.weight", NULL, &L->k_norm},
        {"ffn_norm.weight", NULL, &L->ffn_norm},
    };
    for (size_t i = 0; i < sizeof(map) / sizeof(map[0]); ++i) {
        if (strcmp(field, map[i].n)) continue;
        if (map[i].q) {
            if ((type != ORC_Q8_0 && type != ORC_F16) || (m->wtype && type != m->wtype)) return -2;
            m->wtype = type;
            *map[i].q = data;
        } else {
            if (type != ORC_F32) return -2;
            *map[i].f = (const float*)data;
        }
        return 0;
    }
    return -3;
}

int orc_model_check(const orc_model* m) {
    if (!m || !m->token_embd || !m->output_norm) return -1;
    for (int l = 0; l < m->n_layers; ++l) {
        const orc_layer* L = &m->layers[l];
        if (!L->wq || !L->wk || !L->wv || !L->wo || !L->wgate || !L->wup || !L->wdown ||
            !L->attn_norm || !L->q_norm || !L->k_norm || !L->ffn_norm)
            return -2 - l;
    }
    return 0;
}

/* The model's projection: q8_0 or f16 weights. */
static void mul_mat_w(const orc_model* m, const void* w, int n_rows, int k, const float* x, int T, float* y) {
    if (m->wtype == ORC_F16)
        orc_mul_mat_f16(w, n_rows, k, x, T, y);
    else
        orc_mul_mat_q8(w, n_rows, k, x, T, y);
}

/* ------------------------------------------------------------- decoder */

struct orc_decoder {
    const orc_model* m;
    int max_seq, past, kv_fp16;
    float* k; /* [layer][pos][n_kv][hd] */
    float* v;
};

orc_decoder* orc_decoder_create(const orc_model* m, int max_seq, int kv_fp16) {
    if (!m || orc_model_check(m) || max_seq <= 0) return NULL;
    orc_decoder* d = (orc_decoder*)calloc(1, sizeof(orc_decoder));
    d->m = m;
    d->max_seq = max_seq;
    d->kv_fp16 = kv_fp16;
    const size_t n = (size_t)m->n_layers * (size_t)max_seq * (size_t)m->n_kv * (size_t)m->head_dim;
    d->k = (float*)calloc(n, sizeof(float));
    d->v = (float*)calloc(n, sizeof(float));
    if (!d->k || !d->v) {
        orc_decoder_free(d);
        return NULL;
    }
    return d;
}

void orc_decoder_free(orc_decoder* d) {
    if (!d) return;
    free(d->k);
    free(d->v);
    free(d);
}

int orc_decoder_past_len(const orc_decoder* d) { return d ? d->past : -1; }
/* src/qwen3_decoder.cpp:87-89: stale cache bytes beyond past_len are never read. */
void orc_decoder_reset(orc_decoder* d) {
    if (d) d->past = 0;
}
/* src/cpu_speculative.cpp:22-24 */
int orc_decoder_rewind(orc_decoder* d, int position) {
    if (!d || position < 0 || position > d->past) return -1;
    d->past = position;
    return 0;
}

static inline size_t kv_index(const orc_decoder* d, int layer, int pos) {
    const orc_model* m = d->m;
    return (((size_t)layer * d->max_seq + pos) * m->n_kv) * m->head_dim;
}

int orc_decoder_kv_read(const orc_decoder* d, int layer, int which, int pos0, int n_pos, float* out) {
    if (!d || layer < 0 || layer >= d->m->n_layers || pos0 < 0 || n_pos < 0 || pos0 + n_pos > d->max_seq)
        return -1;
    const float* src = (which ? d->v : d->k) + kv_index(d, layer, pos0);
    memcpy(out, src, sizeof(float) * (size_t)n_pos * d->m->n_kv * d->m->head_dim);
    return 0;
}

int orc_decoder_kv_write(orc_decoder* d, int layer, int which, int pos0, int n_pos, const float* in) {
    if (!d || layer < 0 || layer >= d->m->n_layers || pos0 < 0 || n_pos < 0 || pos0 + n_pos > d->max_seq)
        return -1;
    float* dst = (which ? d->v : d->k) + kv_index(d, layer, pos0);
    const size_t n = (size_t)n_pos * d->m->n_kv * d->m->head_dim;
    for (size_t i = 0; i < n; ++i) dst[i] = d->kv_fp16 ? round_f16(in[i]) : in[i];
    return 0;
}

static inline uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

float orc_synthetic_kv_value(uint32_t seed, int layer, int which, int pos, int head, int dim) {
    uint32_t h = mix32(seed + 0x9E3779B9u * (uint32_t)(layer * 2 + which + 1));
    h = mix32(h ^ ((uint32_t)pos * 0x85EBCA6Bu));
    h = mix32(h ^ ((uint32_t)(head * 1024 + dim) * 0xC2B2AE35u));
    const uint32_t g = mix32(h ^ 0x68E31DA4u);
    const int s = (int)(h & 0xffffu) + (int)(h >> 16) + (int)(g & 0xffffu) + (int)(g >> 16) - 131070;
    return round_f16((float)s * 2.642912e-05f);
}

int orc_decoder_fill_synthetic_kv(orc_decoder* d, int n_pos, uint32_t seed) {
    if (!d || n_pos < 0 || n_pos > d->max_seq) return -1;
    const orc_model* m = d->m;
#pragma omp parallel for schedule(static)
    for (int l = 0; l < m->n_layers; ++l)
        for (int p = 0; p < n_pos; ++p)
            for (int h = 0; h < m->n_kv; ++h)
                for (int e = 0; e < m->head_dim; ++e) {
                    const size_t i = kv_index(d, l, p) + (size_t)h * m->head_dim + e;
                    d->k[i] = orc_synthetic_kv_value(seed, l, 0, p, h, e);
                    d->v[i] = orc_synthetic_kv_value(seed, l, 1, p, h, e);
                }
    d->past = n_pos;
    return 0;
}

/* ggml rms_norm followed by ggml_mul with the weight (src/qwen3.cpp:27-30):
 * float squares summed in double, mean as float, 1/sqrtf(mean + eps), then
 * (x * scale) * w.  `threads` fixes the summation tree: 0 for hidden rows
 * (sum_squares_blocks); 32 for per-head q/k norms (each of 32 partials adds
 * elements i, i + 32, i + 64, i + 96 in order, then one butterfly). */
static void rms_norm_mul(const float* x, const float* w, int n, float eps, float* y, int threads) {
    const double sum = threads ? sum_squares_tree(x, n, threads) : sum_squares_blocks(x, n);
    const float mean = (float)(sum / n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; ++i) y[i] = (x[i] * scale) * w[i];
}

/* ggml_rope_ext NEOX with freq_scale 1, ext_factor 0, attn_factor 1
 * (src/qwen3.cpp:109-118). */
static void rope_neox(float* x, int n_dims, int pos, float base) {
    const float theta_scale = powf(base, -2.0f / (float)n_dims);
    float theta = (float)pos;
    const int half = n_dims / 2;
    for (int i = 0; i < half; ++i) {
        float s, c;
        orc_sincosf(theta, &s, &c);
        const float x0 = x[i], x1 = x[i + half];
        x[i] = x0 * c - x1 * s;
        x[i + half] = x0 * s + x1 * c;
        theta *= theta_scale;
    }
}

static inline float silu(float x) { return x / (1.0f + exp_own(-x)); }

/* One query row's attention in this oracle's (and the CUDA kernels') order:
 * positions j < valid of K and V at kbase + j * stride / vbase + j * stride.
 * Each score q.k is two sequential fmaf chains (even and odd dims) added;
 * softmax(s * scale) per 64-position chunk (chunk max m_c, e = exp(s - m_c),
 * the pair sums e[p] + e[p + 32] then a 32-value xor butterfly for l_c, each
 * context dim one fmaf chain o_c); the chunks merged with weights exp(m_c - M)
 * in chunk order, o = sum w_c o_c / sum w_c l_c. */
/* One 64-position chunk c of one attention row, from K transposed [dim][kt_stride]
 * and V rows `stride` apart: the chunk maximum, the chunk sum (pair sums, then
 * the 32-lane tree) and the unnormalised context, exactly as attn_row_chunked
 * computes them for that chunk. */
static void attn_chunk_stats(const float* restrict qh, const float* restrict kT, size_t kt_stride,
                             const float* restrict vbase, size_t stride, int valid, int hd, float scale, int c,
                             float* restrict cm, float* restrict cl, float* restrict oc) {
    const int n_pos = valid - c * 64 < 64 ? valid - c * 64 : 64;
    float sc[64], e[64], ae[64], ao[64], pair[32];
    for (int p = 0; p < 64; ++p) ae[p] = ao[p] = 0.0f;
    for (int e2 = 0; e2 < hd; e2 += 2) {
        const float* k0 = kT + (size_t)e2 * kt_stride + (size_t)c * 64;
        const float* k1 = kT + (size_t)(e2 + 1) * kt_stride + (size_t)c * 64;
        for (int p = 0; p < n_pos; ++p) {
            ae[p] = fmaf(qh[e2], k0[p], ae[p]);
            ao[p] = fmaf(qh[e2 + 1], k1[p], ao[p]);
        }
    }
    float mx = -INFINITY;
    for (int p = 0; p < 64; ++p) {
        sc[p] = p < n_pos ? (ae[p] + ao[p]) * scale : -INFINITY;
        mx = fmaxf(mx, sc[p]);
    }
    for (int p = 0; p < 64; ++p) e[p] = sc[p] == -INFINITY ? 0.0f : exp_own(sc[p] - mx);
    for (int p = 0; p < 32; ++p) pair[p] = e[p] + e[p + 32];
    *cm = mx;
    *cl = warp_tree_sum(pair);
    for (int e2 = 0; e2 < hd; ++e2) oc[e2] = 0.0f;
    for (int p = 0; p < n_pos; ++p) {
        const float* vp = vbase + (size_t)(c * 64 + p) * stride;
        const float ep = e[p];
        for (int e2 = 0; e2 < hd; ++e2) oc[e2] = fmaf(ep, vp[e2], oc[e2]);
    }
}

/* The merge of attn_row_chunked: weights exp(m_c - M) in chunk order. */
static void attn_merge_chunks(const float* cm, const float* cl, const float* co, int n_chunks, int hd, float* oh) {
    float M = -INFINITY;
    for (int c = 0; c < n_chunks; ++c) M = fmaxf(M, cm[c]);
    float Ls = 0.0f;
    for (int e2 = 0; e2 < hd; ++e2) oh[e2] = 0.0f;
    for (int c = 0; c < n_chunks; ++c) {
        const float wgt = exp_own(cm[c] - M);
        Ls = fmaf(wgt, cl[c], Ls);
        const float* oc = co + (size_t)c * hd;
        for (int e2 = 0; e2 < hd; ++e2) oh[e2] = fmaf(wgt, oc[e2], oh[e2]);
    }
    for (int e2 = 0; e2 < hd; ++e2) oh[e2] = oh[e2] / Ls;
}

static void attn_row_chunked(const float* qh, const float* kbase, const float* vbase, size_t stride, int valid, int hd,
                             float scale, float* oh, const float* kT, size_t kt_stride) {
    /* The loops run position-inner / dim-inner so that the compiler can keep
     * many independent chains in vector lanes; every chain is still the same
     * sequence of fmaf operations as described above. */
    enum { MAXD = 256 };
    const int n_chunks = (valid + 63) / 64;
    float* cm = (float*)malloc(sizeof(float) * (size_t)n_chunks);
    float* cl = (float*)malloc(sizeof(float) * (size_t)n_chunks);
    float* co = (float*)malloc(sizeof(float) * (size_t)n_chunks * hd);
    float kt[MAXD][64];
    if (hd > MAXD) abort();
    for (int c = 0; c < n_chunks; ++c) {
        const int n_pos = valid - c * 64 < 64 ? valid - c * 64 : 64;
        float sc[64], e[64], ae[64], ao[64];
        if (!kT)
            for (int p = 0; p < n_pos; ++p) {
                const float* kj = kbase + (size_t)(c * 64 + p) * stride;
                for (int e2 = 0; e2 < hd; ++e2) kt[e2][p] = kj[e2];
            }
        for (int p = 0; p < 64; ++p) ae[p] = ao[p] = 0.0f;
        for (int e2 = 0; e2 < hd; e2 += 2) {
            /* K of this chunk by dim: the caller's transposed copy, or the local one. */
            const float* k0 = kT ? kT + (size_t)e2 * kt_stride + (size_t)c * 64 : kt[e2];
            const float* k1 = kT ? kT + (size_t)(e2 + 1) * kt_stride + (size_t)c * 64 : kt[e2 + 1];
            for (int p = 0; p < n_pos; ++p) {
                ae[p] = fmaf(qh[e2], k0[p], ae[p]);
                ao[p] = fmaf(qh[e2 + 1], k1[p], ao[p]);
            }
        }
        float mx = -INFINITY;
        for (int p = 0; p < 64; ++p) {
            sc[p] = p < n_pos ? (ae[p] + ao[p]) * scale : -INFINITY;
            mx = fmaxf(mx, sc[p]);
        }
        float pair[32];
        for (int p = 0; p < 64; ++p) e[p] = sc[p] == -INFINITY ? 0.0f : exp_own(sc[p] - mx);
        for (int p = 0; p < 32; ++p) pair[p] = e[p] + e[p + 32];
        cm[c] = mx;
        cl[c] = warp_tree_sum(pair);
        float* oc = co + (size_t)c * hd;
        for (int e2 = 0; e2 < hd; ++e2) oc[e2] = 0.0f;
        for (int p = 0; p < n_pos; ++p) {
            const float* vp = vbase + (size_t)(c * 64 + p) * stride;
            const float ep = e[p];
            for (int e2 = 0; e2 < hd; ++e2) oc[e2] = fmaf(ep, vp[e2], oc[e2]);
        }
    }
    float M = -INFINITY;
    for (int c = 0; c < n_chunks; ++c) M = fmaxf(M, cm[c]);
    float Ls = 0.0f;
    for (int e2 = 0; e2 < hd; ++e2) oh[e2] = 0.0f;
    for (int c = 0; c < n_chunks; ++c) {
        const float wgt = exp_own(cm[c] - M);
        Ls = fmaf(wgt, cl[c], Ls);
        const float* oc = co + (size_t)c * hd;
        for (int e2 = 0; e2 < hd; ++e2) oh[e2] = fmaf(wgt, oc[e2], oh[e2]);
    }
    for (int e2 = 0; e2 < hd; ++e2) oh[e2] = oh[e2] / Ls;
    free(cm); free(cl); free(co);
}

int orc_decoder_run(orc_decoder* d, const float* embeds, int T, float* out_hidden) {
    if (!d || !embeds || T <= 0 || d->past + T > d->max_seq) return -1;
    const orc_model* m = d->m;
    const int H = m->hidden, hd = m->head_dim, nh = m->n_heads, nkv = m->n_kv, F = m->ffn;
    const int past = d->past, kv = past + T, group = nh / nkv;
    const int qd = nh * hd, kd = nkv * hd;
    float* x = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* xn = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* q = (float*)malloc(sizeof(float) * (size_t)T * qd);
    float* k = (float*)malloc(sizeof(float) * (size_t)T * kd);
    float* v = (float*)malloc(sizeof(float) * (size_t)T * kd);
    float* o = (float*)malloc(sizeof(float) * (size_t)T * qd);
    float* proj = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* g = (float*)malloc(sizeof(float) * (size_t)T * F);
    float* u = (float*)malloc(sizeof(float) * (size_t)T * F);
    const int kvp = (kv + 63) / 64 * 64;
    float* kT = (float*)malloc(sizeof(float) * (size_t)kd * kvp);
    const int max_chunks = kvp / 64;
    const size_t row_stats = (size_t)nh * max_chunks * (hd + 2) * sizeof(float);
#ifndef ORC_ATTN_STATS_BYTES
#define ORC_ATTN_STATS_BYTES ((size_t)256 * 1024 * 1024)
#endif
    int tb = (int)(ORC_ATTN_STATS_BYTES / row_stats);
    tb = tb < 1 ? 1 : (tb > T ? T : tb);
    float* a_cm = (float*)malloc(sizeof(float) * (size_t)tb * nh * max_chunks);
    float* a_cl = (float*)malloc(sizeof(float) * (size_t)tb * nh * max_chunks);
    float* a_co = (float*)malloc(sizeof(float) * (size_t)tb * nh * max_chunks * hd);
    memcpy(x, embeds, sizeof(float) * (size_t)T * H);
    const float scale = 1.0f / sqrtf((float)hd);

    for (int l = 0; l < m->n_layers; ++l) {
        const orc_layer* L = &m->layers[l];
        for (int t = 0; t < T; ++t) rms_norm_mul(x + (size_t)t * H, L->attn_norm, H, m->eps, xn + (size_t)t * H, 0);
        mul_mat_w(d->m, L->wq, qd, H, xn, T, q);
        mul_mat_w(d->m, L->wk, kd, H, xn, T, k);
        mul_mat_w(d->m, L->wv, kd, H, xn, T, v);
        for (int t = 0; t < T; ++t) {
            for (int h = 0; h < nh; ++h) {
                float* qh = q + (size_t)t * qd + (size_t)h * hd;
                rms_norm_mul(qh, L->q_norm, hd, m->eps, qh, 32);
                rope_neox(qh, hd, past + t, m->theta);
            }
            for (int h = 0; h < nkv; ++h) {
                float* kh = k + (size_t)t * kd + (size_t)h * hd;
                rms_norm_mul(kh, L->k_norm, hd, m->eps, kh, 32);
                rope_neox(kh, hd, past + t, m->theta);
            }
            /* KV store at past+t (src/qwen3.cpp:123-140). */
            float* kdst = d->k + kv_index(d, l, past + t);
            float* vdst = d->v + kv_index(d, l, past + t);
            for (int i = 0; i < kd; ++i) {
                kdst[i] = d->kv_fp16 ? round_f16(k[(size_t)t * kd + i]) : k[(size_t)t * kd + i];
                vdst[i] = d->kv_fp16 ? round_f16(v[(size_t)t * kd + i]) : v[(size_t)t * kd + i];
            }
        }
        /* GQA attention with a causal mask when T > 1 (src/qwen3.cpp:158-189,
         * src/qwen3_decoder.cpp:142-148): query row t sees positions
         * [0, past + t], context over that valid length only
         * (src/cpu_context.cpp:13-33).  Each score q.k is two sequential fmaf
         * chains (even and odd dims) added.  softmax(s * 1/sqrt(hd)) is evaluated
         * per 64-position chunk (chunk max m_c, e = exp(s - m_c), chunk sum l_c
         * and context o_c) and the chunks are merged with weights
         * exp(m_c - M); the same function as one softmax over the row, in the
         * evaluation order shared with the CUDA kernels. */
        /* K transposed once per layer and KV head ([kv head][dim][position]),
         * shared by every row and query head of the group. */
        const float* kl = d->k + kv_index(d, l, 0);
#pragma omp parallel for collapse(2) schedule(static)
        for (int h = 0; h < nkv; ++h)
            for (int p0 = 0; p0 < kv; p0 += 64) {  /* 64 positions x hd dims at a time (cache-resident) */
                const int p1 = p0 + 64 < kv ? p0 + 64 : kv;
                for (int e2 = 0; e2 < hd; ++e2) {
                    float* dst = kT + ((size_t)h * hd + e2) * kvp;
                    for (int p = p0; p < p1; ++p) dst[p] = kl[(size_t)p * kd + (size_t)h * hd + e2];
                }
            }
        /* The chunk statistics of every row and head, one (KV head, chunk) per
         * work item: its K and V rows are read once for all rows and query heads
         * of the group.  Then each row's chunks are merged in order.  The same
         * operations as attn_row_chunked, row by row.  Rows go in blocks of tb
         * (the statistics of a block stay below ~256 MB for long prompts). */
        const float* vl = d->v + kv_index(d, l, 0);
        for (int t0 = 0; t0 < T; t0 += tb) {
            const int t1 = t0 + tb < T ? t0 + tb : T;
            const int n_chunks_blk = (past + t1 + 63) / 64;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
            for (int kvh = 0; kvh < nkv; ++kvh)
                for (int c = 0; c < n_chunks_blk; ++c)
                    for (int t = t0; t < t1; ++t) {
                        const int valid = past + t + 1;
                        if (c * 64 >= valid) continue;
                        for (int h = kvh * group; h < (kvh + 1) * group; ++h) {
                            const size_t it = (size_t)(t - t0) * nh + h;
                            attn_chunk_stats(q + (size_t)t * qd + (size_t)h * hd, kT + (size_t)kvh * hd * kvp, kvp,
                                             vl + (size_t)kvh * hd, (size_t)kd, valid, hd, scale, c,
                                             a_cm + it * max_chunks + c, a_cl + it * max_chunks + c,
                                             a_co + (it * max_chunks + c) * hd);
                        }
                    }
#pragma omp parallel for collapse(2) schedule(static)
            for (int t = t0; t < t1; ++t)
                for (int h = 0; h < nh; ++h) {
                    const size_t it = (size_t)(t - t0) * nh + h;
                    attn_merge_chunks(a_cm + it * max_chunks, a_cl + it * max_chunks, a_co + it * max_chunks * hd,
                                      (past + t + 1 + 63) / 64, hd, o + (size_t)t * qd + (size_t)h * hd);
                }
        }
        mul_mat_w(d->m, L->wo, H, qd, o, T, proj);
        for (size_t i = 0; i < (size_t)T * H; ++i) x[i] = x[i] + proj[i];
        for (int t = 0; t < T; ++t) rms_norm_mul(x + (size_t)t * H, L->ffn_norm, H, m->eps, xn + (size_t)t * H, 0);
        mul_mat_w(d->m, L->wgate, F, H, xn, T, g);
        mul_mat_w(d->m, L->wup, F, H, xn, T, u);
        for (size_t i = 0; i < (size_t)T * F; ++i) g[i] = silu(g[i]) * u[i];
        mul_mat_w(d->m, L->wdown, H, F, g, T, proj);
        for (size_t i = 0; i < (size_t)T * H; ++i) x[i] = x[i] + proj[i];
    }
    for (int t = 0; t < T; ++t) rms_norm_mul(x + (size_t)t * H, m->output_norm, H, m->eps, out_hidden + (size_t)t * H, 0);
    d->past = kv;
    free(x); free(xn); free(q); free(k); free(v); free(o); free(proj); free(g); free(u); free(kT);
    free(a_cm); free(a_cl); free(a_co);
    return 0;
}

/* src/qwen3_decoder.cpp:174-206: token_embd (q8_0 or f16) @ hidden, one row. */
void orc_decoder_logits(const orc_decoder* d, const float* hidden_row, float* logits) {
    mul_mat_w(d->m, d->m->token_embd, d->m->vocab, d->m->hidden, hidden_row, 1, logits);
}

/* src/generate.cpp:33-66: get_rows / to_float of q8_0 rows (y = d * q) or
 * f16 rows (exact). */
int orc_embed_rows(const orc_model* m, const int32_t* ids, int n, float* out) {
    if (!m || !ids || n <= 0) return -1;
    if (m->wtype == ORC_F16) {
        const uint16_t* tok = (const uint16_t*)m->token_embd;
        for (int p = 0; p < n; ++p) {
            if (ids[p] < 0 || ids[p] >= m->vocab) return -2;
            for (int i = 0; i < m->hidden; ++i)
                out[(size_t)p * m->hidden + i] = h2f(tok[(size_t)ids[p] * m->hidden + i]);
        }
        return 0;
    }
    const int nb = m->hidden / 32;
    const blk_q8* tok = (const blk_q8*)m->token_embd;
    for (int p = 0; p < n; ++p) {
        if (ids[p] < 0 || ids[p] >= m->vocab) return -2;
        const blk_q8* row = tok + (size_t)ids[p] * nb;
        for (int b = 0; b < nb; ++b) {
            const float dd = h2f(row[b].d);
            for (int j = 0; j < 32; ++j) out[(size_t)p * m->hidden + b * 32 + j] = (float)row[b].qs[j] * dd;
        }
    }
    return 0;
}

/* ------------------------------------------------------------- controller */

/* src/cpu_speculative.cpp:27-38 with the n-gram range made explicit. */
int orc_ngram_draft(const int32_t* h, int n, int maximum, int n_min, int n_max, int32_t* out) {
    /* n < 3 is the reference's guard for its fixed n_min = 2; n_min + 1 is its
     * generalisation (the loop below needs a suffix plus one earlier token). */
    if (maximum <= 0 || n < 2 || n < n_min + 1) return 0;
    int top = n_max < n - 1 ? n_max : n - 1;
    for (int size = top; size >= n_min; --size) {
        for (int start = n - size - 1; start >= 0; --start) {
            if (!memcmp(h + n - size, h + start, sizeof(int32_t) * (size_t)size)) {
                const int begin = start + size;
                int count = n - begin;
                if (count > maximum) count = maximum;
                memcpy(out, h + begin, sizeof(int32_t) * (size_t)count);
                return count;
            }
        }
    }
    return 0;
}

/* src/cpu_speculative.cpp:39-50: first max with strict >, optional penalty
 * over the set of the last 100 ids. */
int orc_greedy_choice(const float* raw, int vocab, const int32_t* h, int n, float penalty) {
    if (vocab <= 0) return -1;
    if (penalty <= 1.f) {
        int best = 0;
        for (int i = 1; i < vocab; ++i)
            if (raw[i] > raw[best]) best = i;
        return best;
    }
    float* adj = (float*)malloc(sizeof(float) * (size_t)vocab);
    memcpy(adj, raw, sizeof(float) * (size_t)vocab);
    unsigned char* seen = (unsigned char*)calloc((size_t)vocab, 1);
    for (int i = n > 100 ? n - 100 : 0; i < n; ++i) {
        const int32_t id = h[i];
        if (id < 0 || id >= vocab || seen[id]) continue;
        seen[id] = 1;
        adj[id] = adj[id] > 0 ? adj[id] / penalty : adj[id] * penalty;
    }
    int best = 0;
    for (int i = 1; i < vocab; ++i)
        if (adj[i] > adj[best]) best = i;
    free(adj);
    free(seen);
    return best;
}

static float clamp_penalty(float p) { return p < 1.f ? 1.f : (p > 1.5f ? 1.5f : p); }

/* src/cpu_speculative.cpp:68-147 */
int orc_spec_generate(orc_decoder* d, const float* fused, int seq, int max_new, int eos,
                      int k_max, int n_min, int n_max, float penalty,
                      int32_t* out_ids, orc_counters* c,
                      orc_draft_fn draft, orc_commit_fn commit, void* user) {
    orc_counters local;
    if (!c) c = &local;
    memset(c, 0, sizeof(*c));
    if (!d || !fused || seq <= 0 || max_new <= 0 || !out_ids || k_max < 0 || n_min < 1 || n_max < n_min) return -1;
    const orc_model* m = d->m;
    const int H = m->hidden, V = m->vocab;
    penalty = clamp_penalty(penalty);
    d->past = 0;
    float* hid = (float*)malloc(sizeof(float) * (size_t)seq * H);
    if (orc_decoder_run(d, fused, seq, hid)) { free(hid); return -1; }
    float* raw = (float*)malloc(sizeof(float) * (size_t)V);
    orc_decoder_logits(d, hid + (size_t)(seq - 1) * H, raw);
    free(hid);
    int n = 0, stop = 0;
    int32_t* proposal = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k_max > 0 ? k_max : 1));
    int32_t* inputs = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k_max + 1));
    float* emb = (float*)malloc(sizeof(float) * (size_t)(k_max + 1) * H);
    float* h = (float*)malloc(sizeof(float) * (size_t)(k_max + 1) * H);
#define EMIT(id)                                   \
    do {                                           \
        out_ids[n++] = (id);                       \
        if ((id) == eos) stop = 1;                 \
        else if (n >= max_new) stop = 2;           \
    } while (0)
    int err = 0;
    while (!stop) {
        const int seed = orc_greedy_choice(raw, V, out_ids, n, penalty);
        EMIT(seed);
        if (stop) {
            if (commit) commit(user, out_ids, n, d->past, 1);
            break;
        }
        const int before = d->past;
        int budget = k_max;
        if (max_new - n < budget) budget = max_new - n;
        if (d->max_seq - d->past - 1 < budget) budget = d->max_seq - d->past - 1;
        if (budget < 0) budget = 0;
        int np = draft ? draft(user, out_ids, n, budget, proposal)
                       : orc_ngram_draft(out_ids, n, budget, n_min, n_max, proposal);
        if (np > budget) np = budget;
        if (np < 0) np = 0;
        for (int i = 0; i < np; ++i)
            if (proposal[i] < 0 || proposal[i] >= V) { err = 1; break; }
        if (err) break;
        inputs[0] = seed;
        memcpy(inputs + 1, proposal, sizeof(int32_t) * (size_t)np);
        const int T = 1 + np;
        if (orc_embed_rows(m, inputs, T, emb)) { err = 1; break; }
        if (T > d->max_seq - d->past || orc_decoder_run(d, emb, T, h)) { err = 1; break; }
        c->target_calls++;
        c->drafted_calls += np > 0;
        c->proposed += np;
        c->target_input_tokens += T;
        orc_decoder_logits(d, h, raw);
        int keep = 1;
        for (int i = 0; i < np; ++i) {
            if (proposal[i] != orc_greedy_choice(raw, V, out_ids, n, penalty)) break;
            c->accepted++;
            EMIT(proposal[i]);
            if (stop) break; /* the terminating token is not evaluated */
            ++keep;
            orc_decoder_logits(d, h + (size_t)(i + 1) * H, raw);
        }
        const int position = before + keep;
        if (d->past != position) {
            if (orc_decoder_rewind(d, position)) { err = 1; break; }
            c->rewinds++;
        }
        if (commit) commit(user, out_ids, n, d->past, stop != 0);
    }
#undef EMIT
    c->stop_reason = err ? 0 : stop;
    free(raw); free(proposal); free(inputs); free(emb); free(h);
    return err ? -1 : n;
}

/* src/generate.cpp:235-326 (serial greedy path). */
int orc_greedy_generate(orc_decoder* d, const float* fused, int seq, int max_new, int eos,
                        float penalty, int32_t* out_ids) {
    if (!d || !fused || seq <= 0 || max_new <= 0 || !out_ids) return -1;
    const orc_model* m = d->m;
    const int H = m->hidden, V = m->vocab;
    penalty = clamp_penalty(penalty);
    d->past = 0;
    float* hid = (float*)malloc(sizeof(float) * (size_t)seq * H);
    if (orc_decoder_run(d, fused, seq, hid)) { free(hid); return -1; }
    float* raw = (float*)malloc(sizeof(float) * (size_t)V);
    orc_decoder_logits(d, hid + (size_t)(seq - 1) * H, raw);
    free(hid);
    float* emb = (float*)malloc(sizeof(float) * (size_t)H);
    float* h = (float*)malloc(sizeof(float) * (size_t)H);
    int n = 0, rc = 0;
    for (;;) {
        const int t = orc_greedy_choice(raw, V, out_ids, n, penalty);
        out_ids[n++] = t;
        if (t == eos || n >= max_new) break;
        if (orc_embed_rows(m, &t, 1, emb) || orc_decoder_run(d, emb, 1, h)) { rc = -1; break; }
        orc_decoder_logits(d, h, raw);
    }
    free(raw); free(emb); free(h);
    return rc ? -1 : n;
}

/* ============================================================ reference order
 *
 * A second restatement of the decoder, TEST ONLY, in the reference's own
 * evaluation order rather than the order this oracle shares with the CUDA
 * kernels.  Its only use is to bound how far that shared order sits from the
 * reference's arithmetic (tests/test_reference_order.py).  ggml itself is
 * absent here, so the ggml steps below are restated from its published x86
 * source at the pinned commit (AVX2 q8_0 dot, AVX-512 f32 dot) and cannot be
 * checked bit for bit against the reference binary.
 *
 *  - rms_norm: float squares added in double in element order
 *    (ggml_compute_forward_rms_norm_f32), 1/sqrtf(mean + eps), (x*s)*w;
 *  - q8_0 x q8_0 dot (ggml_vec_dot_q8_0_q8_0, AVX2): eight float lanes, lane j
 *    the int32 sum of the products of bytes 4j..4j+3 of a block; per block
 *    lane_j = fmaf(d_w*d_x, (float)isum_j, lane_j); then hsum_float_8;
 *  - f32 dot (ggml_vec_dot_f32, AVX-512): four 16-lane fmaf accumulators over
 *    64-element steps, reduced 0+2, 1+3, 0+1, then the lanes 8-by-8, 4, 2, 1;
 *    the tail of n % 64 elements added in double;
 *  - attention (src/qwen3.cpp:158-189): scores = K.q over every cached
 *    position, ggml_soft_max_ext / cpu_decode_softmax (src/cpu_softmax.cpp:29-36):
 *    s*scale (+ -inf past the causal limit), max, e = expf(s - max) with the sum
 *    in double, p = e * (float)(1/sum); context = P.V over the valid length
 *    (src/cpu_context.cpp:29, ggml_vec_dot_f32);
 *  - RoPE with libm sinf/cosf, SiLU x / (1 + expf(-x)) with libm expf.
 */

static float ref_hsum8(const float* a) {
    /* hsum_float_8: high 128 + low 128, movehl, movehdup */
    float r[4];
    for (int j = 0; j < 4; ++j) r[j] = a[j + 4] + a[j];
    const float r0 = r[0] + r[2], r1 = r[1] + r[3];
    return r0 + r1;
}

static float ref_dot_q8(const blk_q8* w, const blk_q8* x, int nb) {
    float acc[8] = {0};
    for (int b = 0; b < nb; ++b) {
        const float d = h2f(w[b].d) * h2f(x[b].d);
        for (int j = 0; j < 8; ++j) {
            int s = 0;
            for (int u = 0; u < 4; ++u) s += w[b].qs[4 * j + u] * x[b].qs[4 * j + u];
            acc[j] = fmaf(d, (float)s, acc[j]);
        }
    }
    return ref_hsum8(acc);
}

static void ref_mul_mat_q8(const void* w_blocks, int n_rows, int k, const float* x, int T, float* y) {
    const int nb = k / 32;
    blk_q8* xq = (blk_q8*)malloc(sizeof(blk_q8) * (size_t)nb * (size_t)T);
    for (int t = 0; t < T; ++t) orc_quantize_act_q8(x + (size_t)t * k, k, xq + (size_t)t * nb);
    const blk_q8* w = (const blk_q8*)w_blocks;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < n_rows; ++n)
        for (int t = 0; t < T; ++t) y[(size_t)t * n_rows + n] = ref_dot_q8(w + (size_t)n * nb, xq + (size_t)t * nb, nb);
    free(xq);
}

/* ggml_vec_dot_f32 with strided operands (x[i * sx], y[i * sy]). */
static float ref_dot_f32(int n, const float* x, size_t sx, const float* y, size_t sy) {
    const int np = n & ~63;
    float acc[4][16];
    memset(acc, 0, sizeof(acc));
    for (int i = 0; i < np; i += 64)
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 16; ++l) {
                const int e = i + 16 * j + l;
                acc[j][l] = fmaf(x[(size_t)e * sx], y[(size_t)e * sy], acc[j][l]);
            }
    double sum = 0.0;
    if (np > 0) {
        float v[16];
        for (int l = 0; l < 16; ++l) {
            const float a = acc[0][l] + acc[2][l], b = acc[1][l] + acc[3][l];
            v[l] = a + b;
        }
        for (int w = 8; w > 0; w >>= 1)
            for (int l = 0; l < w; ++l) v[l] = v[l] + v[l + w];
        sum = v[0];
    }
    for (int i = np; i < n; ++i) sum += (double)(x[(size_t)i * sx] * y[(size_t)i * sy]);
    return (float)sum;
}

static void ref_rms_norm_mul(const float* x, const float* w, int n, float eps, float* y) {
    double sum = 0.0;
    for (int i = 0; i < n; ++i) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; ++i) y[i] = (x[i] * scale) * w[i];
}

static void ref_rope_neox(float* x, int n_dims, int pos, float base) {
    const float theta_scale = powf(base, -2.0f / (float)n_dims);
    float theta = (float)pos;
    const int half = n_dims / 2;
    for (int i = 0; i < half; ++i) {
        const float c = cosf(theta), s = sinf(theta);
        const float x0 = x[i], x1 = x[i + half];
        x[i] = x0 * c - x1 * s;
        x[i + half] = x0 * s + x1 * c;
        theta *= theta_scale;
    }
}

/* One query row's attention in the reference's order: scores over the row
 * (ggml_vec_dot_f32), s * scale, max, e = expf(s - max) summed in double,
 * p = e * (float)(1 / sum), then each context dim ggml_vec_dot_f32 of the V
 * column and p over the valid length.  Positions past `valid` (the causal
 * mask's -inf) contribute exact zeros and are left out. */
static void attn_row_ref(const float* qh, const float* kbase, const float* vbase, size_t stride, int valid, int hd,
                         float scale, float* oh) {
    float* p = (float*)malloc(sizeof(float) * (size_t)valid);
    float mx = -INFINITY;
    for (int j = 0; j < valid; ++j) {
        p[j] = ref_dot_f32(hd, kbase + (size_t)j * stride, 1, qh, 1) * scale;
        mx = fmaxf(mx, p[j]);
    }
    double sum = 0.0;
    for (int j = 0; j < valid; ++j) {
        const float e = expf(p[j] - mx);
        sum += (double)e;
        p[j] = e;
    }
    const float inv = (float)(1.0 / sum);
    for (int j = 0; j < valid; ++j) p[j] = p[j] * inv;
    for (int e2 = 0; e2 < hd; ++e2) oh[e2] = ref_dot_f32(valid, vbase + e2, stride, p, 1);
    free(p);
}

/* Test exports of the two orders' building blocks: one attention row over
 * K, V [valid][hd] (ref_order 0: this oracle's chunked order, 1: the
 * reference's), and one q8_0 x q8_0 block dot. */
void orc_attention_row(int ref_order, const float* q, const float* k, const float* v, int valid, int hd, float* out) {
    const float scale = 1.0f / sqrtf((float)hd);
    if (ref_order)
        attn_row_ref(q, k, v, (size_t)hd, valid, hd, scale, out);
    else
        attn_row_chunked(q, k, v, (size_t)hd, valid, hd, scale, out, NULL, 0);
}

float orc_dot_q8_blocks(int ref_order, const void* w, const void* x, int nb) {
    return ref_order ? ref_dot_q8((const blk_q8*)w, (const blk_q8*)x, nb) : dot_q8((const blk_q8*)w, (const blk_q8*)x, nb);
}

int orc_decoder_run_ref(orc_decoder* d, const float* embeds, int T, float* out_hidden) {
    if (!d || !embeds || T <= 0 || d->past + T > d->max_seq || d->m->wtype != ORC_Q8_0) return -1;
    const orc_model* m = d->m;
    const int H = m->hidden, hd = m->head_dim, nh = m->n_heads, nkv = m->n_kv, F = m->ffn;
    const int past = d->past, kv = past + T, group = nh / nkv;
    const int qd = nh * hd, kd = nkv * hd;
    float* x = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* xn = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* q = (float*)malloc(sizeof(float) * (size_t)T * qd);
    float* k = (float*)malloc(sizeof(float) * (size_t)T * kd);
    float* v = (float*)malloc(sizeof(float) * (size_t)T * kd);
    float* o = (float*)malloc(sizeof(float) * (size_t)T * qd);
    float* proj = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* g = (float*)malloc(sizeof(float) * (size_t)T * F);
    float* u = (float*)malloc(sizeof(float) * (size_t)T * F);
    memcpy(x, embeds, sizeof(float) * (size_t)T * H);
    const float scale = 1.0f / sqrtf((float)hd);
    for (int l = 0; l < m->n_layers; ++l) {
        const orc_layer* L = &m->layers[l];
        for (int t = 0; t < T; ++t) ref_rms_norm_mul(x + (size_t)t * H, L->attn_norm, H, m->eps, xn + (size_t)t * H);
        ref_mul_mat_q8(L->wq, qd, H, xn, T, q);
        ref_mul_mat_q8(L->wk, kd, H, xn, T, k);
        ref_mul_mat_q8(L->wv, kd, H, xn, T, v);
        for (int t = 0; t < T; ++t) {
            for (int h = 0; h < nh; ++h) {
                float* qh = q + (size_t)t * qd + (size_t)h * hd;
                ref_rms_norm_mul(qh, L->q_norm, hd, m->eps, qh);
                ref_rope_neox(qh, hd, past + t, m->theta);
            }
            for (int h = 0; h < nkv; ++h) {
                float* kh = k + (size_t)t * kd + (size_t)h * hd;
                ref_rms_norm_mul(kh, L->k_norm, hd, m->eps, kh);
                ref_rope_neox(kh, hd, past + t, m->theta);
            }
            float* kdst = d->k + kv_index(d, l, past + t);
            float* vdst = d->v + kv_index(d, l, past + t);
            for (int i = 0; i < kd; ++i) {
                kdst[i] = d->kv_fp16 ? round_f16(k[(size_t)t * kd + i]) : k[(size_t)t * kd + i];
                vdst[i] = d->kv_fp16 ? round_f16(v[(size_t)t * kd + i]) : v[(size_t)t * kd + i];
            }
        }
#pragma omp parallel for collapse(2) schedule(static)
        for (int t = 0; t < T; ++t) {
            for (int h = 0; h < nh; ++h) {
                const int kvh = h / group;
                attn_row_ref(q + (size_t)t * qd + (size_t)h * hd, d->k + kv_index(d, l, 0) + (size_t)kvh * hd,
                             d->v + kv_index(d, l, 0) + (size_t)kvh * hd, (size_t)nkv * hd, past + t + 1, hd, scale,
                             o + (size_t)t * qd + (size_t)h * hd);
            }
        }
        ref_mul_mat_q8(L->wo, H, qd, o, T, proj);
        for (size_t i = 0; i < (size_t)T * H; ++i) x[i] = x[i] + proj[i];
        for (int t = 0; t < T; ++t) ref_rms_norm_mul(x + (size_t)t * H, L->ffn_norm, H, m->eps, xn + (size_t)t * H);
        ref_mul_mat_q8(L->wgate, F, H, xn, T, g);
        ref_mul_mat_q8(L->wup, F, H, xn, T, u);
        for (size_t i = 0; i < (size_t)T * F; ++i) g[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
        ref_mul_mat_q8(L->wdown, H, F, g, T, proj);
        for (size_t i = 0; i < (size_t)T * H; ++i) x[i] = x[i] + proj[i];
    }
    for (int t = 0; t < T; ++t) ref_rms_norm_mul(x + (size_t)t * H, m->output_norm, H, m->eps, out_hidden + (size_t)t * H);
    d->past = kv;
    free(x); free(xn); free(q); free(k); free(v); free(o); free(proj); free(g); free(u);
    return 0;
}

void orc_decoder_logits_ref(const orc_decoder* d, const float* hidden_row, float* logits) {
    ref_mul_mat_q8(d->m->token_embd, d->m->vocab, d->m->hidden, hidden_row, 1, logits);
}

/* ============================================================ audio front end
 * WhisperMel::compute (src/mel.cpp:153-224), WhisperEncoder::encode
 * (src/whisper_encoder.cpp:98-207), AudioAdaptor::apply
 * (src/audio_adaptor.cpp:39-96) and AudioEncoder::encode
 * (src/audio_encoder.cpp:16-75).
 *
 * The mel follows the reference's own order exactly (float window and twiddle
 * tables formed as at src/mel.cpp:31-45, double sums in ascending index,
 * log10 in double).  The ggml ops of the encoder and adaptor are restated in
 * the order the CUDA kernels evaluate them (the decoder's convention):
 *   - conv1d (kernel 3, padding 1) as im2col x F32 weights: one fmaf chain per
 *     output over j = ic * 3 + k ascending, then + bias, GELU (erf form:
 *     (0.5 x)(1 + erff(x / sqrt 2)), ggml_vec_gelu_erf_f32);
 *   - ggml_norm: mean and variance as double sums, 32 strided partials
 *     (i = l, l + 32, ...) combined by an xor butterfly; y = ((x - mean) *
 *     (1 / sqrtf(var + eps))) * w + b;
 *   - q8_0 linears: the decoder's q8_0 dot (dot_q8), then + bias;
 *   - attention (no mask, scale 1/sqrt(64)): 64-key tiles with a running
 *     maximum and sum (online softmax; per tile the 4-key partial sums of 16
 *     lanes combined by an xor butterfly), P.V as one fmaf chain per tile,
 *     exp = orc_expf, the output divided by the sum at the end.
 * `ref_order` = 1 evaluates the encoder and adaptor in the reference's order
 * instead, for the tests that bound the gap between the two orders: ggml's
 * x86 dot orders (ref_dot_f32 for the conv im2col rows, the scores and P.V;
 * ref_mul_mat_q8 for the q8_0 linears), ggml_norm's sequential double sums,
 * whole-row softmax (max, libm expf, sum in double, scaled by 1/sum:
 * src/whisper_encoder.cpp:157-166, ggml soft_max_ext), libm erff and expf in
 * GELU and SiLU. */

typedef struct {
    const float *attn_ln_w, *attn_ln_b, *ffn_ln_w, *ffn_ln_b;
    const void *q_w, *k_w, *v_w, *o_w, *fc1_w, *fc2_w; /* q8_0 rows */
    const float *q_b, *v_b, *o_b, *fc1_b, *fc2_b;
} orc_audio_layer;

struct orc_audio {
    int n_fft, hop, n_mels, n_bins, n_samples, n_frames, d, n_layers, n_heads, ffn, merge, hidden, enc_T;
    float ad_eps;
    int ref_order;
    float *window, *cos_t, *sin_t; /* [n_bins][n_fft] as in the reference */
    const float *fb, *conv1_w, *conv1_b, *conv2_w, *conv2_b, *pos, *ln_post_w, *ln_post_b;
    const void *ad_fc1_w, *ad_fc2_w;
    const float *ad_fc1_b, *ad_fc2_b, *ad_ln_w, *ad_ln_b;
    orc_audio_layer* layers;
};

orc_audio* orc_audio_create(const int* cfg, float adaptor_eps) {
    orc_audio* a = (orc_audio*)calloc(1, sizeof(orc_audio));
    a->n_fft = cfg[0], a->hop = cfg[1], a->n_mels = cfg[2], a->n_samples = cfg[3], a->n_frames = cfg[4];
    a->d = cfg[5], a->n_layers = cfg[6], a->n_heads = cfg[7], a->ffn = cfg[8], a->merge = cfg[9], a->hidden = cfg[10];
    a->ad_eps = adaptor_eps;
    a->n_bins = a->n_fft / 2 + 1;
    a->enc_T = (a->n_frames + 2 - 3) / 2 + 1;
    if (a->n_fft <= 0 || a->n_mels <= 0 || a->d <= 0 || a->n_heads <= 0 || a->d != a->n_heads * 64 || a->n_layers <= 0) {
        free(a);
        return NULL;
    }
    a->layers = (orc_audio_layer*)calloc((size_t)a->n_layers, sizeof(orc_audio_layer));
    a->window = (float*)malloc(sizeof(float) * (size_t)a->n_fft);
    a->cos_t = (float*)malloc(sizeof(float) * (size_t)a->n_fft * (size_t)a->n_bins);
    a->sin_t = (float*)malloc(sizeof(float) * (size_t)a->n_fft * (size_t)a->n_bins);
    for (int n = 0; n < a->n_fft; ++n) a->window[n] = 0.5f * (1.0f - cos(2.0 * M_PI * n / (double)a->n_fft));
    for (int k = 0; k < a->n_bins; ++k)
        for (int n = 0; n < a->n_fft; ++n) {
            const double ang = 2.0 * M_PI * (double)k * (double)n / (double)a->n_fft;
            a->cos_t[(size_t)k * a->n_fft + n] = (float)cos(ang);
            a->sin_t[(size_t)k * a->n_fft + n] = (float)sin(ang);
        }
    return a;
}

void orc_audio_free(orc_audio* a) {
    if (!a) return;
    free(a->layers);
    free(a->window);
    free(a->cos_t);
    free(a->sin_t);
    free(a);
}

void orc_audio_set_ref_order(orc_audio* a, int ref_order) { a->ref_order = ref_order; }

/* Keeps `data` (the caller owns it): F32 arrays, or q8_0 rows for the linears. */
int orc_audio_set_tensor(orc_audio* a, const char* name, const void* data) {
    const float* f = (const float*)data;
    if (!strcmp(name, "mel_filters")) a->fb = f;
    else if (!strcmp(name, "enc.conv1.w")) a->conv1_w = f;
    else if (!strcmp(name, "enc.conv1.b")) a->conv1_b = f;
    else if (!strcmp(name, "enc.conv2.w")) a->conv2_w = f;
    else if (!strcmp(name, "enc.conv2.b")) a->conv2_b = f;
    else if (!strcmp(name, "enc.pos_embd")) a->pos = f;
    else if (!strcmp(name, "enc.ln_post.w")) a->ln_post_w = f;
    else if (!strcmp(name, "enc.ln_post.b")) a->ln_post_b = f;
    else if (!strcmp(name, "adaptor.fc1.w")) a->ad_fc1_w = data;
    else if (!strcmp(name, "adaptor.fc2.w")) a->ad_fc2_w = data;
    else if (!strcmp(name, "adaptor.fc1.b")) a->ad_fc1_b = f;
    else if (!strcmp(name, "adaptor.fc2.b")) a->ad_fc2_b = f;
    else if (!strcmp(name, "adaptor.ln.w")) a->ad_ln_w = f;
    else if (!strcmp(name, "adaptor.ln.b")) a->ad_ln_b = f;
    else {
        int il = -1, off = 0;
        if (sscanf(name, "enc.blk.%d.%n", &il, &off) != 1 || il < 0 || il >= a->n_layers) return -1;
        orc_audio_layer* L = &a->layers[il];
        const char* s = name + off;
        if (!strcmp(s, "attn_ln.w")) L->attn_ln_w = f;
        else if (!strcmp(s, "attn_ln.b")) L->attn_ln_b = f;
        else if (!strcmp(s, "ffn_ln.w")) L->ffn_ln_w = f;
        else if (!strcmp(s, "ffn_ln.b")) L->ffn_ln_b = f;
        else if (!strcmp(s, "attn_q.w")) L->q_w = data;
        else if (!strcmp(s, "attn_k.w")) L->k_w = data;
        else if (!strcmp(s, "attn_v.w")) L->v_w = data;
        else if (!strcmp(s, "attn_out.w")) L->o_w = data;
        else if (!strcmp(s, "ffn_1.w")) L->fc1_w = data;
        else if (!strcmp(s, "ffn_2.w")) L->fc2_w = data;
        else if (!strcmp(s, "attn_q.b")) L->q_b = f;
        else if (!strcmp(s, "attn_v.b")) L->v_b = f;
        else if (!strcmp(s, "attn_out.b")) L->o_b = f;
        else if (!strcmp(s, "ffn_1.b")) L->fc1_b = f;
        else if (!strcmp(s, "ffn_2.b")) L->fc2_b = f;
        else return -1;
    }
    return 0;
}

/* src/mel.cpp:153-224 (the serial DFT path): reflect padding, window, power
 * spectrum, mel projection, log10, chunk normalisation.  chunk: n_samples
 * values (the caller zero-pads, as src/audio_encoder.cpp:53-55 does);
 * mel: [n_mels][n_frames]. */
void orc_audio_mel(const orc_audio* a, const float* chunk, float* mel) {
    const int N = a->n_samples, pad = a->n_fft / 2, nb = a->n_bins, nf = a->n_fft;
    float* x = (float*)malloc(sizeof(float) * (size_t)(N + 2 * pad));
    for (int i = 0; i < pad; ++i) x[i] = chunk[pad - i];
    for (int i = 0; i < N; ++i) x[pad + i] = chunk[i];
    for (int i = 0; i < pad; ++i) x[pad + N + i] = chunk[N - 2 - i];
#pragma omp parallel
    {
        float* frame = (float*)malloc(sizeof(float) * (size_t)nf);
        double* power = (double*)malloc(sizeof(double) * (size_t)nb);
#pragma omp for schedule(static)
        for (int t = 0; t < a->n_frames; ++t) {
            const int start = t * a->hop;
            for (int n = 0; n < nf; ++n) frame[n] = x[start + n] * a->window[n];
            for (int b = 0; b < nb; ++b) {
                const float* cr = a->cos_t + (size_t)b * nf;
                const float* sr = a->sin_t + (size_t)b * nf;
                double re = 0.0, im = 0.0;
                for (int n = 0; n < nf; ++n) {
                    re += (double)frame[n] * cr[n];
                    im -= (double)frame[n] * sr[n];
                }
                power[b] = re * re + im * im;
            }
            for (int m = 0; m < a->n_mels; ++m) {
                const float* row = a->fb + (size_t)m * nb;
                double acc = 0.0;
                for (int b = 0; b < nb; ++b) acc += (double)row[b] * power[b];
                mel[(size_t)m * a->n_frames + t] = (float)log10(acc > 1e-10 ? acc : 1e-10);
            }
        }
        free(frame);
        free(power);
    }
    free(x);
    const size_t count = (size_t)a->n_mels * (size_t)a->n_frames;
    float mx = mel[0];
    for (size_t i = 0; i < count; ++i) mx = mel[i] > mx ? mel[i] : mx;
    const float floor_v = mx - 8.0f;
    for (size_t i = 0; i < count; ++i) {
        const float v = mel[i] > floor_v ? mel[i] : floor_v;
        mel[i] = (v + 4.0f) / 4.0f;
    }
}

/* erf by its Maclaurin series in double (the CUDA kernels' exact_erff, the
 * same operations in the same order): t_n = (t_(n-1) * -x^2) * (1/n),
 * s += t_n * (1/(2n+1)) until the term is at most 2^-60 of the sum;
 * |x| >= 4 gives +-1.  Tested against libm's erf within 1 ulp. */
float orc_erff(float xf) {
    const double x = (double)xf;
    if (!(fabs(x) < 4.0)) return xf != xf ? xf : (xf > 0.0f ? 1.0f : -1.0f);
    const double mx2 = -x * x;
    double term = x, sum = x;
    for (int n = 1; n <= 128; ++n) {
        term = (term * mx2) * (1.0 / (double)n);
        const double add = term * (1.0 / (double)(2 * n + 1));
        sum = sum + add;
        if (fabs(add) <= fabs(sum) * 8.673617379884035e-19) break;
    }
    return (float)(sum * 1.1283791670955126);
}

/* GELU, erf form (ggml_vec_gelu_erf_f32): (0.5 x)(1 + erf(x / sqrt 2)). */
static inline float gelu_erf(float v) { return (0.5f * v) * (1.0f + orc_erff(v * 0.707106781f)); }

/* conv1d, kernel 3, padding 1: out[t][oc] = gelu(b + sum_j A[t][j] W[oc][j]) (+ pos[t][oc]). */
static void conv_gelu(const float* x, int L, int IC, long sp, long sc, int stride, const float* w, const float* b,
                      const float* pos, int OC, int OL, float* out, int ref) {
    const int J = IC * 3;
    /* W transposed to [J][OC]: the chains of all output channels advance
     * together in vector lanes, each still one fmaf chain over j ascending. */
    float* wt = (float*)malloc(sizeof(float) * (size_t)J * (size_t)OC);
#pragma omp parallel for schedule(static)
    for (int j = 0; j < J; ++j)
        for (int oc = 0; oc < OC; ++oc) wt[(size_t)j * OC + oc] = w[(size_t)oc * J + j];
#pragma omp parallel for schedule(static)
    for (int t = 0; t < OL; ++t) {
        float* col = (float*)malloc(sizeof(float) * (size_t)J);
        float* accs = (float*)malloc(sizeof(float) * (size_t)OC);
        for (int j = 0; j < J; ++j) {
            const int ic = j / 3, k = j % 3, p = t * stride + k - 1;
            col[j] = (p >= 0 && p < L) ? x[(long)p * sp + (long)ic * sc] : 0.f;
        }
        if (!ref) {
            for (int oc = 0; oc < OC; ++oc) accs[oc] = 0.f;
            for (int j = 0; j < J; ++j) {
                const float cj = col[j];
                const float* wr = wt + (size_t)j * OC;
                for (int oc = 0; oc < OC; ++oc) accs[oc] = fmaf(cj, wr[oc], accs[oc]);
            }
        }
        for (int oc = 0; oc < OC; ++oc) {
            const float* wr = w + (size_t)oc * J;
            float acc = accs[oc];
            if (ref) acc = ref_dot_f32(J, col, 1, wr, 1);
            float g = ref ? (0.5f * (acc + b[oc])) * (1.0f + erff((acc + b[oc]) * 0.707106781f)) : gelu_erf(acc + b[oc]);
            if (pos) g = g + pos[(size_t)t * OC + oc];
            out[(size_t)t * OC + oc] = g;
        }
        free(col);
        free(accs);
    }
    free(wt);
}

static double lane_sum_d(double* v) {
    /* 32 lane partials combined by an xor butterfly (every lane ends equal). */
    for (int o = 16; o > 0; o >>= 1) {
        double nv[32];
        for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ o];
        memcpy(v, nv, sizeof(nv));
    }
    return v[0];
}

static void layer_norm_rows(const float* x, int T, int D, const float* w, const float* b, float eps, float* y,
                            int ref) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < T; ++r) {
        const float* xr = x + (size_t)r * D;
        float* yr = y + (size_t)r * D;
        if (ref) {
            /* ggml_norm's sequential double sums. */
            double sum = 0.0;
            for (int i = 0; i < D; ++i) sum += (double)xr[i];
            const float mean = (float)(sum / D);
            double sum2 = 0.0;
            for (int i = 0; i < D; ++i) {
                const float v = xr[i] - mean;
                sum2 += (double)(v * v);
            }
            const float scale = 1.0f / sqrtf((float)(sum2 / D) + eps);
            for (int i = 0; i < D; ++i) yr[i] = ((xr[i] - mean) * scale) * w[i] + b[i];
            continue;
        }
        double p[32];
        for (int l = 0; l < 32; ++l) {
            p[l] = 0.0;
            for (int i = l; i < D; i += 32) p[l] = p[l] + (double)xr[i];
        }
        const float mean = (float)(lane_sum_d(p) / D);
        for (int l = 0; l < 32; ++l) {
            p[l] = 0.0;
            for (int i = l; i < D; i += 32) {
                const float v = xr[i] - mean;
                p[l] = p[l] + (double)(v * v);
            }
        }
        const float var = (float)(lane_sum_d(p) / D);
        const float scale = 1.0f / sqrtf(var + eps);
        for (int i = 0; i < D; ++i) yr[i] = ((xr[i] - mean) * scale) * w[i] + b[i];
    }
}

/* y[T][n] (= | += | gelu | silu) of W q8_0 [n x k] . x[T][k] + b. */
enum { LIN_BIAS = 0, LIN_GELU = 1, LIN_SILU = 2, LIN_RESID = 3 };
static void linear_q8(const void* w, const float* b, int n, int k, const float* x, int T, float* y, int mode,
                      int ref) {
    float* tmp = (float*)malloc(sizeof(float) * (size_t)T * (size_t)n);
    if (ref)
        ref_mul_mat_q8(w, n, k, x, T, tmp);
    else
        orc_mul_mat_q8(w, n, k, x, T, tmp);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < (size_t)T * (size_t)n; ++i) {
        const float v = tmp[i] + (b ? b[i % (size_t)n] : 0.0f);
        if (mode == LIN_GELU) y[i] = ref ? (0.5f * v) * (1.0f + erff(v * 0.707106781f)) : gelu_erf(v);
        else if (mode == LIN_SILU) y[i] = v / (1.0f + (ref ? expf(-v) : exp_own(-v)));
        else if (mode == LIN_RESID) y[i] = y[i] + v;
        else y[i] = v;
    }
    free(tmp);
}

/* One head of one query: q, k, v with row stride ld; out[64].  kt: the head's
 * keys transposed, [64][Tp] (Tp = T rounded up to 64, zero padded), for the
 * kernels' order: the 64 score chains of a tile advance together in vector
 * lanes, each one fmaf chain over the dims in order. */
static void enc_attn_row(const float* q, const float* k, const float* kt, int Tp, const float* v, long ld, int T,
                         int ref_order, float* out) {
    const float scale = 0.125f;
    if (ref_order) {
        float* p = (float*)malloc(sizeof(float) * (size_t)T);
        float mx = -INFINITY;
        for (int j = 0; j < T; ++j) {
            p[j] = ref_dot_f32(64, q, 1, k + (long)j * ld, 1) * scale;
            mx = p[j] > mx ? p[j] : mx;
        }
        double sum = 0.0;
        for (int j = 0; j < T; ++j) {
            p[j] = expf(p[j] - mx);
            sum += (double)p[j];
        }
        const float inv = (float)(1.0 / sum);
        for (int j = 0; j < T; ++j) p[j] *= inv;
        for (int i = 0; i < 64; ++i) out[i] = ref_dot_f32(T, v + i, (size_t)ld, p, 1);
        free(p);
        return;
    }
    float m = -1e30f, l = 0.f, o[64];
    for (int i = 0; i < 64; ++i) o[i] = 0.f;
    static const float zeros[64];
    for (int k0 = 0; k0 < T; k0 += 64) {
        float s[64], p[64], acc[64];
        float tmax = -1e30f;
        for (int c = 0; c < 64; ++c) acc[c] = 0.f;
        for (int i = 0; i < 64; ++i) {
            const float qi = q[i];
            const float* kr = kt + (size_t)i * Tp + k0;
            for (int c = 0; c < 64; ++c) acc[c] = fmaf(qi, kr[c], acc[c]);
        }
        for (int c = 0; c < 64; ++c) {
            s[c] = k0 + c < T ? acc[c] * scale : -1e30f;
            tmax = s[c] > tmax ? s[c] : tmax;
        }
        const float mn = m > tmax ? m : tmax;
        const float alpha = exp_own(m - mn);
        m = mn;
        /* 16 lanes x 4 keys: lane partials from 0 in key order, then the butterfly. */
        float part[16];
        for (int ln = 0; ln < 16; ++ln) {
            float ps = 0.f;
            for (int c = 0; c < 4; ++c) {
                const int kc = 4 * ln + c;
                p[kc] = k0 + kc < T ? exp_own(s[kc] - mn) : 0.f;
                ps = ps + p[kc];
            }
            part[ln] = ps;
        }
        for (int off = 8; off > 0; off >>= 1) {
            float np_[16];
            for (int ln = 0; ln < 16; ++ln) np_[ln] = part[ln] + part[ln ^ off];
            memcpy(part, np_, sizeof(np_));
        }
        l = l * alpha + part[0];
        for (int i = 0; i < 64; ++i) o[i] = o[i] * alpha;
        for (int c = 0; c < 64; ++c) {
            const float pc = p[c];
            const float* vr = k0 + c < T ? v + (long)(k0 + c) * ld : zeros;
            for (int i = 0; i < 64; ++i) o[i] = fmaf(pc, vr[i], o[i]);
        }
    }
    const float inv = 1.0f / l;
    for (int i = 0; i < 64; ++i) out[i] = o[i] * inv;
}

/* src/whisper_encoder.cpp:98-207: mel [n_mels][n_frames] -> out [enc_T][d]
 * (after the final LayerNorm). */
int orc_audio_encoder(const orc_audio* a, const float* mel, float* out) {
    const int d = a->d, T = a->enc_T, H = a->n_heads;
    float* c1 = (float*)malloc(sizeof(float) * (size_t)a->n_frames * d);
    float* h = (float*)malloc(sizeof(float) * (size_t)T * d);
    float* nrm = (float*)malloc(sizeof(float) * (size_t)T * d);
    float* q = (float*)malloc(sizeof(float) * (size_t)T * d);
    float* k = (float*)malloc(sizeof(float) * (size_t)T * d);
    float* v = (float*)malloc(sizeof(float) * (size_t)T * d);
    float* att = (float*)malloc(sizeof(float) * (size_t)T * d);
    float* f = (float*)malloc(sizeof(float) * (size_t)T * a->ffn);
    const int Tp = (T + 63) / 64 * 64;
    float* kt = (float*)malloc(sizeof(float) * (size_t)d * Tp);
    const int ref = a->ref_order;
    conv_gelu(mel, a->n_frames, a->n_mels, 1, a->n_frames, 1, a->conv1_w, a->conv1_b, NULL, d, a->n_frames, c1, ref);
    conv_gelu(c1, a->n_frames, d, d, 1, 2, a->conv2_w, a->conv2_b, a->pos, d, T, h, ref);
    for (int il = 0; il < a->n_layers; ++il) {
        const orc_audio_layer* L = &a->layers[il];
        layer_norm_rows(h, T, d, L->attn_ln_w, L->attn_ln_b, 1e-5f, nrm, ref);
        linear_q8(L->q_w, L->q_b, d, d, nrm, T, q, LIN_BIAS, ref);
        linear_q8(L->k_w, NULL, d, d, nrm, T, k, LIN_BIAS, ref);
        linear_q8(L->v_w, L->v_b, d, d, nrm, T, v, LIN_BIAS, ref);
#pragma omp parallel for schedule(static)
        for (int hh = 0; hh < H; ++hh)
            for (int i = 0; i < 64; ++i)
                for (int j = 0; j < Tp; ++j)
                    kt[((size_t)hh * 64 + i) * Tp + j] = j < T ? k[(size_t)j * d + hh * 64 + i] : 0.f;
#pragma omp parallel for schedule(dynamic, 16)
        for (int idx = 0; idx < H * T; ++idx) {
            const int hh = idx / T, t = idx % T;
            enc_attn_row(q + (size_t)t * d + hh * 64, k + hh * 64, kt + (size_t)hh * 64 * Tp, Tp, v + hh * 64, d, T,
                         a->ref_order, att + (size_t)t * d + hh * 64);
        }
        linear_q8(L->o_w, L->o_b, d, d, att, T, h, LIN_RESID, ref);
        layer_norm_rows(h, T, d, L->ffn_ln_w, L->ffn_ln_b, 1e-5f, nrm, ref);
        linear_q8(L->fc1_w, L->fc1_b, a->ffn, d, nrm, T, f, LIN_GELU, ref);
        linear_q8(L->fc2_w, L->fc2_b, d, a->ffn, f, T, h, LIN_RESID, ref);
    }
    layer_norm_rows(h, T, d, a->ln_post_w, a->ln_post_b, 1e-5f, out, ref);
    free(c1), free(h), free(nrm), free(q), free(k), free(v), free(att), free(f), free(kt);
    return 0;
}

/* src/audio_adaptor.cpp:39-96: enc [frames][d] (frames a multiple of merge)
 * -> out [frames / merge][hidden]. */
int orc_audio_adaptor(const orc_audio* a, const float* enc, int frames, float* out) {
    const int N = frames / a->merge, kin = a->d * a->merge;
    float* a1 = (float*)malloc(sizeof(float) * (size_t)N * a->hidden);
    float* a2 = (float*)malloc(sizeof(float) * (size_t)N * a->hidden);
    const int ref = a->ref_order;
    linear_q8(a->ad_fc1_w, a->ad_fc1_b, a->hidden, kin, enc, N, a1, LIN_SILU, ref);
    linear_q8(a->ad_fc2_w, a->ad_fc2_b, a->hidden, a->hidden, a1, N, a2, LIN_BIAS, ref);
    layer_norm_rows(a2, N, a->hidden, a->ad_ln_w, a->ad_ln_b, a->ad_eps, out, ref);
    free(a1), free(a2);
    return N;
}

/* src/audio_encoder.cpp:16-75: samples -> out [n_tokens][hidden]; returns
 * n_tokens, or -1 (empty input, output too small). */
int orc_audio_encode(const orc_audio* a, const float* samples, int n, float* out, int max_tokens) {
    if (n <= 0) return -1;
    const int stride = a->hop * 2 * a->merge;
    int total = 0;
    for (int off = 0; off < n; off += a->n_samples) {
        const int unpadded = n - off < a->n_samples ? n - off : a->n_samples;
        total += (unpadded - 1) / stride + 1;
    }
    if (total > max_tokens) return -1;
    float* enc_all = (float*)malloc(sizeof(float) * (size_t)total * a->merge * a->d);
    float* chunk = (float*)malloc(sizeof(float) * (size_t)a->n_samples);
    float* mel = (float*)malloc(sizeof(float) * (size_t)a->n_mels * a->n_frames);
    float* enc = (float*)malloc(sizeof(float) * (size_t)a->enc_T * a->d);
    size_t row = 0;
    for (int off = 0; off < n; off += a->n_samples) {
        const int unpadded = n - off < a->n_samples ? n - off : a->n_samples;
        const int trim = ((unpadded - 1) / stride + 1) * a->merge;
        memset(chunk, 0, sizeof(float) * (size_t)a->n_samples);
        memcpy(chunk, samples + off, sizeof(float) * (size_t)unpadded);
        orc_audio_mel(a, chunk, mel);
        orc_audio_encoder(a, mel, enc);
        memcpy(enc_all + row * a->d, enc, sizeof(float) * (size_t)trim * a->d);
        row += (size_t)trim;
    }
    const int N = orc_audio_adaptor(a, enc_all, (int)row, out);
    free(enc_all), free(chunk), free(mel), free(enc);
    return N;
}
