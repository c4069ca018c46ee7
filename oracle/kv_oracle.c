/*
 * kv_oracle.c -- CPU oracle for the KV-cache append + attention path.
 * TEST INFRASTRUCTURE ONLY (see kv_oracle.h for scope, sources and the
 * assumptions A1-A6 under which it restates ggml's op semantics).
 *
 * Build: oracle/build.py (gcc -O3 -ffp-contract=off -pthread).  Contraction
 * must stay off: RoPE and RMSNorm are compared bit-for-bit and their reference
 * form has separately rounded products and sums.
 */
#define _GNU_SOURCE
#include "kv_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#if defined(__x86_64__)
#include <immintrin.h>
#define KVO_X86 1
#endif

/* ======================================================================== */
/* F16 conversion (A3: IEEE round-to-nearest-even, as ggml_cpy F32->F16)      */
/* ======================================================================== */

uint16_t kvo_f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {                       /* inf / nan */
        if (ax == 0x7f800000u) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x1ffu));
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 -> inf */
    if (ax >= 0x38800000u) {                       /* normal half */
        const uint32_t e = (ax >> 23) - 127u + 15u;
        const uint32_t m = ax & 0x7fffffu;
        uint32_t h = (e << 10) | (m >> 13);
        const uint32_t rem = m & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    if (ax <= 0x33000000u) return (uint16_t)sign;  /* <= 2^-25 rounds to 0 */
    {                                              /* subnormal half */
        const uint32_t e = ax >> 23;               /* biased, 102..112 */
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e;           /* 14..24 */
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
}

float kvo_f16_to_f32(uint16_t h)
{
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
    const uint32_t m = (uint32_t)h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        float v = (float)m * (1.0f / 16777216.0f); /* m * 2^-24, exact */
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

void kvo_f32_to_f16_n(const float *src, uint16_t *dst, int64_t n)
{
    for (int64_t i = 0; i < n; i++) dst[i] = kvo_f32_to_f16(src[i]);
}

void kvo_f16_to_f32_n(const uint16_t *src, float *dst, int64_t n)
{
    for (int64_t i = 0; i < n; i++) dst[i] = kvo_f16_to_f32(src[i]);
}

/* ======================================================================== */
/* Thread pool-less parallel for                                            */
/* ======================================================================== */

typedef void (*kvo_task_fn)(void *ctx, int64_t task);

typedef struct {
    kvo_task_fn fn;
    void *ctx;
    int64_t n_tasks;
    _Atomic int64_t next;
} kvo_par;

static void *kvo_par_worker(void *arg)
{
    kvo_par *p = (kvo_par *)arg;
    for (;;) {
        int64_t t = atomic_fetch_add(&p->next, 1);
        if (t >= p->n_tasks) break;
        p->fn(p->ctx, t);
    }
    return NULL;
}

int32_t kvo_online_cores(void)
{
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int32_t)n : 1;
}

static void kvo_parallel(int64_t n_tasks, int32_t n_threads, kvo_task_fn fn, void *ctx)
{
    if (n_tasks <= 0) return;
    if (n_threads <= 0) n_threads = kvo_online_cores();
    if (n_threads > n_tasks) n_threads = (int32_t)n_tasks;
    kvo_par p;
    p.fn = fn;
    p.ctx = ctx;
    p.n_tasks = n_tasks;
    atomic_store(&p.next, 0);
    if (n_threads <= 1) {
        kvo_par_worker(&p);
        return;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)(n_threads - 1));
    int32_t started = 0;
    for (int32_t i = 0; i < n_threads - 1; i++) {
        if (pthread_create(&th[i], NULL, kvo_par_worker, &p) != 0) break;
        started++;
    }
    kvo_par_worker(&p);
    for (int32_t i = 0; i < started; i++) pthread_join(th[i], NULL);
    free(th);
}

/* ======================================================================== */
/* RoPE (A2) -- ggml_rope_ext semantics as used at model.cpp:1396-1403        */
/* ======================================================================== */

/* Dimension at which the rotation of pair index i completes `n_turns` turns
 * over n_ctx_orig positions: the YaRN correction-range formula. */
static float kvo_yarn_dim(int32_t n_dims, int32_t n_ctx_orig, float n_turns, float base)
{
    const float two_pi = 2.0f * (float)M_PI;
    return (float)n_dims * logf((float)n_ctx_orig / (n_turns * two_pi)) / (2.0f * logf(base));
}

void kvo_rope_corr_dims(const kvo_cfg *c, float dims[2])
{
    const float lo = floorf(kvo_yarn_dim(c->n_rot, c->n_ctx_orig, c->rope_beta_fast, c->rope_base));
    const float hi = ceilf(kvo_yarn_dim(c->n_rot, c->n_ctx_orig, c->rope_beta_slow, c->rope_base));
    dims[0] = lo > 0.0f ? lo : 0.0f;
    dims[1] = hi < (float)(c->n_rot - 1) ? hi : (float)(c->n_rot - 1);
}

/* Linear ramp of the YaRN blend over pair index i0/2 between the corr dims. */
static float kvo_yarn_ramp(float lo, float hi, int32_t i0)
{
    const float den = (hi - lo) > 0.001f ? (hi - lo) : 0.001f;
    float y = ((float)(i0 / 2) - lo) / den;
    if (y < 0.0f) y = 0.0f;
    if (y > 1.0f) y = 1.0f;
    return 1.0f - y;
}

void kvo_rope_table(const kvo_cfg *c, int64_t pos0, int64_t npos, float *cs)
{
    const int32_t half = c->n_rot / 2;
    const float step = powf(c->rope_base, -2.0f / (float)c->n_rot);
    float dims[2] = {0.0f, 0.0f};
    if (c->rope_ext_factor != 0.0f) kvo_rope_corr_dims(c, dims);
    for (int64_t p = 0; p < npos; p++) {
        float theta = (float)(pos0 + p);
        float *row = cs + (size_t)p * (size_t)half * 2u;
        for (int32_t i = 0; i < half; i++) {
            const float ff = c->rope_freq_factors ? c->rope_freq_factors[i] : 1.0f;
            const float t_extrap = theta / ff;
            const float t_interp = c->rope_freq_scale * t_extrap;
            float t = t_interp;
            float mscale = c->rope_attn_factor;
            if (c->rope_ext_factor != 0.0f) {
                const float mix = kvo_yarn_ramp(dims[0], dims[1], 2 * i) * c->rope_ext_factor;
                t = t_interp * (1.0f - mix) + t_extrap * mix;
                mscale *= 1.0f + 0.1f * logf(1.0f / c->rope_freq_scale);
            }
            row[2 * i + 0] = cosf(t) * mscale;
            row[2 * i + 1] = sinf(t) * mscale;
            theta *= step;
        }
    }
}

void kvo_rope_row(const kvo_cfg *c, const float *cs_row, const float *x, float *y)
{
    const int32_t d = c->head_dim;
    const int32_t half = c->n_rot / 2;
    for (int32_t i = c->n_rot; i < d; i++) y[i] = x[i];
    for (int32_t i = 0; i < half; i++) {
        const float cth = cs_row[2 * i + 0];
        const float sth = cs_row[2 * i + 1];
        int32_t a, b;
        if (c->rope_mode == 2) { a = i; b = i + half; }      /* NEOX   */
        else                   { a = 2 * i; b = 2 * i + 1; } /* NORMAL */
        const float x0 = x[a];
        const float x1 = x[b];
        y[a] = x0 * cth - x1 * sth;
        y[b] = x0 * sth + x1 * cth;
    }
}

/* ======================================================================== */
/* RMSNorm (A1) -- model.cpp:1071-1074 applied per head at 1385-1386          */
/* ======================================================================== */

void kvo_rms_norm_mul(const float *x, const float *w, int32_t n, float eps, float *y)
{
    double sum = 0.0;
    for (int32_t i = 0; i < n; i++) {
        const float sq = x[i] * x[i];
        sum += (double)sq;
    }
    const float mean = (float)(sum / (double)n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int32_t i = 0; i < n; i++) {
        const float t = x[i] * scale;
        y[i] = t * w[i];
    }
}

/* dory's L2 norm (dory.c:577-580): ggml_scale(ggml_rms_norm(x, 1e-6f/n),
 * 1.0f/sqrtf(n)) -- A1's rms_norm with eps/n, then a float multiply -- and, for
 * Q, ggml_mul by the squared learned scale w (NULL for K; dory.c:646-649). */
void kvo_ngpt_norm(const float *x, const float *w, int32_t n, float eps, float *y)
{
    double sum = 0.0;
    for (int32_t i = 0; i < n; i++) {
        const float sq = x[i] * x[i];
        sum += (double)sq;
    }
    const float mean = (float)(sum / (double)n);
    const float scale = 1.0f / sqrtf(mean + eps / (float)n);
    const float post = 1.0f / sqrtf((float)n);
    for (int32_t i = 0; i < n; i++) {
        const float t = (x[i] * scale) * post;
        y[i] = w ? t * w[i] : t;
    }
}

/* ======================================================================== */
/* append: model.cpp:1382-1414                                               */
/* ======================================================================== */

static int kvo_cfg_ok(const kvo_cfg *c)
{
    if (!c) return 0;
    if (c->n_head <= 0 || c->n_head_kv <= 0 || c->head_dim <= 0) return 0;
    if (c->n_head % c->n_head_kv != 0) return 0;
    if (c->n_rot < 0 || c->n_rot > c->head_dim || (c->n_rot & 1)) return 0;
    if (c->rope_mode != 0 && c->rope_mode != 2) return 0;
    if (c->qk_norm < 0 || c->qk_norm > 2) return 0;
    return 1;
}

int kvo_append(const kvo_cfg *c, int64_t n_ctx, int64_t n_past, int32_t n_new,
               const float *q, int64_t q_stride,
               const float *k, int64_t k_stride,
               const float *v, int64_t v_stride,
               const float *q_norm_w, const float *k_norm_w,
               uint16_t *kcache, uint16_t *vcache, float *q_out)
{
    if (n_past + n_new > n_ctx) return -1;
    return kvo_append_ring(c, 0, n_past, n_new, q, q_stride, k, k_stride, v, v_stride, q_norm_w, k_norm_w,
                           kcache, vcache, q_out);
}

/* dory_kv_write (dory.c:477-522): the token at position pos goes to cell
 * pos mod n_cells (dory_kv_runs splits a batch into at most two contiguous
 * runs; the rows written are the same); n_cells = 0 is the linear cache. */
int kvo_append_ring(const kvo_cfg *c, int64_t n_cells, int64_t n_past, int32_t n_new,
                    const float *q, int64_t q_stride,
                    const float *k, int64_t k_stride,
                    const float *v, int64_t v_stride,
                    const float *q_norm_w, const float *k_norm_w,
                    uint16_t *kcache, uint16_t *vcache, float *q_out)
{
    if (!kvo_cfg_ok(c) || n_past < 0 || n_new < 0 || n_cells < 0 || (n_cells > 0 && n_new > n_cells)) return -1;
    if (c->qk_norm == 1 && (!q_norm_w || !k_norm_w)) return -1;
    if (c->qk_norm == 2 && !q_norm_w) return -1;
    const int32_t d = c->head_dim;
    const int32_t hq = c->n_head, hkv = c->n_head_kv;
    const int32_t half = c->n_rot / 2;
    float *cs = (float *)malloc(sizeof(float) * (size_t)(half > 0 ? half : 1) * 2u);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)d);
    float *rot = (float *)malloc(sizeof(float) * (size_t)d);
    for (int32_t t = 0; t < n_new; t++) {
        const int64_t pos = n_past + t;
        if (half > 0) kvo_rope_table(c, pos, 1, cs);
        /* Q: norm -> rope -> q_out (F32; kvo_attend rounds it to F16, A4) */
        for (int32_t h = 0; h < hq; h++) {
            const float *x = q + (size_t)t * (size_t)q_stride + (size_t)h * (size_t)d;
            const float *src = x;
            if (c->qk_norm == 1) { kvo_rms_norm_mul(x, q_norm_w, d, c->rms_eps, tmp); src = tmp; }
            float *dst = q_out + ((size_t)t * (size_t)hq + (size_t)h) * (size_t)d;
            if (half > 0) kvo_rope_row(c, cs, src, dst);
            else memcpy(dst, src, sizeof(float) * (size_t)d);
            if (c->qk_norm == 2) {   /* nGPT: after RoPE, Q's own per-head scale */
                memcpy(tmp, dst, sizeof(float) * (size_t)d);
                kvo_ngpt_norm(tmp, q_norm_w + (size_t)h * (size_t)d, d, c->rms_eps, dst);
            }
        }
        /* K: norm -> rope -> F16 cache row; V: F16 cache row */
        for (int32_t h = 0; h < hkv; h++) {
            const float *x = k + (size_t)t * (size_t)k_stride + (size_t)h * (size_t)d;
            const float *src = x;
            if (c->qk_norm == 1) { kvo_rms_norm_mul(x, k_norm_w, d, c->rms_eps, tmp); src = tmp; }
            if (half > 0) kvo_rope_row(c, cs, src, rot);
            else memcpy(rot, src, sizeof(float) * (size_t)d);
            if (c->qk_norm == 2) {
                memcpy(tmp, rot, sizeof(float) * (size_t)d);
                kvo_ngpt_norm(tmp, NULL, d, c->rms_eps, rot);
            }
            const int64_t row = n_cells > 0 ? pos % n_cells : pos;
            uint16_t *kd = kcache + ((size_t)row * (size_t)hkv + (size_t)h) * (size_t)d;
            kvo_f32_to_f16_n(rot, kd, d);
            const float *vx = v + (size_t)t * (size_t)v_stride + (size_t)h * (size_t)d;
            uint16_t *vd = vcache + ((size_t)row * (size_t)hkv + (size_t)h) * (size_t)d;
            kvo_f32_to_f16_n(vx, vd, d);
        }
    }
    free(cs);
    free(tmp);
    free(rot);
    return 0;
}

/* ======================================================================== */
/* attention: model.cpp:1416-1445 (default branch)                           */
/* ======================================================================== */

/* F32-accumulated dot product of two F16 vectors (A4).  Sixteen lanes in two
 * groups of eight, fused multiply-add, fixed tree reduction; the scalar and
 * the AVX2 versions produce identical bits. */
static float kvo_dot16_generic(const uint16_t *a, const uint16_t *b, int32_t n)
{
    float acc0[8] = {0}, acc1[8] = {0};
    int32_t i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 8; l++) {
            acc0[l] = fmaf(kvo_f16_to_f32(a[i + l]), kvo_f16_to_f32(b[i + l]), acc0[l]);
            acc1[l] = fmaf(kvo_f16_to_f32(a[i + 8 + l]), kvo_f16_to_f32(b[i + 8 + l]), acc1[l]);
        }
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++)
            acc0[l] = fmaf(kvo_f16_to_f32(a[i + l]), kvo_f16_to_f32(b[i + l]), acc0[l]);
    float s[8], t[4], u[2];
    for (int l = 0; l < 8; l++) s[l] = acc0[l] + acc1[l];
    for (int l = 0; l < 4; l++) t[l] = s[l] + s[l + 4];
    u[0] = t[0] + t[2];
    u[1] = t[1] + t[3];
    float r = u[0] + u[1];
    for (; i < n; i++) r = fmaf(kvo_f16_to_f32(a[i]), kvo_f16_to_f32(b[i]), r);
    return r;
}

#ifdef KVO_X86
__attribute__((target("avx2,fma,f16c")))
static float kvo_dot16_avx2(const uint16_t *a, const uint16_t *b, int32_t n)
{
    __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
    int32_t i = 0;
    for (; i + 16 <= n; i += 16) {
        __m256 a0 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(a + i)));
        __m256 b0 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(b + i)));
        __m256 a1 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(a + i + 8)));
        __m256 b1 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(b + i + 8)));
        acc0 = _mm256_fmadd_ps(a0, b0, acc0);
        acc1 = _mm256_fmadd_ps(a1, b1, acc1);
    }
    for (; i + 8 <= n; i += 8) {
        __m256 a0 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(a + i)));
        __m256 b0 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(b + i)));
        acc0 = _mm256_fmadd_ps(a0, b0, acc0);
    }
    __m256 s = _mm256_add_ps(acc0, acc1);
    __m128 t = _mm_add_ps(_mm256_castps256_ps128(s), _mm256_extractf128_ps(s, 1));
    __m128 u = _mm_add_ps(t, _mm_movehl_ps(t, t));
    __m128 r = _mm_add_ss(u, _mm_shuffle_ps(u, u, 1));
    float out = _mm_cvtss_f32(r);
    for (; i < n; i++) out = fmaf(kvo_f16_to_f32(a[i]), kvo_f16_to_f32(b[i]), out);
    return out;
}

/* acc[0..n) += p * f16(v[0..n)), fused. */
__attribute__((target("avx2,fma,f16c")))
static void kvo_axpy16_avx2(float *acc, float p, const uint16_t *v, int32_t n)
{
    const __m256 pb = _mm256_set1_ps(p);
    int32_t i = 0;
    for (; i + 8 <= n; i += 8) {
        __m256 vv = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(v + i)));
        _mm256_storeu_ps(acc + i, _mm256_fmadd_ps(pb, vv, _mm256_loadu_ps(acc + i)));
    }
    for (; i < n; i++) acc[i] = fmaf(p, kvo_f16_to_f32(v[i]), acc[i]);
}
#endif

static void kvo_axpy16_generic(float *acc, float p, const uint16_t *v, int32_t n)
{
    for (int32_t i = 0; i < n; i++) acc[i] = fmaf(p, kvo_f16_to_f32(v[i]), acc[i]);
}

static int kvo_have_avx2(void)
{
#ifdef KVO_X86
    static int cached = -1;
    if (cached < 0) {
        __builtin_cpu_init();
        cached = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") ? 1 : 0;
    }
    return cached;
#else
    return 0;
#endif
}

static float kvo_dot16(const uint16_t *a, const uint16_t *b, int32_t n)
{
#ifdef KVO_X86
    if (kvo_have_avx2()) return kvo_dot16_avx2(a, b, n);
#endif
    return kvo_dot16_generic(a, b, n);
}

static void kvo_axpy16(float *acc, float p, const uint16_t *v, int32_t n)
{
#ifdef KVO_X86
    if (kvo_have_avx2()) { kvo_axpy16_avx2(acc, p, v, n); return; }
#endif
    kvo_axpy16_generic(acc, p, v, n);
}

#define KVO_KEY_BLOCK 256

typedef struct {
    const kvo_cfg *c;
    int64_t n_past, n_kv, n_blocks;
    int32_t n_new, r;
    float scale;
    const uint16_t *q16;     /* [n_new][hq][d] */
    const uint16_t *kc, *vc; /* [n_ctx][hkv][d] */
    float *w;                /* [n_new][hq][n_kv]  scores, then F16-rounded P */
    float *part;             /* [n_new][hq][n_blocks][d] */
    float *out;
    const void *mask;        /* NULL: causal; else [n_new] rows of mask_stride (A6) */
    int64_t mask_stride;
    int32_t mask_f16, flash;
} kvo_att;

static float kvo_mask_at(const kvo_att *a, int32_t t, int64_t kk)
{
    const int64_t i = (int64_t)t * a->mask_stride + kk;
    return a->mask_f16 ? kvo_f16_to_f32(((const uint16_t *)a->mask)[i]) : ((const float *)a->mask)[i];
}

/* phase 1: scores for one (token, kv head, key block), all r heads of the group */
static void kvo_att_scores(void *vctx, int64_t task)
{
    kvo_att *a = (kvo_att *)vctx;
    const kvo_cfg *c = a->c;
    const int32_t d = c->head_dim, hq = c->n_head, hkv = c->n_head_kv;
    const int64_t blk = task % a->n_blocks;
    const int64_t rest = task / a->n_blocks;
    const int32_t kvh = (int32_t)(rest % hkv);
    const int32_t t = (int32_t)(rest / hkv);
    /* keys <= lim are visible (causal), or every key with a mask */
    const int64_t lim = a->mask ? a->n_kv - 1 : a->n_past + t;
    const int64_t k0 = blk * KVO_KEY_BLOCK;
    int64_t k1 = k0 + KVO_KEY_BLOCK;
    if (k1 > a->n_kv) k1 = a->n_kv;
    for (int64_t kk = k0; kk < k1; kk++) {
        const uint16_t *krow = a->kc + ((size_t)kk * (size_t)hkv + (size_t)kvh) * (size_t)d;
        for (int32_t j = 0; j < a->r; j++) {
            const int32_t h = kvh * a->r + j;
            float *w = a->w + ((size_t)t * (size_t)hq + (size_t)h) * (size_t)a->n_kv;
            if (kk > lim) { w[kk] = -INFINITY; continue; }
            const uint16_t *qrow = a->q16 + ((size_t)t * (size_t)hq + (size_t)h) * (size_t)d;
            w[kk] = kvo_dot16(krow, qrow, d) * a->scale;
            if (a->mask) w[kk] += kvo_mask_at(a, t, kk);   /* A5: w = s*scale + mask, two roundings */
        }
    }
}

/* phase 2: softmax of one (token, head) row (A5), then P rounded to F16 (A4);
 * the flash branch (A6) keeps exact weights e/sum in float */
static void kvo_att_softmax(void *vctx, int64_t task)
{
    kvo_att *a = (kvo_att *)vctx;
    float *w = a->w + (size_t)task * (size_t)a->n_kv;
    float mx = -INFINITY;
    for (int64_t kk = 0; kk < a->n_kv; kk++) if (w[kk] > mx) mx = w[kk];
    if (a->flash) {
        if (mx == -INFINITY) {   /* no visible key: the flash branch's output is 0 */
            for (int64_t kk = 0; kk < a->n_kv; kk++) w[kk] = 0.0f;
            return;
        }
        double sum = 0.0;
        for (int64_t kk = 0; kk < a->n_kv; kk++) {
            const double e = exp((double)w[kk] - (double)mx);
            w[kk] = (float)e;
            sum += e;
        }
        for (int64_t kk = 0; kk < a->n_kv; kk++) w[kk] = (float)((double)w[kk] / sum);
        return;
    }
    double sum = 0.0;
    for (int64_t kk = 0; kk < a->n_kv; kk++) {
        const float e = expf(w[kk] - mx);
        w[kk] = e;
        sum += (double)e;
    }
    const float inv = (float)(1.0 / sum);
    for (int64_t kk = 0; kk < a->n_kv; kk++)
        w[kk] = kvo_f16_to_f32(kvo_f32_to_f16(w[kk] * inv));
}

/* phase 3: partial P.V for one (token, kv head, key block), all r heads */
static void kvo_att_pv(void *vctx, int64_t task)
{
    kvo_att *a = (kvo_att *)vctx;
    const kvo_cfg *c = a->c;
    const int32_t d = c->head_dim, hq = c->n_head, hkv = c->n_head_kv;
    const int64_t blk = task % a->n_blocks;
    const int64_t rest = task / a->n_blocks;
    const int32_t kvh = (int32_t)(rest % hkv);
    const int32_t t = (int32_t)(rest / hkv);
    const int64_t lim = a->mask ? a->n_kv - 1 : a->n_past + t;
    const int64_t k0 = blk * KVO_KEY_BLOCK;
    int64_t k1 = k0 + KVO_KEY_BLOCK;
    if (k1 > a->n_kv) k1 = a->n_kv;
    if (k1 > lim + 1) k1 = lim + 1;
    for (int32_t j = 0; j < a->r; j++) {
        const int32_t h = kvh * a->r + j;
        float *acc = a->part + (((size_t)t * (size_t)hq + (size_t)h) * (size_t)a->n_blocks + (size_t)blk) * (size_t)d;
        memset(acc, 0, sizeof(float) * (size_t)d);
        const float *p = a->w + ((size_t)t * (size_t)hq + (size_t)h) * (size_t)a->n_kv;
        for (int64_t kk = k0; kk < k1; kk++) {
            const uint16_t *vrow = a->vc + ((size_t)kk * (size_t)hkv + (size_t)kvh) * (size_t)d;
            kvo_axpy16(acc, p[kk], vrow, d);
        }
    }
}

/* phase 4: sum the key-block partials of one (token, head) in block order */
static void kvo_att_reduce(void *vctx, int64_t task)
{
    kvo_att *a = (kvo_att *)vctx;
    const int32_t d = a->c->head_dim, hq = a->c->n_head;
    const int32_t t = (int32_t)(task / hq), h = (int32_t)(task % hq);
    float *o = a->out + (size_t)t * (size_t)hq * (size_t)d + (size_t)h * (size_t)d;
    const float *base = a->part + ((size_t)t * (size_t)hq + (size_t)h) * (size_t)a->n_blocks * (size_t)d;
    for (int32_t i = 0; i < d; i++) o[i] = 0.0f;
    for (int64_t b = 0; b < a->n_blocks; b++)
        for (int32_t i = 0; i < d; i++) o[i] += base[(size_t)b * (size_t)d + (size_t)i];
}

int kvo_attend(const kvo_cfg *c, int64_t n_past, int32_t n_new,
               const float *q_roped, const uint16_t *kcache, const uint16_t *vcache,
               float *out, int32_t n_threads)
{
    return kvo_attend_ex(c, n_past, n_new, q_roped, kcache, vcache, NULL, 0, 0, 0, out, n_threads);
}

int kvo_attend_ex(const kvo_cfg *c, int64_t n_past, int32_t n_new,
                  const float *q_roped, const uint16_t *kcache, const uint16_t *vcache,
                  const void *mask, int32_t mask_f16, int64_t mask_stride, int32_t flash,
                  float *out, int32_t n_threads)
{
    if (!kvo_cfg_ok(c) || n_past < 0 || n_new <= 0) return -1;
    if (mask && mask_stride < n_past + n_new) return -1;
    const int32_t d = c->head_dim, hq = c->n_head, hkv = c->n_head_kv;
    kvo_att a;
    a.c = c;
    a.n_past = n_past;
    a.n_new = n_new;
    a.n_kv = n_past + n_new;
    a.r = hq / hkv;
    a.scale = 1.0f / sqrtf((float)d);
    a.n_blocks = (a.n_kv + KVO_KEY_BLOCK - 1) / KVO_KEY_BLOCK;
    a.kc = kcache;
    a.vc = vcache;
    a.out = out;
    a.mask = mask;
    a.mask_stride = mask_stride;
    a.mask_f16 = mask_f16;
    a.flash = flash;
    const size_t nq = (size_t)n_new * (size_t)hq * (size_t)d;
    uint16_t *q16 = (uint16_t *)malloc(sizeof(uint16_t) * nq);
    float *w = (float *)malloc(sizeof(float) * (size_t)n_new * (size_t)hq * (size_t)a.n_kv);
    float *part = (float *)malloc(sizeof(float) * (size_t)n_new * (size_t)hq * (size_t)a.n_blocks * (size_t)d);
    if (!q16 || !w || !part) { free(q16); free(w); free(part); return -2; }
    kvo_f32_to_f16_n(q_roped, q16, (int64_t)nq);  /* A4: src1 converted to F16 */
    a.q16 = q16;
    a.w = w;
    a.part = part;
    const int64_t grp_tasks = (int64_t)n_new * hkv * a.n_blocks;
    kvo_parallel(grp_tasks, n_threads, kvo_att_scores, &a);
    kvo_parallel((int64_t)n_new * hq, n_threads, kvo_att_softmax, &a);
    kvo_parallel(grp_tasks, n_threads, kvo_att_pv, &a);
    kvo_parallel((int64_t)n_new * hq, n_threads, kvo_att_reduce, &a);
    free(q16);
    free(w);
    free(part);
    return 0;
}

/* dory_fill_attn_mask (dory.c:553-575): with head = pos0 + n_tokens - 1, cell c
 * is visible to the query at p = pos0 + q iff the newest write into it,
 * head - ((head - c) mod n_cells), is a real position (>= 0) no later than p. */
void kvo_ring_mask(int64_t n_cells, int64_t pos0, int32_t n_tokens, float *dst)
{
    const int64_t head = pos0 + n_tokens - 1;
    for (int32_t q = 0; q < n_tokens; q++) {
        const int64_t p = pos0 + q;
        for (int64_t cc = 0; cc < n_cells; cc++) {
            int64_t m = (head - cc) % n_cells;
            if (m < 0) m += n_cells;
            const int64_t last_write = head - m;
            dst[(size_t)q * (size_t)n_cells + (size_t)cc] = (last_write >= 0 && last_write <= p) ? 0.0f : -INFINITY;
        }
    }
}

/* ======================================================================== */
/* context sizing: model.cpp:869-885 (kv_cache_bytes), 1002-1059 (auto_n_ctx) */
/* ======================================================================== */

uint64_t kvo_kv_cache_bytes(int32_t n_layer, int32_t n_head_kv, int32_t head_dim, int64_t n_ctx)
{
    const uint64_t per_token = (uint64_t)n_layer * (uint64_t)head_dim * (uint64_t)n_head_kv * 2u * 2u;
    return per_token * (uint64_t)n_ctx;
}

int64_t kvo_auto_n_ctx(int64_t avail, uint64_t per_tok, int64_t n_ctx_train, int64_t longrope_orig)
{
    if (avail <= 0) return 4096;
    const uint64_t reserve = (uint64_t)384 << 20;
    uint64_t budget = (uint64_t)avail;
    budget -= budget < reserve ? budget : reserve;
    budget = (uint64_t)((double)budget * 0.8);
    int64_t raw = per_tok > 0 ? (int64_t)(budget / per_tok) : 4096;
    int64_t n_ctx = (raw / 64) * 64;
    int64_t limit = n_ctx_train > 0 ? n_ctx_train : 262144;
    if (longrope_orig > 0 && longrope_orig < limit) limit = longrope_orig;
    if (n_ctx > limit) n_ctx = limit;
    if (n_ctx < 512) n_ctx = 512 < limit ? 512 : limit;
    return n_ctx;
}

/* ======================================================================== */
/* seeded synthetic inputs                                                   */
/* ======================================================================== */
/* splitmix64 output function over a per-(seed, stream) starting state; an
 * approximately standard normal value is the Irwin-Hall sum of twelve 16-bit
 * uniforms, computed exactly so that every platform gets the same bits. */

static inline uint64_t kvo_mix64(uint64_t x)
{
    x ^= x >> 30;
    x *= 0xBF58476D1CE4E5B9ull;
    x ^= x >> 27;
    x *= 0x94D049BB133111EBull;
    x ^= x >> 31;
    return x;
}

uint64_t kvo_bits(uint64_t seed, uint64_t stream, uint64_t ctr)
{
    const uint64_t key = kvo_mix64(seed ^ kvo_mix64(stream + 0x6B76B200ull));
    return kvo_mix64(key + ctr * 0x9E3779B97F4A7C15ull);
}

static inline uint32_t kvo_sum4x16(uint64_t w)
{
    return (uint32_t)(w & 0xffffu) + (uint32_t)((w >> 16) & 0xffffu) +
           (uint32_t)((w >> 32) & 0xffffu) + (uint32_t)(w >> 48);
}

float kvo_normal(uint64_t seed, uint64_t stream, uint64_t idx)
{
    const uint64_t key = kvo_mix64(seed ^ kvo_mix64(stream + 0x6B76B200ull));
    const uint64_t c = idx * 3u;
    const uint32_t s = kvo_sum4x16(kvo_mix64(key + c * 0x9E3779B97F4A7C15ull)) +
                       kvo_sum4x16(kvo_mix64(key + (c + 1u) * 0x9E3779B97F4A7C15ull)) +
                       kvo_sum4x16(kvo_mix64(key + (c + 2u) * 0x9E3779B97F4A7C15ull));
    return (float)(s + 6u) * (1.0f / 65536.0f) - 6.0f;
}

typedef struct {
    uint64_t seed, stream, idx0;
    int64_t n, chunk;
    float *f32;
    uint16_t *f16;
} kvo_gen;

static void kvo_gen_task(void *vctx, int64_t task)
{
    kvo_gen *g = (kvo_gen *)vctx;
    const int64_t i0 = task * g->chunk;
    int64_t i1 = i0 + g->chunk;
    if (i1 > g->n) i1 = g->n;
    for (int64_t i = i0; i < i1; i++) {
        const float v = kvo_normal(g->seed, g->stream, g->idx0 + (uint64_t)i);
        if (g->f32) g->f32[i] = v;
        else g->f16[i] = kvo_f32_to_f16(v);
    }
}

static void kvo_gen_run(uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n, float *f32, uint16_t *f16)
{
    kvo_gen g = {seed, stream, idx0, n, 1 << 16, f32, f16};
    const int64_t tasks = (n + g.chunk - 1) / g.chunk;
    kvo_parallel(tasks, tasks > 1 ? 0 : 1, kvo_gen_task, &g);
}

void kvo_gen_normal_f32(uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n, float *out)
{
    kvo_gen_run(seed, stream, idx0, n, out, NULL);
}

void kvo_gen_normal_f16(uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n, uint16_t *out)
{
    kvo_gen_run(seed, stream, idx0, n, NULL, out);
}

void kvo_gen_uniform_f32(uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n,
                         float lo, float hi, float *out)
{
    for (int64_t i = 0; i < n; i++) {
        const float u = (float)(kvo_bits(seed, stream, idx0 + (uint64_t)i) >> 41) * (1.0f / 8388608.0f);
        out[i] = lo + u * (hi - lo);
    }
}

typedef struct {
    uint64_t seed, stream;
    int64_t row0;
    int32_t hkv, d, h0, nh;
    uint16_t *out;
} kvo_rows;

static void kvo_rows_task(void *vctx, int64_t r)
{
    kvo_rows *g = (kvo_rows *)vctx;
    const uint64_t row = (uint64_t)(g->row0 + r);
    for (int32_t hh = 0; hh < g->nh; hh++) {
        const uint64_t base = row * (uint64_t)g->hkv * (uint64_t)g->d + (uint64_t)(g->h0 + hh) * (uint64_t)g->d;
        uint16_t *dst = g->out + ((size_t)r * (size_t)g->nh + (size_t)hh) * (size_t)g->d;
        for (int32_t i = 0; i < g->d; i++)
            dst[i] = kvo_f32_to_f16(kvo_normal(g->seed, g->stream, base + (uint64_t)i));
    }
}

void kvo_gen_cache_rows(uint64_t seed, uint64_t stream, int64_t row0, int64_t nrows,
                        int32_t n_head_kv, int32_t head_dim, int32_t h0, int32_t nh,
                        uint16_t *out)
{
    kvo_rows g = {seed, stream, row0, n_head_kv, head_dim, h0, nh, out};
    kvo_parallel(nrows, nrows > 64 ? 0 : 1, kvo_rows_task, &g);
}
