/*
 * kv_oracle.h -- CPU oracle for the KV-cache append + attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links or calls this
 * code; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * (and `bench.py --impl reference`) load it, and only as the checker or as the
 * timed CPU baseline.
 *
 * What it restates
 * ----------------
 * The reference (GGML-Loader, src/model.cpp) expresses the hot path as a ggml op
 * sequence inside build_graph():
 *   QK-Norm   ggml_rms_norm + ggml_mul            model.cpp:1382-1387, 1071-1074
 *   RoPE      ggml_rope_ext on Q and K            model.cpp:1389-1404 (params 1312-1316)
 *   append    ggml_cpy F32 -> F16 cache view      model.cpp:1406-1414
 *   scores    ggml_mul_mat(K, Q)                  model.cpp:1436
 *   softmax   ggml_soft_max_ext(KQ, mask, scale)  model.cpp:1437 (mask 1579-1586)
 *   PV        ggml_mul_mat(V_trans, KQ)           model.cpp:1439-1444
 * Cache layout: one F16 tensor [head_dim, n_head_kv, n_ctx] per layer for K and
 * for V (model.cpp:855-856), i.e. position-major rows of n_head_kv*head_dim.
 *
 * PARITY UNPINNED.  The arithmetic of those ops lives in the third-party ggml
 * submodule (https://github.com/NekoFemDev/ggml.git, pinned commit unknown),
 * which is not vendored in the reference checkout, and the reference ships no
 * tests, golden vectors or fixtures for this path.  The op semantics below are
 * restated from the mathematics and ggml's documented CPU behaviour; the
 * following fine points are ASSUMPTIONS:
 *   A1 rms_norm sums (float)(x*x) sequentially in double, mean = (float)(sum/n),
 *      scale = 1.0f/sqrtf(mean+eps), y = x*scale, then a separate *gamma.
 *   A2 rope_ext builds its angle table by iterated float multiplication
 *      theta_{i+1} = theta_i * powf(base, -2/n_dims) starting at theta_0 = pos,
 *      divides by freq_factors[i] when given, applies the YaRN ramp only when
 *      ext_factor != 0, and takes libm cosf/sinf times mscale.  The rotation is
 *      x0*c - x1*s, x0*s + x1*c in float with NO fused multiply-add (this file
 *      is compiled with -ffp-contract=off).
 *   A3 cpy F32->F16 rounds to nearest even (IEEE).
 *   A4 mul_mat with an F16 src0 converts the F32 src1 to F16 (RNE) and
 *      accumulates products in F32 (summation order is implementation-defined;
 *      parity on attention outputs is therefore checked within a tolerance).
 *   A5 soft_max_ext: w = s*scale + mask, m = max w, e = expf(w - m) in float,
 *      sum accumulated in double, p = e * (float)(1.0/sum); a row whose w are
 *      all -inf gives NaN (expf(-inf - -inf)).
 *   A6 flash_attn_ext (the opt-in branch, model.cpp:1426-1434) computes the
 *      same softmax(w) . V with an online softmax and never rounds the
 *      normalised weights to F16; its CPU kernel's own accumulation order and
 *      precision are not restated -- the oracle takes the exact weights
 *      exp(w - m) / sum in double, rounded once to float, with F32 accumulation
 *      of P . V, and a row whose w are all -inf gives 0 (its sum is 0).
 * What reference code pins (the reference's MoE engine, src/moe_stream, which
 * computes the same decode attention without ggml on an F32 cache; compiled
 * from its sources by oracle/build.py):
 *   - its scalar backend (compute_backend.c:42-86): the NEOX rotation bit for
 *     bit given the same table; RMSNorm and softmax within 2e-6 (it sums in
 *     float);
 *   - its attention_block (qwen_model.c:456-524, driven by ref_attention.c):
 *     the GQA mapping h / (n_head / n_head_kv), the scale 1/sqrtf(hd), the
 *     causal range 0..pos, softmax and P.V, per-head Q/K RMSNorm -- outputs
 *     within max-abs 2e-3 / rel-L2 1e-3 at the benchmark shapes (2k-32k keys);
 *     its stored K row equals the oracle's rotation with its table entries bit
 *     for bit, its V row the oracle's F16 row after RNE;
 *   - its RoPE table (qwen_model.c:346-353, angles in double): every entry
 *     within (pos + 2) * 2^-22 of the oracle's (NEOX, no freq factors).
 * Still unpinned at the bit level (the MoE engine does not perform them):
 * A1's double sum, A2's iterated float angles, A4's F16 rounding of Q and of
 * the normalised P, A5's double sum, all of A6, and the NORMAL pairing, freq
 * factors and YaRN of A2.
 */
#ifndef KV_ORACLE_H
#define KV_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-layer attention parameters (mirrors hparams, model.h:63-95). */
typedef struct {
    int32_t n_head;          /* query heads (whole model, not a shard)         */
    int32_t n_head_kv;       /* KV heads                                       */
    int32_t head_dim;        /* n_embd_head                                    */
    int32_t n_rot;           /* rotated dims per head (<= head_dim, even)      */
    int32_t rope_mode;       /* 0 = NORMAL (adjacent pairs), 2 = NEOX (halves) */
    int32_t n_ctx_orig;      /* YaRN original context (only if ext_factor!=0)  */
    float   rope_base;       /* freq_base                                      */
    float   rope_freq_scale; /* freq_scale (1.0 for every reference arch)      */
    float   rope_attn_factor;/* mscale                                         */
    float   rope_ext_factor; /* 0 disables the YaRN ramp                       */
    float   rope_beta_fast;
    float   rope_beta_slow;
    const float *rope_freq_factors; /* [n_rot/2] or NULL                      */
    int32_t qk_norm;         /* 1: per-head RMSNorm on Q and K before RoPE;
                                2: dory's nGPT L2 norm after RoPE (Q scaled) */
    float   rms_eps;
} kvo_cfg;

/* ---- scalar helpers --------------------------------------------------- */
uint16_t kvo_f32_to_f16(float f);   /* IEEE binary16, round-to-nearest-even (A3) */
float    kvo_f16_to_f32(uint16_t h);
void     kvo_f32_to_f16_n(const float *src, uint16_t *dst, int64_t n);
void     kvo_f16_to_f32_n(const uint16_t *src, float *dst, int64_t n);

/* YaRN correction dims for the ramp (ggml_rope_yarn_corr_dims semantics). */
void kvo_rope_corr_dims(const kvo_cfg *c, float dims[2]);

/* RoPE table for positions pos0 .. pos0+npos-1: cs[(p*(n_rot/2) + i)*2 + {0,1}]
 * = (cos, sin) of pair i at position pos0+p (A2). */
void kvo_rope_table(const kvo_cfg *c, int64_t pos0, int64_t npos, float *cs);

/* y = rms_norm(x) * w over n elements (A1). */
void kvo_rms_norm_mul(const float *x, const float *w, int32_t n, float eps, float *y);

/* Rotate one head row of head_dim floats with the table row of its position. */
void kvo_rope_row(const kvo_cfg *c, const float *cs_row, const float *x, float *y);

/* ---- the path ------------------------------------------------------------
 * kvo_append: QK-Norm -> RoPE -> F16 cast of K and V rows into the cache at
 * rows [n_past, n_past+n_new) (model.cpp:1382-1414).  q/k/v point at the first
 * element of token 0's Q/K/V block; consecutive tokens are *_stride floats
 * apart (a fused phi3 QKV row uses one stride for all three, model.cpp:1088-1094).
 * kcache/vcache: [n_ctx][n_head_kv][head_dim] F16 of one layer.
 * q_out: [n_new][n_head][head_dim] F32, the rotated (and normed) Q.
 * Returns 0, or -1 on a bad argument. */
int kvo_append(const kvo_cfg *c, int64_t n_ctx, int64_t n_past, int32_t n_new,
               const float *q, int64_t q_stride,
               const float *k, int64_t k_stride,
               const float *v, int64_t v_stride,
               const float *q_norm_w, const float *k_norm_w,
               uint16_t *kcache, uint16_t *vcache, float *q_out);

/* kvo_attend: the default (non flash-attn) attention of model.cpp:1416-1445
 * over cache rows [0, n_past+n_new) with the causal mask of model.cpp:1579-1586.
 * q_roped: [n_new][n_head][head_dim] F32 (kvo_append's q_out).
 * out: [n_new][n_head*head_dim] F32.  n_threads <= 0 means all online cores.
 * The result does not depend on n_threads. */
int kvo_attend(const kvo_cfg *c, int64_t n_past, int32_t n_new,
               const float *q_roped, const uint16_t *kcache, const uint16_t *vcache,
               float *out, int32_t n_threads);

/* Ring cache (dory.c:391-575): kvo_append_ring writes the token at position p
 * to cell p mod n_cells (0: the linear cache, as kvo_append), RoPE at p;
 * kvo_ring_mask fills dory_fill_attn_mask's [n_tokens][n_cells] F32 0/-inf
 * visibility for a batch at positions [pos0, pos0+n_tokens). */
int kvo_append_ring(const kvo_cfg *c, int64_t n_cells, int64_t n_past, int32_t n_new,
                    const float *q, int64_t q_stride,
                    const float *k, int64_t k_stride,
                    const float *v, int64_t v_stride,
                    const float *q_norm_w, const float *k_norm_w,
                    uint16_t *kcache, uint16_t *vcache, float *q_out);
void kvo_ring_mask(int64_t n_cells, int64_t pos0, int32_t n_tokens, float *dst);
/* dory's L2 norm (dory.c:577-580) of one head vector, times w (Q's squared
 * learned scale, dory.c:646-649) when w != NULL. */
void kvo_ngpt_norm(const float *x, const float *w, int32_t n, float eps, float *y);

/* kvo_attend_ex: kvo_attend with the caller's additive mask (NULL: causal) of
 * n_new rows, mask_stride elements apart, F16 (mask_f16) or F32, added to each
 * scaled score (A5), and flash != 0 for the ggml_flash_attn_ext branch
 * (model.cpp:1426-1434) under A6. */
int kvo_attend_ex(const kvo_cfg *c, int64_t n_past, int32_t n_new,
                  const float *q_roped, const uint16_t *kcache, const uint16_t *vcache,
                  const void *mask, int32_t mask_f16, int64_t mask_stride, int32_t flash,
                  float *out, int32_t n_threads);

/* ---- context sizing (model.cpp:869-885, 1002-1059) ----------------------- */
uint64_t kvo_kv_cache_bytes(int32_t n_layer, int32_t n_head_kv, int32_t head_dim, int64_t n_ctx);
/* avail: bytes available (<=0: unreadable -> 4096); per_tok: bytes per position;
 * n_ctx_train: 0 -> 262144 cap; longrope_orig > 0 clamps (phi3 + LongRoPE). */
int64_t kvo_auto_n_ctx(int64_t avail, uint64_t per_tok, int64_t n_ctx_train, int64_t longrope_orig);

/* ---- seeded synthetic inputs (bit-identical to the product's generator) -- */
uint64_t kvo_bits(uint64_t seed, uint64_t stream, uint64_t ctr);
float    kvo_normal(uint64_t seed, uint64_t stream, uint64_t idx);
void kvo_gen_normal_f32(uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n, float *out);
void kvo_gen_normal_f16(uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n, uint16_t *out);
void kvo_gen_uniform_f32(uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n,
                         float lo, float hi, float *out);
/* Cache rows [row0, row0+nrows) of one tensor whose element (row, h, d) has
 * index row*row_elems + h*head_dim + d; only heads [h0, h0+nh) are written,
 * packed as [nrows][nh][head_dim]. */
void kvo_gen_cache_rows(uint64_t seed, uint64_t stream, int64_t row0, int64_t nrows,
                        int32_t n_head_kv, int32_t head_dim, int32_t h0, int32_t nh,
                        uint16_t *out);

int32_t kvo_online_cores(void);

#ifdef __cplusplus
}
#endif
#endif /* KV_ORACLE_H */
