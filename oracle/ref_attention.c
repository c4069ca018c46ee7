/*
 * ref_attention.c -- TEST INFRASTRUCTURE ONLY.  Drives the reference's own
 * single-token attention so the CPU oracle (kv_oracle.c) can be checked
 * against reference code, not only against its own restatement.
 *
 * The reference's dense path (src/model.cpp) runs on ggml, which is not
 * vendored.  Its MoE engine (src/moe_stream) has a ggml-free decode attention
 * that computes the same operation on an F32 cache:
 *   qwen_model.c:346-353  RoPE table: cos/sin of pos * base^(-2i/hd) in double
 *   qwen_model.c:456-524  attention_block: per-head RMSNorm (Q/K norm) and
 *                         NEOX RoPE of q and k, k/v stored at row pos, then
 *                         for query head h the KV head h / (n_head/n_head_kv),
 *                         s = (q . k) * 1/sqrtf(hd), softmax over keys 0..pos,
 *                         out = sum_t p_t v_t
 * This file includes that translation unit (qwen_model.c, found through the
 * include path that oracle/build.py passes) and supplies only what a harness
 * needs around it: a model loaded by the reference's own qwen_load() from a
 * minimal GGUF file that the test writes (so its RoPE table is the
 * reference's), cache rows given by the test, and a backend whose matmul
 * returns the test's Q/K/V rows instead of projecting a hidden state.  RMSNorm,
 * RoPE and softmax stay the reference's scalar backend (compute_backend.c);
 * with use_norm == 0 the Q/K norm is skipped (identity), for the architectures
 * whose attention has none.
 *
 * Built by oracle/build.py into oracle/_ref/libref_attention.so from the
 * reference's sources where they lie; nothing in the product links it.
 */
#include "qwen_model.c"

/* the rows the harness's matmul hands back for attn_q / attn_k / attn_v */
static const float *g_rows_q, *g_rows_k, *g_rows_v;
static const struct qwen_model *g_model;

static void harness_matmul(void *self, uint32_t type, const uint8_t *w, uint64_t wkey, uint64_t ne0,
                           uint64_t ne1, const float *x, float *y)
{
    (void)self; (void)type; (void)wkey; (void)ne0; (void)x;
    const qwen_layer_t *L = &g_model->layers[0];
    const float *src = NULL;
    if (w == L->attn_q.data) src = g_rows_q;
    else if (w == L->attn_k.data) src = g_rows_k;
    else if (w == L->attn_v.data) src = g_rows_v;
    if (src) memcpy(y, src, (size_t)ne1 * sizeof(float));
    else memset(y, 0, (size_t)ne1 * sizeof(float));   /* attn_output: unused */
}

static void harness_rmsnorm_identity(void *self, float *out, const float *x, const float *w, int n, float eps)
{
    (void)self; (void)w; (void)eps;
    memmove(out, x, (size_t)n * sizeof(float));
}

/* Geometry of the model a GGUF file describes (after qwen_load); -1 on failure. */
int ref_model_geometry(const char *gguf_path, int max_seq, int *n_head, int *n_head_kv, int *head_dim,
                       float *rope_theta, float *eps)
{
    struct qwen_model *m = qwen_load(gguf_path, (size_t)1 << 20, 1, max_seq, 0);
    if (!m) return -1;
    *n_head = m->n_head;
    *n_head_kv = m->n_head_kv;
    *head_dim = m->head_dim;
    *rope_theta = m->rope_theta;
    *eps = m->eps;
    qwen_free(m);
    return 0;
}

/*
 * One decode step of layer 0 at position `pos`:
 *   k_rows, v_rows  [pos][n_head_kv*head_dim] F32: cache rows 0..pos-1
 *   q [n_head*head_dim], k, v [n_head_kv*head_dim]: the projection outputs
 *   use_norm        1: the reference's Q/K RMSNorm with the file's gamma
 * Outputs (any may be NULL):
 *   attn_out [n_head*head_dim]           the attention output (m->attn)
 *   k_out, v_out [n_head_kv*head_dim]    cache row pos as stored (K rotated)
 *   cos_out, sin_out [max_seq][head_dim/2] the reference's RoPE table
 * Returns 0, or -1 when the model cannot be loaded, -2 on a bad position.
 */
int ref_attention_step(const char *gguf_path, int max_seq, int pos, const float *k_rows, const float *v_rows,
                       const float *q, const float *k, const float *v, int use_norm, float *attn_out,
                       float *k_out, float *v_out, float *cos_out, float *sin_out)
{
    if (pos < 0 || pos >= max_seq) return -2;
    struct qwen_model *m = qwen_load(gguf_path, (size_t)1 << 20, 1, max_seq, 0);
    if (!m) return -1;
    const size_t nkvd = (size_t)m->n_head_kv * (size_t)m->head_dim;
    if (pos > 0) {
        memcpy(m->k_cache, k_rows, (size_t)pos * nkvd * sizeof(float));
        memcpy(m->v_cache, v_rows, (size_t)pos * nkvd * sizeof(float));
    }
    static compute_backend_t be;
    be = *compute_backend_scalar();
    be.name = "harness";
    be.matmul = harness_matmul;
    if (!use_norm) be.rmsnorm = harness_rmsnorm_identity;
    g_model = m;
    g_rows_q = q;
    g_rows_k = k;
    g_rows_v = v;
    m->be = &be;

    float *xbn = alloc_f32((size_t)m->n_embd), *xh = alloc_f32((size_t)m->n_embd);
    int rc = (xbn && xh) ? 0 : -1;
    if (rc == 0) {
        attention_block(m, &m->layers[0], 0, xbn, xh, pos);
        if (attn_out) memcpy(attn_out, m->attn, (size_t)m->n_head * m->head_dim * sizeof(float));
        if (k_out) memcpy(k_out, m->k_cache + (size_t)pos * nkvd, nkvd * sizeof(float));
        if (v_out) memcpy(v_out, m->v_cache + (size_t)pos * nkvd, nkvd * sizeof(float));
        const size_t tab = (size_t)max_seq * (size_t)(m->head_dim / 2) * sizeof(float);
        if (cos_out) memcpy(cos_out, m->rope_cos, tab);
        if (sin_out) memcpy(sin_out, m->rope_sin, tab);
    }
    free(xbn);
    free(xh);
    m->be = compute_backend_scalar();
    g_model = NULL;
    qwen_free(m);
    return rc;
}
