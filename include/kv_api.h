/*
 * kv_api.h -- C ABI of the B200 KV-cache append + attention path.
 *
 * This is the drop-in boundary for GGML-Loader's per-layer KV-cache hot path
 * (src/model.cpp in the reference).  A caller that today builds the ggml op
 * sequence in build_graph() for the phi3 / qwen2 / qwen3 / llama architectures
 * calls, per layer:
 *
 *     kv_append(ctx, layer, n_past, n_new, q, k, v, ...)   -- replaces the
 *         QK-Norm (model.cpp:1382-1387), ggml_rope_ext (1389-1404) and the
 *         ggml_cpy of K/V into the cache view (1406-1414);
 *     kv_attend(ctx, layer, n_past, n_new, out, ...)        -- replaces the
 *         attention over cache rows [0, n_past+n_new): ggml_mul_mat(K,Q),
 *         ggml_soft_max_ext with the causal mask, ggml_mul_mat(V^T, KQ) and the
 *         output permute (1416-1445), or the flash-attn branch (1426-1434).
 *
 * and at start-up kv_alloc() in place of init_kv_cache() (model.cpp:821-867),
 * with the context auto-sizing of auto_n_ctx() (model.cpp:1002-1059) computed
 * from free HBM instead of /proc/meminfo.
 *
 * Conventions
 *  - All tensors passed to kv_append / kv_attend are DEVICE pointers, F32.
 *  - Calls are ordered on the given CUDA stream (a cudaStream_t passed as
 *    void*; NULL = the legacy default stream).  No call blocks the host except
 *    kv_alloc, kv_free and the row import/export helpers.
 *  - Errors are negative return codes; the library never exits the process
 *    (the reference prints and calls exit(1), model.cpp:859-865).
 *  - One host thread drives one kv_ctx; the context's scratch is shared by
 *    its calls, so calls on one context must not overlap on the device.
 */
#ifndef KV_API_H
#define KV_API_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes -------------------------------------------------------- */
#define KV_OK              0
#define KV_E_ARG          -1  /* bad argument or unsupported shape          */
#define KV_E_OOM          -2  /* device or host allocation failed           */
#define KV_E_RANGE        -3  /* row range outside [0, n_ctx) / batch limit */
#define KV_E_CUDA         -4  /* CUDA runtime error                         */
#define KV_E_COMM         -5  /* collective (NCCL) error                    */
#define KV_E_TIMEOUT      -6  /* a bounded device-side wait gave up         */
#define KV_E_STATE        -7  /* call order violated (attend w/o append)    */
#define KV_E_UNSUPPORTED  -8  /* feature not built / not available          */

/* ---- RoPE modes (ggml values, model.cpp:1395) ---------------------------- */
#define KV_ROPE_NORMAL 0      /* adjacent pairs (llama)                   */
#define KV_ROPE_NEOX   2      /* split halves (phi3 / qwen2 / qwen3)      */

typedef struct kv_ctx kv_ctx;

/*
 * Model attention parameters, the subset of `struct hparams` (model.h:63-95)
 * that the path reads, plus allocation and sharding options.
 */
typedef struct kv_config {
    int32_t n_layer;            /* hparams::n_layer                               */
    int32_t n_head;             /* hparams::n_head (query heads, whole model)     */
    int32_t n_head_kv;          /* hparams::n_head_kv                             */
    int32_t head_dim;           /* hparams::n_embd_head; 64, 96, 128 or 256 (256:
                                   whole-head RoPE)                             */
    int32_t n_rot;              /* hparams::n_rot (even, <= head_dim)             */
    int32_t rope_mode;          /* KV_ROPE_NORMAL (llama) / KV_ROPE_NEOX (others) */
    float   rope_base;          /* hparams::rope_freq_base                        */
    float   rope_freq_scale;    /* 1.0 for every reference architecture           */
    float   rope_attn_factor;   /* hparams::rope_attn_factor (mscale)             */
    float   rope_ext_factor;    /* 1.0 with phi3 LongRoPE, else 0 (model.cpp:1312)*/
    float   rope_beta_fast;     /* 32 with LongRoPE, else 0                       */
    float   rope_beta_slow;     /* 1 with LongRoPE, else 0                        */
    int32_t n_ctx_orig;         /* hparams::n_ctx_orig                            */
    const float *rope_freq_factors; /* HOST [n_rot/2] or NULL; copied by kv_alloc.
                                   phi3 rope_factors_short (model.cpp:555-557) or
                                   llama3 rope_freqs                             */
    int32_t qk_norm;            /* 1: hparams::has_qk_norm (qwen3): RMSNorm * gamma
                                   before RoPE.  2: dory's nGPT handling
                                   (dory.c:577-580, 646-649): after RoPE,
                                   rms_norm(x, rms_eps/head_dim) / sqrt(head_dim),
                                   Q then times q_norm_w [n_head][head_dim] (the
                                   squared learned scale); k_norm_w unused     */
    float   rms_eps;            /* hparams::rms_eps                               */
    int64_t n_ctx;              /* cache positions (<= 2^31); 0 = auto from free HBM */
    int64_t n_ctx_train;        /* auto-sizing clamp; 0 = 262144 cap              */
    int32_t longrope_clamp;     /* 1: auto-sizing also clamps to n_ctx_orig
                                   (phi3 with LongRoPE, model.cpp:1037-1039)     */
    int32_t n_batch_max;        /* max n_new per call; 0 = 512                    */
    int32_t device;             /* CUDA device ordinal; -1 = current device       */
    int32_t n_shards;           /* GPUs sharing the cache by KV head; 0/1 = one   */
    int32_t shard;              /* this context's shard index in [0, n_shards)    */
    const void *comm_id;        /* 128-byte id from kv_comm_unique_id() on shard 0,
                                   the same bytes on every shard; n_shards > 1    */
    int64_t ring_cells;         /* 0: linear cache, position p in row p.  > 0: a
                                   ring of ring_cells rows (dory.c:391-522), the
                                   token at position p in row p % ring_cells;
                                   n_ctx then bounds the positions (RoPE table)  */
    int32_t flash_attn;         /* 1: kv_attend (and kv_forward) take the flash-attn
                                   branch, as decode_session::use_flash_attn
                                   selects it (model.h:381-384); see
                                   KV_ATTN_FLASH at kv_attend_mask              */
} kv_config;

/* Defaults: NEOX RoPE, base 10000, scale 1, attn factor 1, no YaRN, eps 1e-6,
 * n_ctx 0 (auto), n_batch_max 512, device -1, one shard, linear cache.  Shape
 * fields 0.
 *
 * Ring caches (ring_cells > 0; dory's sliding and global rings, one context
 * per ring size, per-loop slots as extra layers): kv_append's n_past is the
 * position of the first new token (RoPE and the cell p % ring_cells; n_new <=
 * ring_cells), and kv_attend attends over the min(ring_cells, n_past + n_new)
 * cells in use with dory_fill_attn_mask's visibility (dory.c:553-575: a cell
 * is visible to the query at p when its newest write is a real position <= p),
 * built on the device; kv_attend_mask takes the caller's mask over those cells
 * instead (mask_stride >= the cells in use). */
int kv_config_init(kv_config *cfg);

/* Bytes of the whole K+V cache at n_ctx positions, all layers and all shards:
 * exactly kv_cache_bytes() of the reference (model.cpp:869-885); a ring
 * configuration holds min(ring_cells, n_ctx) rows.  UINT64_MAX when the product
 * does not fit 64 bits. */
uint64_t kv_cache_bytes(const kv_config *cfg, int64_t n_ctx);

/* Context auto-sizing rule of auto_n_ctx() (model.cpp:1002-1059) applied to
 * `free_bytes` of one GPU: (free - 384 MiB) * 0.8 / per-position bytes of this
 * shard (cache rows + RoPE table row), rounded down to a multiple of 64,
 * clamped to n_ctx_train (262144 if 0) and n_ctx_orig with longrope_clamp,
 * floor 512.  free_bytes <= 0 gives the reference's fallback, 4096. */
int64_t kv_auto_n_ctx(const kv_config *cfg, int64_t free_bytes);

/* Allocate the cache (+ RoPE table + scratch) on the configured device;
 * replaces init_kv_cache (model.cpp:821-867).  With cfg->n_ctx == 0 the size
 * comes from kv_auto_n_ctx(cudaMemGetInfo free).  With n_shards > 1 this
 * context owns KV heads [shard*n_head_kv/n_shards, (shard+1)*...) and the
 * matching query heads, and joins the collective identified by comm_id (every
 * shard must call kv_alloc concurrently, one process or thread per GPU).
 * Returns KV_OK, KV_E_ARG, KV_E_OOM, KV_E_CUDA or KV_E_COMM. */
int kv_alloc(const kv_config *cfg, kv_ctx **out);

/* Release everything kv_alloc acquired.  NULL is a no-op. */
int kv_free(kv_ctx *ctx);

/* Positions the cache holds (the n_ctx actually allocated). */
int kv_n_ctx(const kv_ctx *ctx, int64_t *n_ctx);

/*
 * Append n_new tokens' K and V rows at cache rows [n_past, n_past+n_new) of
 * `layer`, after QK-Norm (if cfg->qk_norm) and RoPE of K; also rotates Q into
 * the context for the following kv_attend.  Replaces model.cpp:1382-1414.
 *
 * q: token t's Q block (n_head*head_dim floats, heads outer) at q + t*q_stride;
 * k, v likewise with n_head_kv*head_dim floats.  For phi3's fused QKV output
 * (model.cpp:1088-1094) pass q = row, k = row + n_head*head_dim,
 * v = row + (n_head+n_head_kv)*head_dim and all three strides equal to the
 * fused row width.  q_norm_w / k_norm_w: [head_dim] gamma of this layer, or
 * NULL without QK-Norm.  Sharded contexts read only their own heads.
 * The F32 -> F16 cast rounds to nearest even; cache bytes equal the reference
 * CPU path's bit for bit.
 */
int kv_append(kv_ctx *ctx, int32_t layer, int64_t n_past, int32_t n_new,
              const float *q, int64_t q_stride,
              const float *k, int64_t k_stride,
              const float *v, int64_t v_stride,
              const float *q_norm_w, const float *k_norm_w,
              void *stream);

/*
 * kv_append with the QKV bias of qwen2-style layers (model.cpp:1099-1102,
 * ggml_add of attn_q/k/v.bias to the projections) added inside the append's
 * load: q_bias [n_head*head_dim], k_bias and v_bias [n_head_kv*head_dim], F32
 * device pointers of this layer, or NULL (no bias).  Each element is one
 * rounded F32 add before QK-Norm and RoPE, as ggml_add is.  kv_append is this
 * call with three NULL biases.
 */
int kv_append_bias(kv_ctx *ctx, int32_t layer, int64_t n_past, int32_t n_new,
                   const float *q, int64_t q_stride,
                   const float *k, int64_t k_stride,
                   const float *v, int64_t v_stride,
                   const float *q_norm_w, const float *k_norm_w,
                   const float *q_bias, const float *k_bias, const float *v_bias,
                   void *stream);

/*
 * Attention of the n_new tokens last appended to `layer` (same layer, n_past
 * and n_new as that kv_append) over cache rows [0, n_past+n_new) with the
 * causal mask k <= n_past+t (model.cpp:1579-1586) and scale 1/sqrt(head_dim).
 * out: [n_new][n_head*head_dim] F32, heads outer -- the layout of
 * `cur` after ggml_cont_2d at model.cpp:1444.  With n_shards > 1 every shard
 * receives the whole gathered output.  Only rows < n_past+n_new are read, so
 * rewinding n_past and overwriting rows is allowed (cmd_chat.cpp:749-764).
 */
int kv_attend(kv_ctx *ctx, int32_t layer, int64_t n_past, int32_t n_new,
              float *out, void *stream);

/* Mask element types and flags of kv_attend_mask. */
#define KV_MASK_F32    0   /* ggml_soft_max_ext's mask (model.cpp:1437)          */
#define KV_MASK_F16    1   /* the flash branch's ggml_cast mask (model.cpp:1431) */
#define KV_ATTN_FLASH  1u  /* the ggml_flash_attn_ext branch (model.cpp:1426-1434) */

/*
 * kv_attend with the reference's explicit additive mask in place of the
 * implicit causal one, and the choice of the reference's two attention
 * branches (decode_session::use_flash_attn, model.h:381-384).  Same call order
 * and output as kv_attend.
 *
 * mask: DEVICE pointer to n_new rows of at least n_past+n_new elements,
 * mask_stride elements apart (the [n_kv, n_new] mask model.cpp:1579-1586
 * builds, rows padded as ggml pads them), F32 (KV_MASK_F32) or F16
 * (KV_MASK_F16); the score of token t and key k is dot*scale + mask[t][k], so
 * -inf removes the key.  NULL keeps the implicit causal mask.  Rows starting on
 * 16-byte boundaries are read with vector loads.
 * flags: 0 = the default branch (ggml_soft_max_ext then ggml_mul_mat: the
 * normalised weights rounded to F16); KV_ATTN_FLASH = the ggml_flash_attn_ext
 * branch: the weights exp(s - max) are not normalised before the F16 rounding
 * (the output is divided by their sum), and a row whose keys are all masked
 * gives 0 (the default branch gives NaN, as ggml's soft_max of an all -inf
 * row).  The flash branch's output layout [head_dim, n_head, n_new] is the
 * same memory order as `out` here.
 * Returns KV_OK, KV_E_ARG (unknown type or flag, mask_stride < n_past+n_new)
 * or the codes of kv_attend.
 */
int kv_attend_mask(kv_ctx *ctx, int32_t layer, int64_t n_past, int32_t n_new,
                   const void *mask, int32_t mask_type, int64_t mask_stride,
                   uint32_t flags, float *out, void *stream);

/*
 * One step of the path over every layer: for layer l in [0, n_layer),
 * kv_append then kv_attend with inputs at q + l*in_layer_stride (likewise k,
 * v), gammas at q_norm_w + l*norm_layer_stride, output at
 * out + l*out_layer_stride.  The per-layer loop of forward_step
 * (model.cpp:1318, 1496-1597) restricted to this path, driven from C++.
 */
int kv_forward(kv_ctx *ctx, int64_t n_past, int32_t n_new,
               const float *q, int64_t q_stride,
               const float *k, int64_t k_stride,
               const float *v, int64_t v_stride, int64_t in_layer_stride,
               const float *q_norm_w, const float *k_norm_w, int64_t norm_layer_stride,
               float *out, int64_t out_layer_stride, void *stream);

/*
 * Decode attention that allocates nothing.  No counterpart in the reference:
 * it exists for callers that cannot call cudaMalloc -- a host framework that
 * owns and plans all device memory up front (ggml's graph allocator, a serving
 * engine that reserves HBM for its own pool) and runs this op as a callback in
 * the middle of its compute, where an allocation would fail for lack of free
 * memory or stall the device.  Such a caller cannot hold a kv_ctx (kv_alloc
 * allocates), so it passes its own cache and buffers:
 *   k_cache, v_cache: one layer's cache, [rows][n_head_kv][head_dim] F16,
 *                     16-byte aligned; rows [0, n_kv) are attended, the new
 *                     token's K/V already written at row n_kv-1;
 *   q:   the new token's rotated query, [n_head][head_dim] F32 (device);
 *   out: [n_head*head_dim] F32 (device), the layout kv_attend writes.
 * It runs kv_attend's decode attention kernel (its default branch -- not the
 * flash-attn one -- over a plain grid, launched cooperatively so the driver
 * starts it only with all its CTAs resident).  Its scratch is a fixed 16 MiB
 * array built into the library (held by every GPU that loads it until exit);
 * a call needs about 32 bytes of it per (KV head, key) for scores -- about
 * 56k keys with 8 KV heads, 14k with 32 -- and returns KV_E_RANGE, with
 * kv_last_error() saying so, when the shape does not fit.  The first call on
 * a device looks up the array's device address and sets up the kernel, so
 * make it before any stream capture; a cudaDeviceReset() invalidates that
 * set-up for the rest of the process.  Calls share the array: calls that
 * overlap on the GPU race and must be serialised.
 */
int kv_attend_decode_noalloc(const uint16_t *k_cache, const uint16_t *v_cache,
                             int32_t n_head, int32_t n_head_kv, int32_t head_dim, int64_t n_kv,
                             const float *q, float *out, void *stream);

/* Copy cache rows [row0, row0+nrows) of K (which = 0) or V (which = 1) of
 * `layer` to / from host memory in the reference layout [row][head][dim] F16
 * (this context's heads only).  Synchronous.  Used for checking, for the
 * reference's /save-/load style rebuilds and for tests. */
int kv_export_rows(kv_ctx *ctx, int32_t layer, int32_t which, int64_t row0,
                   int64_t nrows, uint16_t *host_dst);
int kv_import_rows(kv_ctx *ctx, int32_t layer, int32_t which, int64_t row0,
                   int64_t nrows, const uint16_t *host_src);

/* Shard geometry of a context: first global query head, query heads, first
 * global KV head, KV heads. */
int kv_shard_info(const kv_ctx *ctx, int32_t *q_head0, int32_t *n_q_heads,
                  int32_t *kv_head0, int32_t *n_kv_heads);

/* 128-byte identifier for a new collective; call on shard 0 and hand the
 * bytes to every shard's kv_config.comm_id.  KV_E_UNSUPPORTED when NCCL
 * (libnccl.so.2) cannot be loaded. */
int kv_comm_unique_id(void *id_out);

/* Deferred device-side errors: waits for `stream`, then returns KV_E_TIMEOUT
 * (and clears the record) if a bounded wait inside one of this context's
 * kernels expired since the last check -- the outputs of that call are not
 * valid -- else KV_OK.  The context stays usable either way. */
int kv_status(kv_ctx *ctx, void *stream);

const char *kv_strerror(int code);
/* Detail of the last failing call on this host thread ("" if none). */
const char *kv_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* KV_API_H */
