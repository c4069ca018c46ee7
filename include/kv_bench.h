/*
 * kv_bench.h -- measurement and synthetic-data helpers of the KV path library.
 *
 * Not part of the reference-facing boundary (kv_api.h): the reference has no
 * counterpart for these.  They exist so the benchmark and the tests can fill a
 * multi-GiB cache with seeded data on the device and time individual kernels.
 */
#ifndef KV_BENCH_H
#define KV_BENCH_H

#include "kv_api.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Fill cache rows [row0, row0+nrows) of K and V of every layer with the seeded
 * generator: element (row, global head h, dim d) of layer l's K gets
 * normal(seed, stream_base + 2l, row*n_head_kv*head_dim + h*head_dim + d), V
 * uses stream_base + 2l + 1, rounded to F16 (nearest even).  normal() is the
 * Irwin-Hall sum of twelve 16-bit uniforms from splitmix64, exact in F32, so
 * the CPU oracle regenerates identical bits. */
int kv_fill_synthetic(kv_ctx *ctx, uint64_t seed, uint64_t stream_base,
                      int64_t row0, int64_t nrows, void *stream);

/* dst[i] = normal(seed, stream, idx0 + i) for i < n, on the device. */
int kv_gen_normal_device(float *dst, uint64_t seed, uint64_t stream,
                         uint64_t idx0, int64_t n, void *cuda_stream);

/* Per-kernel timing with CUDA events recorded around each launch on the
 * launching stream.  Kernel ids below.  Enabling adds one event pair per
 * launch; totals accumulate until kv_profile_reset. */
#define KV_K_APPEND   0
#define KV_K_ATTN     1
#define KV_K_PREFILL  2   /* both tensor-core passes */
#define KV_K_PFOLD    3   /* the prefill statistics / output folds */
#define KV_K_GATHER   4
#define KV_K_PREFILL2 5   /* the one-pass chunk kernel on CTA pairs (head_dim 128) */
#define KV_K_COUNT    6
int kv_profile_enable(kv_ctx *ctx, int on);
int kv_profile_reset(kv_ctx *ctx);
/* Synchronizes the recorded events; returns launches and summed milliseconds. */
int kv_profile_read(kv_ctx *ctx, int32_t kernel, int64_t *launches, double *total_ms);
const char *kv_kernel_name(int32_t kernel);

/* Number of kernels this library launched since kv_alloc (host-side count). */
int64_t kv_launch_count(const kv_ctx *ctx);

/* Failure injection for tests.  what = 1: in the next decode launch the tile
 * producer withholds one tile, so the consumers' bounded wait expires (the
 * call's output is invalid and kv_status reports KV_E_TIMEOUT; no fault, no
 * hang).  limit_ns > 0 also sets the bound of every device-side wait of this
 * context (default 1 s); 0 keeps it. */
int kv_debug_inject(kv_ctx *ctx, int32_t what, uint64_t limit_ns);

/* Host-only pieces of kv_alloc, callable without a GPU (for checking):
 * the (cos, sin) RoPE table kv_alloc uploads, rows pos0 .. pos0+npos-1,
 * out[(p*(n_rot/2) + i)*2 + {0,1}]; and the heads shard `shard` of
 * cfg->n_shards owns. */
int kv_rope_table_host(const kv_config *cfg, int64_t pos0, int64_t npos, float *out);
int kv_shard_geometry(const kv_config *cfg, int32_t shard, int32_t *q_head0, int32_t *n_q_heads,
                      int32_t *kv_head0, int32_t *n_kv_heads);

/* The decode split's CTA count for a layer of n_kv keys over n_kv_heads_local
 * KV heads on a GPU with sm_count SMs (host arithmetic only): one CTA per SM
 * at most, at least 256 (head, key) rows a CTA, at least one per head, and a
 * multiple of the heads when that idles at most 5 % of them. */
int kv_decode_ctas(int32_t sm_count, int32_t n_kv_heads_local, int64_t n_kv, int32_t *n_cta);

/* The decode grid for a layer (host arithmetic only): n_cta CTAs in clusters
 * of cluster_ctas CTAs (1: no clusters), clusters_per_head per local KV head.
 * max_clusters[q] (q = 2..8; NULL: none) is the number of q-CTA clusters the
 * device holds at once.  One cluster per head when the head's keys fit its
 * CTAs (>= 256 keys each) at >= 85 % of kv_decode_ctas' CTA count; else no
 * clusters. */
int kv_decode_shape(int32_t sm_count, int32_t n_kv_heads_local, int64_t n_kv, const int32_t *max_clusters,
                    int32_t *n_cta, int32_t *cluster_ctas, int32_t *clusters_per_head);

/* 1 when a decode grid of n_cta CTAs is resident at once on sm_count SMs
 * holding blocks_per_sm CTAs each, else 0 (host arithmetic only).  The decode
 * kernel's CTAs wait on one another, so kv_alloc refuses a device where its
 * largest grid does not fit (blocks_per_sm from the CUDA occupancy query). */
int kv_decode_grid_fits(int32_t sm_count, int32_t blocks_per_sm, int32_t n_cta);

/* Per-CTA phase stamps of the decode kernel, in the measurement build only
 * (compiled with KV_PHASE_STAMPS: `python ggml-loader_b200/build.py --stamps`):
 * each launch records %globaltimer at its phases (entry, first tile issued,
 * griddepcontrol.wait returned, query rows rotated, K loop done, statistics
 * published / known, V loop done, output ticket, collector start / done,
 * exit) into a ring of launches.  Sets *ring and *max_cta, copies the ring
 * ([ring][max_cta][16]) to host_dst unless it is NULL, and returns the number
 * of launches stamped so far (launch i in slot i % ring); other builds return
 * KV_E_UNSUPPORTED. */
int64_t kv_debug_stamps(kv_ctx *ctx, unsigned long long *host_dst, int32_t *ring, int32_t *max_cta);

#ifdef __cplusplus
}
#endif
#endif /* KV_BENCH_H */
