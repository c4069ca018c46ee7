// kv_internal.h -- shared declarations of the KV path library (host <-> kernels).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace kvb {

// ---------------------------------------------------------------------------
// kv_append: QK-Norm + RoPE + RNE cast of one layer's new rows
// ---------------------------------------------------------------------------
struct AppendParams {
    const float *q, *k, *v;          // token 0 of each block (global heads)
    int64_t q_stride, k_stride, v_stride;
    const float *q_norm_w, *k_norm_w; // [D] or null
    const float *q_bias, *k_bias, *v_bias;   // [heads*D] (global heads) or null: added first
    int32_t n_new;
    int64_t n_past;
    int32_t hq_loc, hkv_loc;         // heads owned by this context
    int32_t hq0, hkv0;               // first owned global head
    int32_t n_rot, rope_mode, qk_norm;   // qk_norm: 0 none, 1 RMSNorm * gamma before RoPE, 2 nGPT after RoPE
    float eps;                       // RMSNorm's eps (nGPT: 1e-6 / D)
    float post;                      // nGPT: 1 / sqrt(D)
    const float2 *rope;              // [n_ctx][n_rot/2] (cos, sin)
    __half *kc, *vc;                 // layer cache [rows][hkv_loc][D]
    __half *qbuf;                    // [n_new][hq_loc][D]  rotated Q, F16
    int64_t ring;                    // 0: position p in row p; > 0: in row p % ring (ring cache)
};

cudaError_t launch_append(int D, bool vec_loads, const AppendParams &p, cudaStream_t st);
// a ring cache's visibility mask for a chunk at positions [pos0, pos0+n_tokens):
// [n_tokens] F16 rows of `stride` elements over its n_used cells
cudaError_t launch_ring_mask(__half *dst, int64_t stride, int64_t n_cells, int64_t pos0, int n_tokens, int64_t n_used,
                             cudaStream_t st);

// ---------------------------------------------------------------------------
// attention of kv_attend (kv_attend.cu): one TMA-fed, tensor-core kernel per
// layer and group of <= 8 query rows, chained with programmatic dependent launch
// ---------------------------------------------------------------------------
constexpr int kMaxLocalHeads = 64;   // KV heads one context may own
constexpr int kMaxShards = 8;        // KV-head shards exchanging outputs over peer memory

struct AttnParams {
    int32_t hkv, r, hq_loc;          // local KV heads, GQA group, local query heads
    int32_t hq0, hkv0;               // first owned global head (inputs are replicated rows)
    int64_t n_kv, n_past;
    int32_t row0, nrows;             // query rows of this launch (row = t*r + j), nrows <= attn_rows()
    int32_t n_cta;                   // CTAs; hkv <= n_cta <= min(SMs, attn_max_ctas(), hkv*n_kv), all resident
    // cluster mode (cq > 1, head_dim <= 128): clusters of cq CTAs, ncl of them
    // per local head (n_cta = hkv * ncl * cq); a cluster's CTAs exchange the
    // statistics and partial outputs through distributed shared memory
    int32_t cq, ncl;
    // tiles sent to L2 ahead of the ring where the producer waits longest: the
    // count in bits 0-7 (0: none); bit 8: at its first wait (behind the previous
    // kernel's tail), bit 9: at its first wait among the V tiles (behind the
    // statistics exchange)
    int32_t l2pf;
    float scale;
    // single-token append done inside the kernel (decode): fused = 1
    int32_t fused;
    const float *q, *k, *v;          // token 0's Q/K/V blocks (global heads)
    int64_t q_stride;
    const float *q_norm_w, *k_norm_w;
    const float *q_bias, *k_bias, *v_bias;   // [heads*D] (global heads) or null: added first
    int32_t qk_norm, n_rot, rope_mode;
    float eps;
    const float2 *rope;              // [n_ctx][n_rot/2]
    __half *kc, *vc;                 // this layer's cache [n_ctx][hkv][D] (new rows written here)
    // a cache row the previous launch in the stream may still be writing
    // (the row a fused launch of this layer appended), -1 if none
    int64_t hz_row;
    // multi-token: rotated Q from the append kernel
    const __half *qbuf;              // [n_new][hq_loc][D]
    // scratch
    float *S;                        // scores: CTA c, tile i, warp w -> S + ((c*S_tiles + i)*8 + w)*128
    int64_t S_tiles;                 // tiles reserved per CTA
    unsigned long long *stats;       // [n_cta][2][8][2] (max, sum of exp) per (CTA, segment, row),
                                     // each word = epoch << 32 | float bits
    uint32_t epoch;                  // tag of this launch's statistics (never 0)
    long long *acc;                  // [hkv][8][D] output accumulators, fixed point 2^-40, zero between calls
    unsigned *counters;              // [hkv] output tickets, zero between calls
    unsigned *nonfin;                // [hkv] rows (bit per row) with a non-finite partial output, zero between calls
    unsigned *err;                   // error word (1: consumer tile wait, 2: producer, 4: statistics wait)
    uint64_t limit_ns;               // bound of every device-side wait
    int32_t inject;                  // test hook: 1 = producers withhold tile 1
    // the caller's additive mask (nullptr: the implicit causal mask): score =
    // dot*scale + mask[token*mask_stride + key], F16 when mask_f16
    const void *mask;
    int64_t mask_stride;
    int32_t mask_f16;
    // 1: the flash-attn branch -- weights exp(s - M) rounded to F16 unnormalised,
    // the partial output scaled by 1/Z; a row without a visible key gives 0
    int32_t flash;
    // 1: every key < n_kv is visible (a ring cache's single token), no causal bound
    int32_t all_keys;
    // 1: the producer waits for the previous kernel before its first tile (a ring
    // cache's new rows may sit in any tile)
    int32_t wait_first;
    // output
    float *out;
    int64_t out_stride;
    int32_t out_head0;
    // KV-head shards exchanging decode outputs over NVLink (n_peers = shards, 0 = none):
    // rx[g] = shard g's receive buffer, 2 parities x rx_stride words, one word
    // per output float of the full row (written by the shard that owns each
    // head) = epoch << 32 | float bits, so a word is valid once its tag shows
    // the launch; xticket counts this launch's converted local heads
    int32_t n_peers, shard;
    // 0: push -- a head's words go into every peer's buffer, the collector
    // polls its own; 1: pull -- a head's words stay in this shard's buffer,
    // the collector polls each peer's buffer over NVLink (no remote stores)
    int32_t xpull;
    unsigned long long *rx[kMaxShards];
    int64_t rx_stride;
    unsigned *xticket;
    // CTAs [span_a[h], span_b[h]] cover local head h; span_slot[h] is the
    // segment index head h has in CTA span_a[h] (1 when that CTA starts in head h-1)
    int16_t span_a[kMaxLocalHeads], span_b[kMaxLocalHeads];
    int8_t span_slot[kMaxLocalHeads];
    // builds with KV_PHASE_STAMPS only (measurement): [n_cta][kStampSlots]
    // %globaltimer stamps of this launch's phases, nullptr otherwise
    unsigned long long *stamps;
};
constexpr int kStampSlots = 16;

// query rows per launch (8), keys per tile (128), the column-box width of the
// K/V tensor maps (64 halves, 128-byte swizzle; 32, 64-byte swizzle at 96), and
// the floats of score scratch one tile takes
int attn_rows();
int attn_tile_keys();
int attn_box_width(int D);
int attn_tile_scores();
int attn_max_ctas();   // CTAs one launch may have (a head's span is read in one sweep)
cudaError_t attn_prepare(int D);
// CTAs of the attention kernel one SM holds at once (the fewest over its instances)
cudaError_t attn_occupancy(int D, int *blocks_per_sm);
// clusters of q CTAs of the attention kernel the device holds at once (0: no
// cluster mode at this head_dim)
cudaError_t attn_cluster_occupancy(int D, int q, int *clusters);
constexpr int kMaxClusterCtas = 8;
// the split's per-launch tables (score tiles per CTA, each head's CTA span) for ap.n_cta CTAs
void attn_split(AttnParams &ap, int hkv, int64_t n_kv);
// CTAs of the plain (cluster-less) decode split
int attn_plain_ctas(int sm_count, int hkv, int64_t n_kv);
// one layer's K or V cache [rows][hkv][D] F16 as the attention kernel's tensor map (KV_OK or an error code)
int encode_cache_map(CUtensorMap *m, const void *base, int64_t rows, int hkv, int D);
// pdl: launch as a programmatic dependent of the previous kernel in the stream;
// coop: as a cooperative launch (the driver starts the grid only with every CTA resident)
cudaError_t launch_attn(int D, const CUtensorMap &kmap, const CUtensorMap &vmap, const AttnParams &p,
                        cudaStream_t st, bool pdl, bool coop);

// ---------------------------------------------------------------------------
// chunked-prefill attention (kv_prefill.cu): tcgen05 tensor cores, two passes
// ---------------------------------------------------------------------------
struct PrefillParams {
    int32_t hkv, r, hq_loc, D;
    int64_t n_past;
    int32_t n_new;
    int32_t tb;        // tokens per 128-row query tile (tb * r <= 128)
    int32_t nt;        // query tiles a CTA holds (prefill_tiles: 2, or 1 at head_dim 256; 4 a CTA pair)
    int32_t dv;        // the heads' real width in the output rows (the kernel's D, or 96 run as 128)
    int32_t nblk;      // blocks of nt query tiles: ceil(n_new / (nt tb)); pair = kv head * nblk + block
    int64_t s_all;     // key tiles of one KV head summed over its blocks
    int32_t n_cta, kseg;
    float scale;
    int32_t mode;      // 0 one pass (online softmax), 2 the exact two passes (long contexts)
    float *pstat;      // [n_cta][kseg][nt tiles][128] (m, l) per segment and row
    float *pout;       // [n_cta][kseg][nt tiles][128][D] partial outputs of split pairs
    float2 *rstat;     // [hkv * nblk][256] (M, 1/Z) per pair and row (exact passes)
    float *out;        // row t at out + t*out_stride, head h at (out_head0 + h)*D
    int64_t out_stride;
    int32_t out_head0;
    const void *mask;  // as AttnParams: the caller's additive mask, nullptr = causal
    int64_t mask_stride;
    int32_t mask_f16;
    int32_t mask_vec;  // mask rows start on 16-byte boundaries: vector loads
    int32_t flash;     // the flash-attn branch: a row without a visible key gives 0
    unsigned *err;
    uint64_t limit_ns;
};

bool prefill_supported(int D);
int prefill_tiles(int D);
int prefill_kernel_dim(int D);   // the kernel instance a head_dim runs on
int prefill_max_segments();
cudaError_t prefill_prepare(int D);
// which: 0 the one-pass attention kernel, 1 the fold of pairs split over CTAs;
// the exact two passes: 2 statistics kernel, 3 statistics fold, 4 output kernel
cudaError_t launch_prefill(int D, int which, const CUtensorMap &qmap, const CUtensorMap &kmap,
                           const CUtensorMap &vmap, const PrefillParams &p, cudaStream_t st);
// The CTA-pair (tcgen05 cta_group::2) form of the one-pass kernel at head_dim
// 128: p.nt = 4 query tiles a 2-CTA cluster, p.n_cta clusters (2 * n_cta
// CTAs); kmap32 is the layer's K map with 32-key boxes.  prepare returns the
// number of its clusters the device holds at once (0: not available).
cudaError_t prefill_pair_prepare(int *clusters);
cudaError_t launch_prefill_pair(const CUtensorMap &qmap, const CUtensorMap &kmap32, const CUtensorMap &vmap,
                                const PrefillParams &p, cudaStream_t st);

// ---------------------------------------------------------------------------
// gather / layout helpers
// ---------------------------------------------------------------------------
// out[t][g*cols + c] = src[g][t][c] for g < G, t < n_new, c < cols
cudaError_t launch_unshard(float *out, int64_t out_stride, const float *src, int G, int n_new,
                           int cols, cudaStream_t st);

// ---------------------------------------------------------------------------
// synthetic data (bench / tests)
// ---------------------------------------------------------------------------
struct FillParams {
    __half *cache;                   // base of all layers
    int32_t n_layer, D, hkv_loc, hkv_total, hkv0;
    int64_t n_ctx, row0, nrows;
    uint64_t seed, stream_base;
};
cudaError_t launch_fill(const FillParams &p, cudaStream_t st);
cudaError_t launch_gen_normal(float *dst, uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n,
                              cudaStream_t st);

// Records the detail string kv_last_error() returns on this host thread.
int set_last_error(int code, const char *msg);

}  // namespace kvb
