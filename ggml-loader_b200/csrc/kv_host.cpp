// kv_host.cpp -- host side of the KV path library: the C ABI of include/kv_api.h
// and include/kv_bench.h.
//
// Owns the per-context device memory (cache, RoPE table, scratch), the context
// sizing rule, argument checking and the kernel launch sequence of one layer:
//   kv_append -> append kernel
//   kv_attend -> scores kernel + P.V kernel (per group of query rows)
//                [+ NCCL all-gather of the head outputs when sharded]
// Compiled with -ffp-contract=off: the RoPE table is compared bit-for-bit with
// the CPU path, whose products and sums are separately rounded.
#include <dlfcn.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <exception>
#include <new>
#include <string>
#include <system_error>
#include <thread>
#include <vector>

#include "kv_api.h"
#include "kv_bench.h"
#include "kv_internal.h"

namespace {

// the fewest keys a decode CTA streams (two 128-key tiles): more CTAs than
// that would spend more time in the statistics exchange than they save
constexpr int kDecodeMinKeys = 256;

// a fixed buffer: recording an error never allocates, so it also works while
// reporting a failed host allocation
thread_local char g_last_error[512];

int fail(int code, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char *what)
{
    return fail(KV_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// C callers cannot catch a C++ exception: the entry points that allocate host
// memory (the RoPE table, TMA descriptor and segment-table vectors, error
// strings) run their body through this and return KV_E_OOM instead of letting
// std::bad_alloc (or a failed thread start) end the caller's process.
template <class F>
int guarded(const char *what, F &&fn) noexcept
{
    try {
        return fn();
    } catch (const std::bad_alloc &) {
        return fail(KV_E_OOM, "%s: host memory allocation failed", what);
    } catch (const std::exception &ex) {
        return fail(KV_E_OOM, "%s: host resources exhausted (%s)", what, ex.what());
    } catch (...) {
        return fail(KV_E_OOM, "%s: host resources exhausted", what);
    }
}

#define KV_CUDA(call)                                     \
    do {                                                  \
        cudaError_t e_ = (call);                          \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
    } while (0)

// ---------------------------------------------------------------------------
// NCCL, loaded at run time so single-GPU use needs no NCCL at all
// ---------------------------------------------------------------------------
struct NcclId {
    char internal[128];
};
typedef struct ncclComm *ncclComm_t;
constexpr int kNcclFloat32 = 7;

struct NcclApi {
    bool tried = false;
    void *h = nullptr;
    int (*GetUniqueId)(NcclId *) = nullptr;
    int (*CommInitRank)(ncclComm_t *, int, NcclId, int) = nullptr;
    int (*AllGather)(const void *, void *, size_t, int, ncclComm_t, cudaStream_t) = nullptr;
    int (*CommDestroy)(ncclComm_t) = nullptr;
    const char *(*GetErrorString)(int) = nullptr;
};

NcclApi &nccl()
{
    static NcclApi api;
    if (!api.tried) {
        api.tried = true;
        api.h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!api.h) api.h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (api.h) {
            api.GetUniqueId = (int (*)(NcclId *))dlsym(api.h, "ncclGetUniqueId");
            api.CommInitRank = (int (*)(ncclComm_t *, int, NcclId, int))dlsym(api.h, "ncclCommInitRank");
            api.AllGather = (int (*)(const void *, void *, size_t, int, ncclComm_t, cudaStream_t))dlsym(
                api.h, "ncclAllGather");
            api.CommDestroy = (int (*)(ncclComm_t))dlsym(api.h, "ncclCommDestroy");
            api.GetErrorString = (const char *(*)(int))dlsym(api.h, "ncclGetErrorString");
            if (!api.GetUniqueId || !api.CommInitRank || !api.AllGather || !api.CommDestroy) {
                api.GetUniqueId = nullptr;
            }
        }
    }
    return api;
}

// ---------------------------------------------------------------------------
// RoPE table: (cos, sin) per (position, pair), the ggml_rope_ext angle schedule
// (model.cpp:1396-1403 with the parameters of model.cpp:1312-1316)
// ---------------------------------------------------------------------------
float yarn_dim(int n_dims, int n_ctx_orig, float n_turns, float base)
{
    const float two_pi = 2.0f * (float)M_PI;
    return (float)n_dims * logf((float)n_ctx_orig / (n_turns * two_pi)) / (2.0f * logf(base));
}

struct RopeSpec {
    int n_rot;
    float base, freq_scale, attn_factor, ext_factor, beta_fast, beta_slow;
    int n_ctx_orig;
    const float *ff;  // [n_rot/2] or null
};

void rope_rows(const RopeSpec &r, int64_t p0, int64_t p1, float *out)
{
    const int half = r.n_rot / 2;
    const float step = powf(r.base, -2.0f / (float)r.n_rot);
    float lo = 0.0f, hi = 0.0f;
    if (r.ext_factor != 0.0f) {
        const float a = floorf(yarn_dim(r.n_rot, r.n_ctx_orig, r.beta_fast, r.base));
        const float b = ceilf(yarn_dim(r.n_rot, r.n_ctx_orig, r.beta_slow, r.base));
        lo = a > 0.0f ? a : 0.0f;
        hi = b < (float)(r.n_rot - 1) ? b : (float)(r.n_rot - 1);
    }
    for (int64_t p = p0; p < p1; p++) {
        float theta = (float)p;
        float *row = out + (size_t)(p - p0) * (size_t)half * 2u;
        for (int i = 0; i < half; i++) {
            const float f = r.ff ? r.ff[i] : 1.0f;
            const float t_ext = theta / f;
            const float t_int = r.freq_scale * t_ext;
            float t = t_int;
            float ms = r.attn_factor;
            if (r.ext_factor != 0.0f) {
                const float den = (hi - lo) > 0.001f ? (hi - lo) : 0.001f;
                float y = ((float)i - lo) / den;  // pair index == i0/2
                y = y < 0.0f ? 0.0f : (y > 1.0f ? 1.0f : y);
                const float mix = (1.0f - y) * r.ext_factor;
                t = t_int * (1.0f - mix) + t_ext * mix;
                ms *= 1.0f + 0.1f * logf(1.0f / r.freq_scale);
            }
            row[2 * i + 0] = cosf(t) * ms;
            row[2 * i + 1] = sinf(t) * ms;
            theta *= step;
        }
    }
}

void build_rope_table(const RopeSpec &r, int64_t n_pos, float *out)
{
    const int64_t half = r.n_rot / 2;
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 1;
    if (nt > 32) nt = 32;
    if (n_pos < 4096) nt = 1;
    const int64_t chunk = (n_pos + nt - 1) / nt;
    std::vector<std::thread> th;
    th.reserve(nt);
    int64_t handed = 0;   // rows [0, handed) belong to started threads
    for (unsigned w = 0; w < nt; w++) {
        const int64_t a = (int64_t)w * chunk, b = std::min(n_pos, a + chunk);
        if (a >= b) break;
        try {
            th.emplace_back([&r, a, b, out, half] { rope_rows(r, a, b, out + (size_t)a * (size_t)half * 2u); });
        } catch (const std::system_error &) {
            break;   // no thread to be had: this thread computes the rest
        }
        handed = b;
    }
    if (handed < n_pos) rope_rows(r, handed, n_pos, out + (size_t)handed * (size_t)half * 2u);
    for (auto &t : th) t.join();
}

}  // namespace

// The decode split's per-launch tables for ap.n_cta CTAs over hkv heads of
// n_kv keys: the score tiles a CTA owns and each head's CTA span.  CTA c
// covers the flattened (head, key) rows [c*T/C, (c+1)*T/C), T = hkv * n_kv.
void kvb::attn_split(AttnParams &ap, int hkv, int64_t n_kv)
{
    const int64_t T = (int64_t)hkv * n_kv, C = ap.n_cta, tk = attn_tile_keys();
    // score tiles of the longest CTA range: ceil(ceil(T/C)/128) + 1 (a range
    // that crosses a head boundary starts a second partial tile)
    ap.S_tiles = ((T + C - 1) / C + tk - 1) / tk + 1;
    auto lo = [&](int64_t cc) { return cc * T / C; };
    auto cta_of = [&](int64_t x) {
        int64_t cc = std::min<int64_t>(C - 1, x * C / T);
        while (cc + 1 < C && lo(cc + 1) <= x) cc++;
        while (cc > 0 && lo(cc) > x) cc--;
        return cc;
    };
    for (int h = 0; h < hkv; h++) {
        const int64_t a = cta_of((int64_t)h * n_kv), b = cta_of((int64_t)(h + 1) * n_kv - 1);
        ap.span_a[h] = (int16_t)a;
        ap.span_b[h] = (int16_t)b;
        ap.span_slot[h] = (int8_t)(lo(a) < (int64_t)h * n_kv ? 1 : 0);
    }
}

int kvb::set_last_error(int code, const char *msg)
{
    snprintf(g_last_error, sizeof(g_last_error), "%s", msg ? msg : "");
    return code;
}

// ---------------------------------------------------------------------------
// the context
// ---------------------------------------------------------------------------
struct Pending {
    bool on = false;
    int layer = -1;
    int64_t n_past = 0;
    int n_new = 0;
    const float *q = nullptr, *k = nullptr, *v = nullptr;
    int64_t q_stride = 0, k_stride = 0, v_stride = 0;
    const float *qn = nullptr, *kn = nullptr;
    const float *qb = nullptr, *kb = nullptr, *vb = nullptr;   // projection biases or null
    cudaStream_t st = nullptr;
};

struct kv_ctx {
    kv_config cfg{};
    std::vector<float> freq_factors;
    int device = 0;
    int sm_count = 148;
    int64_t n_ctx = 0;        // positions (the RoPE table)
    int64_t rows = 0;         // cache rows: n_ctx, or the ring's cells
    int64_t ring = 0;         // ring cells (0: linear cache)
    __half *ring_mask = nullptr;   // ring caches: [n_batch_max][rows] F16 visibility of a chunk
    int D = 0, hq_loc = 0, hkv_loc = 0, r = 1, hq0 = 0, hkv0 = 0;
    float scale = 1.0f;

    __half *cache = nullptr;  // [n_layer][2][rows][hkv_loc][D]
    int64_t layer_elems = 0;  // rows * hkv_loc * D
    float2 *rope = nullptr;   // [n_ctx][n_rot/2]
    __half *qbuf = nullptr;   // [n_batch_max][hq_loc][D]
    float *S = nullptr;       // score scratch, attn_tile_scores() floats per (CTA, tile)
    int64_t S_floats = 0;
    unsigned long long *stats = nullptr;  // [max_cta][2][8][2] epoch-tagged (max, sum) slots
    uint32_t epoch = 0;                   // tag of the last attention launch
    long long *acc = nullptr; // [hkv_loc][8][D] fixed-point output accumulators
    unsigned *ctl = nullptr;  // [2][hkv_loc]: output tickets, non-finite flags; then the peer-exchange ticket
    unsigned *err = nullptr;  // device error word of the bounded waits
    float *local_out = nullptr;   // sharded prefill: [n_batch_max][hq_loc*D]
    // sharded decode over peer memory: this shard's receive buffer [2][n_head*D]
    // F32 + flags [2][n_shards][hkv_loc], and every shard's buffer mapped here
    unsigned long long *rx = nullptr;   // this shard's receive buffer [2][rx_stride] tagged words
    int64_t rx_stride = 0;
    unsigned long long *peer_rx[kvb::kMaxShards] = {};
    bool peers = false;
    float *gathered = nullptr;    // [n_shards][n_batch_max][hq_loc*D]
    int max_cta = 0;
    std::vector<CUtensorMap> kmaps, vmaps;  // per layer: [n_ctx][hkv_loc][D] F16, swizzled column boxes
    uint64_t limit_ns = 1000000000ull;      // bound of every device-side wait (1 s)
    int inject = 0;                         // test hook, applies to the next decode launch
    bool coop = false;                      // attention kernels as cooperative launches
    // sharded decode: the collector loads the peers' heads from their buffers
    // (pull) instead of every shard storing its heads into every peer's
    // buffer (push) -- with two shards, where pull measured ahead (2 B200s,
    // same box: llama-3.2-3B 32k 644.0 -> 624.9 us/token, llama-3.1-8B 128k
    // 1635.3 -> 1622.6); with eight push did (llama-3.2-3B 32k 462.2 -> 423.3:
    // the collector's polls stay local instead of crossing NVLink per peer)
    bool xpull = false;
    int max_clusters[kvb::kMaxClusterCtas + 1] = {};   // q-CTA clusters of the attention kernel held at once
    int force_q = 0;                        // KV_B200_CLUSTER: 0 policy, < 0 none, q > 1 that size
    int min_keys = kDecodeMinKeys;          // KV_B200_MIN_KEYS: fewest keys a decode CTA streams
    int dec_sms = 0;                        // SMs the decode split uses (KV_B200_DECODE_SMS, <= sm_count)
    int l2pf = -1;                          // KV_B200_L2PF: tiles prefetched to L2 at the long stage waits
                                            // (-1: the default rule of l2pf_default)

    Pending pend;  // a deferred single-token kv_append
    // state of the last kv_append (kv_attend must follow it)
    int last_layer = -1;
    int64_t last_n_past = -1;
    int last_n_new = 0;
    // chunked prefill on the tensor cores (head_dim 64/128, chunks of >= 32 query rows)
    bool pf = false;
    int pf_D = 0;                           // the chunk kernel's head_dim (128 for a 96-wide head)
    std::vector<CUtensorMap> pf_kmaps, pf_vmaps;   // head_dim 96: 64-wide boxes, columns 96-127 zero-filled
    // the CTA-pair chunk kernel (head_dim 128): each layer's K with 32-key
    // boxes; empty when the device cannot run its clusters (or
    // KV_B200_PREFILL_PAIR=0)
    std::vector<CUtensorMap> pf2_kmaps;
    int pf_tb = 0;                          // tokens per 128-row query tile
    CUtensorMap qmap{};                     // qbuf [n_batch_max][hq_loc][D], box 64 x r x tb
    float *pf_stat = nullptr;               // [sm_count][kseg][2 tiles][128][2]
    float *pf_out = nullptr;                // [sm_count][kseg][2 tiles][128][D]
    float2 *pf_rstat = nullptr;             // [hkv_loc * blocks][256] (M, 1/Z) of the exact passes
    // the cache row the last fused attention launch appended (stream, layer):
    // the next launch on that stream for that layer must not read it early
    cudaStream_t hz_stream = nullptr;
    int hz_layer = -1;
    int64_t hz_row = -1;

    ncclComm_t comm = nullptr;

    std::atomic<int64_t> launches{0};
#ifdef KV_PHASE_STAMPS
    // measurement builds: phase stamps of the last kStampRing attention launches
    static constexpr int kStampRing = 256;
    unsigned long long *stamps = nullptr;   // [kStampRing][max_cta][kStampSlots]
    int64_t stamp_next = 0;
#endif
    bool prof_on = false;
    struct Rec {
        int k;
        cudaEvent_t a, b;
    };
    std::vector<Rec> recs;
    std::vector<cudaEvent_t> ev_pool;

    __half *k_layer(int l) const { return cache + (int64_t)l * 2 * layer_elems; }
    __half *v_layer(int l) const { return cache + ((int64_t)l * 2 + 1) * layer_elems; }
};

namespace {

constexpr int64_t kMaxPositions = (int64_t)1 << 31;

bool shape_ok(const kv_config *c, std::string &why)
{
    char buf[256];
    if (c->n_layer <= 0 || c->n_head <= 0 || c->n_head_kv <= 0) { why = "n_layer, n_head and n_head_kv must be > 0"; return false; }
    if (c->head_dim != 64 && c->head_dim != 96 && c->head_dim != 128 && c->head_dim != 256) {
        snprintf(buf, sizeof(buf), "head_dim %d unsupported (64, 96, 128, 256)", c->head_dim);
        why = buf;
        return false;
    }
    if (c->n_head % c->n_head_kv != 0) { why = "n_head must be a multiple of n_head_kv"; return false; }
    if (c->n_rot < 0 || c->n_rot > c->head_dim || (c->n_rot & 1)) { why = "n_rot must be even and <= head_dim"; return false; }
    if (c->rope_mode != KV_ROPE_NORMAL && c->rope_mode != KV_ROPE_NEOX) { why = "rope_mode must be 0 (NORMAL) or 2 (NEOX)"; return false; }
    if (c->n_rot > 0 && !(c->rope_base > 0.0f)) { why = "rope_base must be > 0"; return false; }
    if (c->qk_norm < 0 || c->qk_norm > 2) { why = "qk_norm must be 0, 1 (RMSNorm) or 2 (nGPT)"; return false; }
    if ((c->head_dim == 256 || c->qk_norm == 2) && c->n_rot != 0 && c->n_rot != c->head_dim) {
        why = "head_dim 256 and the nGPT norm rotate whole heads (n_rot 0 or head_dim)";
        return false;
    }
    if (c->rope_ext_factor != 0.0f && c->n_ctx_orig <= 0) { why = "YaRN (ext_factor != 0) needs n_ctx_orig > 0"; return false; }
    const int ns = c->n_shards <= 1 ? 1 : c->n_shards;
    if (c->n_head_kv % ns != 0) { why = "n_head_kv must be a multiple of n_shards"; return false; }
    if (c->n_head_kv / ns > kvb::kMaxLocalHeads) { why = "more than 64 KV heads per shard"; return false; }
    if (ns > 1 && (c->shard < 0 || c->shard >= ns)) { why = "shard out of range"; return false; }
    if (c->n_batch_max < 0) { why = "n_batch_max must be >= 0"; return false; }
    if (c->ring_cells < 0) { why = "ring_cells must be >= 0"; return false; }
    if (c->ring_cells > 0 && c->n_ctx <= 0) { why = "a ring cache needs n_ctx (its positions) > 0"; return false; }
    // TMA descriptors address at most 2^32 rows; 2^31 positions already exceed
    // any device's memory at every supported shape, and keep the sizing
    // arithmetic far from overflow
    if (c->n_ctx > kMaxPositions) { why = "n_ctx above 2^31 positions"; return false; }
    return true;
}

uint64_t per_position_bytes(const kv_config *c)
{
    const int ns = c->n_shards <= 1 ? 1 : c->n_shards;
    const uint64_t cache = (uint64_t)c->n_layer * (uint64_t)(c->n_head_kv / ns) * (uint64_t)c->head_dim * 2u * 2u;
    const uint64_t rope = (uint64_t)(c->n_rot / 2) * sizeof(float2);
    return cache + rope;
}

cudaStream_t to_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

int ensure_device(const kv_ctx *ctx)
{
    int cur = -1;
    KV_CUDA(cudaGetDevice(&cur));
    if (cur != ctx->device) KV_CUDA(cudaSetDevice(ctx->device));
    return KV_OK;
}

cudaEvent_t pool_event(kv_ctx *ctx)
{
    if (!ctx->ev_pool.empty()) {
        cudaEvent_t e = ctx->ev_pool.back();
        ctx->ev_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Wraps one kernel launch: counts it and, when profiling, brackets it with events.
template <class F>
int launch(kv_ctx *ctx, int kernel_id, cudaStream_t st, const char *what, F &&fn)
{
    cudaEvent_t a = nullptr, b = nullptr;
    if (ctx->prof_on) {
        a = pool_event(ctx);
        b = pool_event(ctx);
        cudaEventRecord(a, st);
    }
    cudaError_t e = fn();
    if (e != cudaSuccess) return cuda_fail(e, what);
    ctx->launches.fetch_add(1, std::memory_order_relaxed);
    if (ctx->prof_on) {
        cudaEventRecord(b, st);
        try {
            ctx->recs.push_back({kernel_id, a, b});
        } catch (const std::bad_alloc &) {
            return fail(KV_E_OOM, "%s: no host memory for its profiling record", what);
        }
    }
    return KV_OK;
}

// CTAs of the balanced decode split: one per SM, never fewer than the heads
// (so a CTA's key range spans at most two heads), never more than the rows,
// and at least 256 (head, key) rows a CTA: short caches take fewer CTAs, so
// the statistics exchange and the output combine have fewer parties
// (qwen2-0.5B at 2k keys: 12.5 -> 11.6 us a layer; 512 or more rows a CTA is
// slower).
int decode_ctas_for(int sm_count, int hkv_loc, int64_t n_kv, int min_keys = kDecodeMinKeys)
{
    const int64_t T = (int64_t)hkv_loc * n_kv;
    const int64_t mk = std::max(128, min_keys);
    int64_t c = std::min<int64_t>(std::min(sm_count, kvb::attn_max_ctas()), (T + mk - 1) / mk);
    // a multiple of the heads when that idles at most 5 % of the CTAs: every CTA
    // then covers one head, one statistics poll and one output flush instead
    // of two for the CTAs that straddle heads (8 heads: 144 of 148 SMs;
    // llama-3.2-3B 32k 28.7 -> 27.1 us a layer, llama-3.1-8B 128k 91.1 -> 87.6)
    if (c >= hkv_loc) {
        const int64_t a = c / hkv_loc * hkv_loc;
        if (a * 20 >= c * 19) c = a;
    }
    c = std::max<int64_t>(c, hkv_loc);
    c = std::min<int64_t>(c, T);
    return (int)c;
}

// whether a grid of n_cta CTAs is resident at once with blocks_per_sm on each SM
bool decode_grid_fits(int sm_count, int blocks_per_sm, int n_cta)
{
    return sm_count > 0 && blocks_per_sm > 0 && n_cta > 0 && (int64_t)sm_count * blocks_per_sm >= n_cta;
}

// The decode grid: n_cta CTAs in clusters of cq (cq = 1: no clusters), ncl
// clusters per local head.  max_clusters[q] is the number of q-CTA clusters
// the device holds at once (0: not possible); force_q > 0 asks for that
// cluster size (several clusters per head where one does not cover it),
// force_q < 0 for none.
//  * One cluster per head, when the head's keys fit a cluster's CTAs (>= 256
//    keys each) and the grid keeps at least 85 % of the CTAs of the split
//    without clusters: the statistics and the partial outputs never leave the
//    cluster's shared memory (short contexts, many heads; measured on B200:
//    qwen2-0.5B 11.8 -> 10.1 us a layer, phi3-mini 18.4 -> 16.5).
//  * Else no clusters.  Several clusters per head (a cluster-level exchange,
//    then a global one among the clusters) measured slower than the plain
//    split on one-head shards (11.3 -> 14.9 us a layer at 32k: the two levels
//    add their latencies, and clusters of 8 fit only 120 of the 148 SMs), so
//    the policy does not choose it.
struct DecodeShape {
    int n_cta, cq, ncl;
};

DecodeShape decode_shape_for(int sm_count, int hkv_loc, int64_t n_kv, const int *max_clusters, int force_q,
                             int min_keys = kDecodeMinKeys)
{
    const int c0 = decode_ctas_for(sm_count, hkv_loc, n_kv, min_keys);
    DecodeShape none{c0, 1, 1};
    if (!max_clusters || force_q < 0) return none;
    auto fits = [&](int q, int ncl) { return q <= kvb::kMaxClusterCtas && max_clusters[q] >= hkv_loc * ncl; };
    if (force_q > 1) {
        const int q = std::min(force_q, kvb::kMaxClusterCtas);
        const int ncl = std::max(1, c0 / (hkv_loc * q));
        return fits(q, ncl) && (int64_t)hkv_loc * ncl * q <= std::min(sm_count, kvb::attn_max_ctas()) ? DecodeShape{hkv_loc * ncl * q, q, ncl}
                                                                                                   : none;
    }
    const int64_t per_head_keys = (n_kv + 255) / 256;
    const int qa = (int)std::min<int64_t>({(int64_t)kvb::kMaxClusterCtas, sm_count / hkv_loc, per_head_keys});
    if (qa >= 2 && (int64_t)hkv_loc * qa * 100 >= (int64_t)c0 * 85 && fits(qa, 1)) return DecodeShape{hkv_loc * qa, qa, 1};
    return none;
}

// The decode kernel's L2 prefetch (AttnParams::l2pf) by the tiles a CTA
// streams: while the producer waits behind the previous kernel's tail for
// its first free stage, the next 2 tiles (ranges of 8-31 K tiles) or 4 (32 or
// more) go to L2, so HBM keeps streaming.  Measured on one B200: llama-3.2-3B
// at 32k (14 tiles a CTA) 74.1 -> 75.0 % of the HBM roofline with 2 (4: no
// gain), llama-3.1-8B at 128k (56 tiles) 94.1 -> 96.5 % with 4 (8: 96.0 %);
// prefetching behind the statistics exchange as well lost at 32k (the poll's
// loads queue behind the prefetch traffic), so only the first wait does it.
int l2pf_default(int hkv_loc, int64_t n_kv, int n_cta)
{
    const int64_t tiles = ((int64_t)hkv_loc * n_kv / std::max(1, n_cta) + 127) / 128;
    const int n = tiles >= 32 ? 4 : tiles >= 8 ? 2 : 0;
    return n ? (n | 0x100) : 0;
}

}  // namespace

int kvb::attn_plain_ctas(int sm_count, int hkv, int64_t n_kv)
{
    return decode_ctas_for(sm_count, hkv, n_kv);
}

namespace {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

int encode_map(CUtensorMap *m, CUtensorMapDataType dt, int rank, void *base, const cuuint64_t *dims,
               const cuuint64_t *strides, const cuuint32_t *box, CUtensorMapSwizzle swizzle)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(KV_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = fn(m, dt, (cuuint32_t)rank, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(KV_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return KV_OK;
}

}  // namespace

// One layer's K or V cache [rows][hkv][D] F16 as the attention kernel's
// tensor map: boxes of one head x 128 keys x a 64-wide column block with
// 128-byte swizzle (32 wide, 64-byte swizzle at head_dim 96).
int kvb::encode_cache_map(CUtensorMap *m, const void *base, int64_t rows, int hkv, int D)
{
    const int bw = attn_box_width(D);
    const CUtensorMapSwizzle sw = bw == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)hkv, (cuuint64_t)rows};
    const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)hkv * D * 2};
    const cuuint32_t box[3] = {(cuuint32_t)bw, 1, (cuuint32_t)attn_tile_keys()};
    return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box, sw);
}

namespace {

void unmap_peers(kv_ctx *ctx);

void free_all(kv_ctx *ctx)
{
    for (auto &r : ctx->recs) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    for (auto e : ctx->ev_pool) cudaEventDestroy(e);
    ctx->recs.clear();
    ctx->ev_pool.clear();
    if (ctx->cfg.n_shards > 1 && ctx->comm) {
        // no shard may still write into a buffer about to be unmapped: all
        // shards reach this point with their work complete
        cudaDeviceSynchronize();
        int *d = nullptr;
        if (cudaMalloc(&d, sizeof(int) * ctx->cfg.n_shards) == cudaSuccess) {
            nccl().AllGather(d + ctx->cfg.shard, d, 1, 2, ctx->comm, nullptr);
            cudaDeviceSynchronize();
            cudaFree(d);
        }
    }
    unmap_peers(ctx);
    if (ctx->comm && nccl().CommDestroy) nccl().CommDestroy(ctx->comm);
    ctx->comm = nullptr;
    void *ptrs[] = {ctx->cache, ctx->rope, ctx->qbuf, ctx->S, ctx->stats, ctx->acc, ctx->ctl, ctx->err,
                    ctx->local_out, ctx->gathered, ctx->pf_stat, ctx->pf_out, ctx->pf_rstat, ctx->ring_mask};
    for (void *p : ptrs)
        if (p) cudaFree(p);
#ifdef KV_PHASE_STAMPS
    if (ctx->stamps) cudaFree(ctx->stamps);
#endif
}


// Sharded decode exchanges head outputs over NVLink instead of an NCCL
// all-gather: each shard allocates a receive buffer, its CUDA IPC handle goes to
// every shard (one ncclAllGather at kv_alloc) and each shard maps the others'.
// Returns KV_OK and leaves ctx->peers false (NCCL path) when the mapping is not
// possible; an error code only for a failed collective.
int map_peers(kv_ctx *ctx)
{
    const kv_config &c = ctx->cfg;
    const int G = c.n_shards;
    if (G > kvb::kMaxShards) return KV_OK;
    ctx->rx_stride = (int64_t)c.n_head * ctx->D;
    const size_t bytes = (size_t)2 * ctx->rx_stride * sizeof(unsigned long long);
    if (cudaMalloc(&ctx->rx, bytes) != cudaSuccess || cudaMemset(ctx->rx, 0, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(KV_E_OOM, "peer receive buffer");
    }
    cudaIpcMemHandle_t mine;
    const bool have = cudaIpcGetMemHandle(&mine, ctx->rx) == cudaSuccess;
    if (!have) cudaGetLastError();
    // every shard's handle (a zeroed handle marks a shard without one)
    std::vector<unsigned char> all((size_t)G * sizeof(cudaIpcMemHandle_t), 0);
    unsigned char *dev = nullptr;
    if (cudaMalloc(&dev, all.size()) != cudaSuccess) return fail(KV_E_OOM, "handle exchange buffer");
    cudaMemset(dev, 0, all.size());
    if (have)
        cudaMemcpy(dev + (size_t)c.shard * sizeof(mine), &mine, sizeof(mine), cudaMemcpyHostToDevice);
    const int nr = nccl().AllGather(dev + (size_t)c.shard * sizeof(mine), dev, sizeof(mine), 1 /* uint8 */,
                                    ctx->comm, nullptr);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), dev, all.size(), cudaMemcpyDeviceToHost);
    cudaFree(dev);
    if (nr != 0 || e != cudaSuccess) return fail(KV_E_COMM, "IPC handle exchange failed");
    bool ok = true;
    for (int g = 0; g < G && ok; g++) {
        if (g == c.shard) {
            ctx->peer_rx[g] = ctx->rx;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, all.data() + (size_t)g * sizeof(h), sizeof(h));
        bool zero = true;
        for (size_t i = 0; i < sizeof(h); i++) zero = zero && ((unsigned char *)&h)[i] == 0;
        void *p = nullptr;
        if (zero || cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
        } else {
            ctx->peer_rx[g] = static_cast<unsigned long long *>(p);
        }
    }
    // every shard must agree: one that could not map its peers uses NCCL, so all do
    int flag = ok ? 1 : 0;
    int *dflag = nullptr;
    std::vector<int> flags(G, 0);
    if (cudaMalloc(&dflag, G * sizeof(int)) == cudaSuccess) {
        cudaMemcpy(dflag + c.shard, &flag, sizeof(int), cudaMemcpyHostToDevice);
        if (nccl().AllGather(dflag + c.shard, dflag, 1, 2 /* int32 */, ctx->comm, nullptr) == 0 &&
            cudaDeviceSynchronize() == cudaSuccess)
            cudaMemcpy(flags.data(), dflag, G * sizeof(int), cudaMemcpyDeviceToHost);
        cudaFree(dflag);
    }
    ctx->peers = true;
    for (int g = 0; g < G; g++) ctx->peers = ctx->peers && flags[g] == 1;
    // KV_B200_EXCHANGE: "pull" (the collector loads the peers' heads from
    // their buffers; the default with two shards), "push" (every shard stores
    // its heads into every peer's buffer; the default with more), "nccl" (the
    // NCCL all-gather after the kernel, for decode too)
    const char *env = getenv("KV_B200_EXCHANGE");
    ctx->xpull = G == 2;
    if (env && strcmp(env, "nccl") == 0) ctx->peers = false;
    if (env && strcmp(env, "pull") == 0) ctx->xpull = true;
    if (env && strcmp(env, "push") == 0) ctx->xpull = false;
    return KV_OK;
}

void unmap_peers(kv_ctx *ctx)
{
    for (int g = 0; g < kvb::kMaxShards; g++)
        if (ctx->peer_rx[g] && ctx->peer_rx[g] != ctx->rx) cudaIpcCloseMemHandle(ctx->peer_rx[g]);
    if (ctx->rx) cudaFree(ctx->rx);
    ctx->rx = nullptr;
}

// The single-token append a kv_append deferred to the following kv_attend.
int run_append(kv_ctx *ctx, const Pending &pd)
{
    const kv_config &c = ctx->cfg;
    kvb::AppendParams p;
    p.q = pd.q; p.k = pd.k; p.v = pd.v;
    p.q_stride = pd.q_stride; p.k_stride = pd.k_stride; p.v_stride = pd.v_stride;
    p.q_norm_w = pd.qn; p.k_norm_w = pd.kn;
    p.q_bias = pd.qb; p.k_bias = pd.kb; p.v_bias = pd.vb;
    p.n_new = pd.n_new; p.n_past = pd.n_past;
    p.hq_loc = ctx->hq_loc; p.hkv_loc = ctx->hkv_loc; p.hq0 = ctx->hq0; p.hkv0 = ctx->hkv0;
    p.n_rot = c.n_rot; p.rope_mode = c.rope_mode; p.qk_norm = c.qk_norm;
    // nGPT's L2 norm is rms_norm(x, 1e-6 / D) * (1 / sqrt(D)) (dory.c:577-580)
    p.eps = c.qk_norm == 2 ? c.rms_eps / (float)ctx->D : c.rms_eps;
    p.post = 1.0f / sqrtf((float)ctx->D);
    p.rope = ctx->rope;
    p.kc = ctx->k_layer(pd.layer); p.vc = ctx->v_layer(pd.layer);
    p.ring = ctx->ring;
    p.qbuf = ctx->qbuf;
    auto al16 = [](const void *x) { return ((uintptr_t)x & 15u) == 0; };
    const bool vec = al16(pd.q) && al16(pd.k) && al16(pd.v) && al16(pd.qn) && al16(pd.kn) &&
                     (pd.n_new == 1 || ((pd.q_stride | pd.k_stride | pd.v_stride) & 3) == 0);
    return launch(ctx, KV_K_APPEND, pd.st, "append kernel", [&] { return kvb::launch_append(ctx->D, vec, p, pd.st); });
}

int flush_pending(kv_ctx *ctx)
{
    if (!ctx->pend.on) return KV_OK;
    ctx->pend.on = false;
    return run_append(ctx, ctx->pend);
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int kv_config_init(kv_config *cfg)
{
    if (!cfg) return fail(KV_E_ARG, "cfg is NULL");
    std::memset(cfg, 0, sizeof(*cfg));
    cfg->rope_mode = KV_ROPE_NEOX;
    cfg->rope_base = 10000.0f;
    cfg->rope_freq_scale = 1.0f;
    cfg->rope_attn_factor = 1.0f;
    cfg->rms_eps = 1e-6f;
    cfg->n_batch_max = 512;
    cfg->device = -1;
    cfg->n_shards = 1;
    return KV_OK;
}

uint64_t kv_cache_bytes(const kv_config *cfg, int64_t n_ctx)
{
    if (!cfg || n_ctx < 0) return 0;
    const uint64_t per_token = (uint64_t)cfg->n_layer * (uint64_t)cfg->head_dim * (uint64_t)cfg->n_head_kv * 2u * 2u;
    // a ring holds min(ring_cells, n_ctx) rows whatever the positions (dory_kv_cost, dory.c:373-389)
    const int64_t rows = cfg->ring_cells > 0 ? std::min<int64_t>(cfg->ring_cells, n_ctx) : n_ctx;
    if (per_token > 0 && (uint64_t)rows > UINT64_MAX / per_token) return UINT64_MAX;   // saturate
    return per_token * (uint64_t)rows;
}

int64_t kv_auto_n_ctx(const kv_config *cfg, int64_t free_bytes)
{
    if (!cfg) return 0;
    if (free_bytes <= 0) return 4096;  // N_CTX_DEFAULT (model.h:43)
    const uint64_t reserve = (uint64_t)384 << 20;
    uint64_t budget = (uint64_t)free_bytes;
    budget -= std::min(budget, reserve);
    budget = (uint64_t)((double)budget * 0.8);
    const uint64_t per_tok = per_position_bytes(cfg);
    const int64_t raw = per_tok > 0 ? (int64_t)(budget / per_tok) : 4096;
    int64_t n_ctx = (raw / 64) * 64;
    int64_t limit = cfg->n_ctx_train > 0 ? cfg->n_ctx_train : 262144;
    if (cfg->longrope_clamp && cfg->n_ctx_orig > 0) limit = std::min<int64_t>(limit, cfg->n_ctx_orig);
    if (n_ctx > limit) n_ctx = limit;
    if (n_ctx < 512) n_ctx = std::min<int64_t>(512, limit);
    return n_ctx;
}

static int alloc_impl(const kv_config *cfg_in, kv_ctx **out)
{
    std::string why;
    if (!shape_ok(cfg_in, why)) return fail(KV_E_ARG, "kv_alloc: %s", why.c_str());

    // every early return, and an exception, frees what was set up so far
    struct Owner {
        kv_ctx *p;
        ~Owner()
        {
            if (p) {
                free_all(p);
                delete p;
            }
        }
    } own{new kv_ctx()};
    kv_ctx *ctx = own.p;
    ctx->cfg = *cfg_in;
    kv_config &c = ctx->cfg;
    if (c.n_shards <= 1) { c.n_shards = 1; c.shard = 0; }
    if (c.n_batch_max == 0) c.n_batch_max = 512;
    if (c.rope_freq_factors && c.n_rot > 0) {
        ctx->freq_factors.assign(c.rope_freq_factors, c.rope_freq_factors + c.n_rot / 2);
        c.rope_freq_factors = ctx->freq_factors.data();
    } else {
        c.rope_freq_factors = nullptr;
    }
    c.comm_id = nullptr;

    auto bail = [](int code) { return code; };
    cudaError_t e;
    if (c.device >= 0) {
        e = cudaSetDevice(c.device);
        if (e != cudaSuccess) return bail(cuda_fail(e, "cudaSetDevice"));
    }
    e = cudaGetDevice(&ctx->device);
    if (e != cudaSuccess) return bail(cuda_fail(e, "cudaGetDevice"));
    e = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, ctx->device);
    if (e != cudaSuccess) return bail(cuda_fail(e, "cudaDeviceGetAttribute"));

    ctx->D = c.head_dim;
    ctx->hkv_loc = c.n_head_kv / c.n_shards;
    ctx->r = c.n_head / c.n_head_kv;
    ctx->hq_loc = ctx->hkv_loc * ctx->r;
    ctx->hkv0 = c.shard * ctx->hkv_loc;
    ctx->hq0 = c.shard * ctx->hq_loc;
    if (ctx->hkv_loc > ctx->sm_count)   // the attention kernel keeps one CTA per SM, all resident
        return bail(fail(KV_E_UNSUPPORTED, "%d local KV heads exceed the device's %d SMs", ctx->hkv_loc,
                         ctx->sm_count));
    ctx->scale = 1.0f / sqrtf((float)ctx->D);

    if (c.n_ctx <= 0) {
        size_t fr = 0, tot = 0;
        e = cudaMemGetInfo(&fr, &tot);
        ctx->n_ctx = std::min(kv_auto_n_ctx(&c, e == cudaSuccess ? (int64_t)fr : -1), kMaxPositions);
        fprintf(stderr,
                "n_ctx=auto: free HBM %.0f MiB, reserve 384 MiB, %.1f KiB per position -> n_ctx=%lld\n",
                (double)fr / (1024.0 * 1024.0), (double)per_position_bytes(&c) / 1024.0, (long long)ctx->n_ctx);
    } else {
        ctx->n_ctx = c.n_ctx;
    }
    c.n_ctx = ctx->n_ctx;
    ctx->ring = c.ring_cells > 0 ? std::min<int64_t>(c.ring_cells, ctx->n_ctx) : 0;
    ctx->rows = ctx->ring ? ctx->ring : ctx->n_ctx;
    c.ring_cells = ctx->ring;
    if (c.n_batch_max > ctx->rows) c.n_batch_max = (int32_t)ctx->rows;

    const int64_t D = ctx->D;
    ctx->layer_elems = ctx->rows * ctx->hkv_loc * D;   // <= 2^31 x 64 x 256
    if ((double)c.n_layer * 4.0 * (double)ctx->layer_elems > 0x1p60)   // beyond any device, and near size_t's range
        return bail(fail(KV_E_OOM, "a cache of %lld rows x %d layers is beyond any device's memory",
                         (long long)ctx->rows, c.n_layer));
    const size_t cache_bytes = (size_t)c.n_layer * 2u * (size_t)ctx->layer_elems * sizeof(__half);
    e = cudaMalloc(&ctx->cache, cache_bytes);
    if (e != cudaSuccess) {
        return bail(fail(KV_E_OOM, "failed to allocate KV cache (%lld rows x %d layers, %.0f MiB requested): %s",
                         (long long)ctx->rows, c.n_layer, (double)cache_bytes / (1024.0 * 1024.0),
                         cudaGetErrorString(e)));
    }
    cudaGetLastError();

    const int half = c.n_rot / 2;
    if (half > 0) {
        std::vector<float> table((size_t)ctx->n_ctx * (size_t)half * 2u);
        RopeSpec rs{c.n_rot, c.rope_base, c.rope_freq_scale, c.rope_attn_factor, c.rope_ext_factor,
                    c.rope_beta_fast, c.rope_beta_slow, c.n_ctx_orig, c.rope_freq_factors};
        build_rope_table(rs, ctx->n_ctx, table.data());
        e = cudaMalloc(&ctx->rope, table.size() * sizeof(float));
        if (e != cudaSuccess) return bail(fail(KV_E_OOM, "RoPE table allocation: %s", cudaGetErrorString(e)));
        e = cudaMemcpy(ctx->rope, table.data(), table.size() * sizeof(float), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return bail(cuda_fail(e, "RoPE table upload"));
    }

    // score scratch: CTA c of a launch owns S_tiles(n_kv) tiles from
    // c*S_tiles on; C*S_tiles <= T/128 + 3C for T = hkv_loc*n_kv rows
    ctx->max_cta = std::max(std::min(ctx->sm_count, kvb::attn_max_ctas()), ctx->hkv_loc);
    ctx->S_floats = ((int64_t)ctx->hkv_loc * ctx->rows / kvb::attn_tile_keys() + 3 * (int64_t)ctx->max_cta + 1) *
                    kvb::attn_tile_scores();
    const size_t n_part = (size_t)ctx->max_cta * 2u * 8u;
    struct { void **p; size_t bytes; } allocs[] = {
        {(void **)&ctx->qbuf, (size_t)c.n_batch_max * ctx->hq_loc * D * sizeof(__half)},
        {(void **)&ctx->S, (size_t)ctx->S_floats * sizeof(float)},
        {(void **)&ctx->stats, n_part * 2u * sizeof(unsigned long long)},
        {(void **)&ctx->acc, (size_t)ctx->hkv_loc * 8u * (size_t)D * sizeof(long long)},
        {(void **)&ctx->ctl, (2u * (size_t)ctx->hkv_loc + 1u) * sizeof(unsigned)},
        {(void **)&ctx->err, sizeof(unsigned)},
        {(void **)&ctx->ring_mask, ctx->ring ? (size_t)c.n_batch_max * (size_t)ctx->rows * sizeof(__half) : 0},
    };
    for (auto &a : allocs) {
        if (a.bytes == 0) continue;
        e = cudaMalloc(a.p, a.bytes);
        if (e != cudaSuccess) return bail(fail(KV_E_OOM, "scratch allocation (%zu bytes): %s", a.bytes, cudaGetErrorString(e)));
    }
    e = cudaMemset(ctx->ctl, 0, (2u * (size_t)ctx->hkv_loc + 1u) * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(ctx->stats, 0, n_part * 2u * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(ctx->acc, 0, (size_t)ctx->hkv_loc * 8u * (size_t)D * sizeof(long long));
    if (e == cudaSuccess) e = cudaMemset(ctx->err, 0, sizeof(unsigned));
    if (e != cudaSuccess) return bail(cuda_fail(e, "cudaMemset"));
    e = kvb::attn_prepare(ctx->D);
    if (e != cudaSuccess) return bail(cuda_fail(e, "attn_prepare"));
    {
        // the attention kernel's CTAs wait on one another: its largest grid
        // must be resident at once on this device
        int bps = 0;
        e = kvb::attn_occupancy(ctx->D, &bps);
        if (e != cudaSuccess) return bail(cuda_fail(e, "attention kernel occupancy"));
        if (!decode_grid_fits(ctx->sm_count, bps, ctx->max_cta))
            return bail(fail(KV_E_UNSUPPORTED,
                             "the attention kernel's %d CTAs cannot be resident at once (%d SMs x %d CTAs an SM)",
                             ctx->max_cta, ctx->sm_count, bps));
        const char *cv = getenv("KV_B200_COOPERATIVE");
        ctx->coop = cv && cv[0] == '1';
        for (int q = 2; q <= kvb::kMaxClusterCtas; q++) {
            e = kvb::attn_cluster_occupancy(ctx->D, q, &ctx->max_clusters[q]);
            if (e != cudaSuccess) {   // no cluster mode on this device
                cudaGetLastError();
                ctx->max_clusters[q] = 0;
            }
        }
        ctx->dec_sms = ctx->sm_count;
        const char *ds = getenv("KV_B200_DECODE_SMS");
        if (ds && *ds) ctx->dec_sms = std::max(1, std::min(ctx->sm_count, atoi(ds)));
        const char *mk = getenv("KV_B200_MIN_KEYS");
        if (mk && *mk) ctx->min_keys = std::max(128, std::min(1 << 20, atoi(mk)));
        const char *cl = getenv("KV_B200_CLUSTER");
        if (cl && *cl) ctx->force_q = atoi(cl) <= 1 ? -1 : atoi(cl);
        const char *pf = getenv("KV_B200_L2PF");
        if (pf && *pf) {
            ctx->l2pf = std::max(0, std::min(16, atoi(pf)));
            const char *at = getenv("KV_B200_L2PF_AT");   // entry, exchange or both (default)
            const bool entry = !at || strcmp(at, "exchange") != 0, exch = !at || strcmp(at, "entry") != 0;
            ctx->l2pf |= (entry ? 0x100 : 0) | (exch ? 0x200 : 0);
        }
    }
#ifdef KV_PHASE_STAMPS
    {
        const size_t sb = (size_t)kv_ctx::kStampRing * ctx->max_cta * kvb::kStampSlots * sizeof(unsigned long long);
        e = cudaMalloc(&ctx->stamps, sb);
        if (e == cudaSuccess) e = cudaMemset(ctx->stamps, 0, sb);
        if (e != cudaSuccess) return bail(fail(KV_E_OOM, "stamp buffer"));
    }
#endif

    // TMA descriptors: each layer's K and V as [n_ctx][hkv_loc][D] F16, box =
    // one head x 128 keys x a 64-wide column block with 128-byte swizzle (32
    // wide, 64-byte swizzle at head_dim 96)
    ctx->kmaps.resize(c.n_layer);
    ctx->vmaps.resize(c.n_layer);
    for (int l = 0; l < c.n_layer; l++) {
        int rc = kvb::encode_cache_map(&ctx->kmaps[l], ctx->k_layer(l), ctx->rows, ctx->hkv_loc, ctx->D);
        if (rc == KV_OK) rc = kvb::encode_cache_map(&ctx->vmaps[l], ctx->v_layer(l), ctx->rows, ctx->hkv_loc, ctx->D);
        if (rc != KV_OK) return bail(rc);
    }

    // chunked prefill: the tensor-core path, when chunks can hold 32+ query rows
    // (head_dim 96 runs the 128 kernel: its 64-wide boxes read columns 96-127
    // past the row's end, which TMA fills with zeros)
    const int pfD = kvb::prefill_kernel_dim(ctx->D);
    if (kvb::prefill_supported(pfD) && ctx->r <= 128 && (int64_t)c.n_batch_max * ctx->r >= 32) {
        ctx->pf_D = pfD;
        ctx->pf_tb = std::min(128 / ctx->r, (int)c.n_batch_max);   // the Q box's tokens
        const cuuint64_t qdims[3] = {(cuuint64_t)D, (cuuint64_t)ctx->hq_loc, (cuuint64_t)c.n_batch_max};
        const cuuint64_t qstr[2] = {(cuuint64_t)D * 2, (cuuint64_t)ctx->hq_loc * D * 2};
        const cuuint32_t qbox[3] = {64, (cuuint32_t)ctx->r, (cuuint32_t)ctx->pf_tb};
        int rc = encode_map(&ctx->qmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, ctx->qbuf, qdims, qstr, qbox,
                            CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc != KV_OK) return bail(rc);
        const int kseg = kvb::prefill_max_segments();
        const size_t slots = (size_t)ctx->sm_count * kseg * 256u;   // segments x two 128-row tiles
        e = cudaMalloc(&ctx->pf_stat, slots * 2u * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&ctx->pf_out, slots * (size_t)pfD * sizeof(float));
        const int ntile = kvb::prefill_tiles(pfD);
        const size_t nblk = (size_t)(c.n_batch_max + ntile * ctx->pf_tb - 1) / (ntile * ctx->pf_tb);
        if (e == cudaSuccess) e = cudaMalloc(&ctx->pf_rstat, (size_t)ctx->hkv_loc * nblk * 256u * sizeof(float2));
        if (e != cudaSuccess) return bail(fail(KV_E_OOM, "prefill scratch: %s", cudaGetErrorString(e)));
        e = kvb::prefill_prepare(pfD);
        if (e != cudaSuccess) return bail(cuda_fail(e, "prefill_prepare"));
        if (pfD != ctx->D) {
            ctx->pf_kmaps.resize(c.n_layer);
            ctx->pf_vmaps.resize(c.n_layer);
            const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)ctx->hkv_loc, (cuuint64_t)ctx->rows};
            const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)ctx->hkv_loc * D * 2};
            const cuuint32_t box[3] = {64, 1, (cuuint32_t)kvb::attn_tile_keys()};
            for (int l = 0; l < c.n_layer; l++) {
                int rc2 = encode_map(&ctx->pf_kmaps[l], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, ctx->k_layer(l), dims,
                                     strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
                if (rc2 == KV_OK)
                    rc2 = encode_map(&ctx->pf_vmaps[l], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, ctx->v_layer(l), dims,
                                     strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
                if (rc2 != KV_OK) return bail(rc2);
            }
        }
        if (pfD == 128 && ctx->D == 128) {
            const char *pe = getenv("KV_B200_PREFILL_PAIR");
            int clusters = 0;
            e = (pe && pe[0] == '0') ? cudaSuccess : kvb::prefill_pair_prepare(&clusters);
            if (e != cudaSuccess) {   // no pair kernel on this device: the one-CTA kernel runs
                cudaGetLastError();
                clusters = 0;
            }
            if (clusters > 0) {
                ctx->pf2_kmaps.resize(c.n_layer);
                const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)ctx->hkv_loc, (cuuint64_t)ctx->rows};
                const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)ctx->hkv_loc * D * 2};
                const cuuint32_t box[3] = {64, 1, 32};
                for (int l = 0; l < c.n_layer; l++) {
                    const int rc2 = encode_map(&ctx->pf2_kmaps[l], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, ctx->k_layer(l),
                                               dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
                    if (rc2 != KV_OK) return bail(rc2);
                }
            }
        }
        ctx->pf = true;
    }

    if (c.n_shards > 1) {
        if (!cfg_in->comm_id) return bail(fail(KV_E_ARG, "n_shards > 1 needs comm_id"));
        NcclApi &api = nccl();
        if (!api.GetUniqueId) return bail(fail(KV_E_UNSUPPORTED, "libnccl.so.2 could not be loaded"));
        const size_t cols = (size_t)ctx->hq_loc * D;
        e = cudaMalloc(&ctx->local_out, (size_t)c.n_batch_max * cols * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&ctx->gathered, (size_t)c.n_shards * c.n_batch_max * cols * sizeof(float));
        if (e != cudaSuccess) return bail(fail(KV_E_OOM, "gather buffers: %s", cudaGetErrorString(e)));
        NcclId id;
        std::memcpy(id.internal, cfg_in->comm_id, sizeof(id.internal));
        const int rc = api.CommInitRank(&ctx->comm, c.n_shards, id, c.shard);
        if (rc != 0) {
            ctx->comm = nullptr;
            return bail(fail(KV_E_COMM, "ncclCommInitRank: %s", api.GetErrorString ? api.GetErrorString(rc) : "error"));
        }
        const int prc = map_peers(ctx);
        if (prc) return bail(prc);
    }
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return bail(cuda_fail(e, "kv_alloc sync"));
    own.p = nullptr;
    *out = ctx;
    return KV_OK;
}

int kv_alloc(const kv_config *cfg_in, kv_ctx **out)
{
    if (!cfg_in || !out) return fail(KV_E_ARG, "NULL argument");
    *out = nullptr;
    return guarded("kv_alloc", [&] { return alloc_impl(cfg_in, out); });
}

int kv_free(kv_ctx *ctx)
{
    if (!ctx) return KV_OK;
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != ctx->device) cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    const int dev = ctx->device;
    free_all(ctx);
    delete ctx;
    if (cur >= 0 && cur != dev) cudaSetDevice(cur);
    return KV_OK;
}

int kv_n_ctx(const kv_ctx *ctx, int64_t *n_ctx)
{
    if (!ctx || !n_ctx) return fail(KV_E_ARG, "NULL argument");
    *n_ctx = ctx->n_ctx;
    return KV_OK;
}

int kv_shard_info(const kv_ctx *ctx, int32_t *q_head0, int32_t *n_q_heads, int32_t *kv_head0, int32_t *n_kv_heads)
{
    if (!ctx) return fail(KV_E_ARG, "NULL context");
    if (q_head0) *q_head0 = ctx->hq0;
    if (n_q_heads) *n_q_heads = ctx->hq_loc;
    if (kv_head0) *kv_head0 = ctx->hkv0;
    if (n_kv_heads) *n_kv_heads = ctx->hkv_loc;
    return KV_OK;
}

int kv_append(kv_ctx *ctx, int32_t layer, int64_t n_past, int32_t n_new,
              const float *q, int64_t q_stride, const float *k, int64_t k_stride,
              const float *v, int64_t v_stride, const float *q_norm_w, const float *k_norm_w,
              void *stream)
{
    return kv_append_bias(ctx, layer, n_past, n_new, q, q_stride, k, k_stride, v, v_stride, q_norm_w, k_norm_w,
                          nullptr, nullptr, nullptr, stream);
}

int kv_append_bias(kv_ctx *ctx, int32_t layer, int64_t n_past, int32_t n_new,
                   const float *q, int64_t q_stride, const float *k, int64_t k_stride,
                   const float *v, int64_t v_stride, const float *q_norm_w, const float *k_norm_w,
                   const float *q_bias, const float *k_bias, const float *v_bias, void *stream)
{
    if (!ctx) return fail(KV_E_ARG, "NULL context");
    const kv_config &c = ctx->cfg;
    if (layer < 0 || layer >= c.n_layer) return fail(KV_E_ARG, "layer %d out of range", layer);
    if (n_new <= 0 || n_past < 0) return fail(KV_E_ARG, "n_new must be > 0 and n_past >= 0");
    if (n_new > c.n_batch_max) return fail(KV_E_RANGE, "n_new %d exceeds n_batch_max %d", n_new, c.n_batch_max);
    if (n_past > ctx->n_ctx - n_new)   // (n_past + n_new could overflow)
        return fail(KV_E_RANGE, "positions [%lld, %lld) exceed n_ctx %lld", (long long)n_past,
                    (long long)(n_past + n_new), (long long)ctx->n_ctx);
    if (ctx->ring && n_new > ctx->ring)   // a batch longer than the ring would overwrite its own rows
        return fail(KV_E_RANGE, "n_new %d exceeds the ring's %lld cells", n_new, (long long)ctx->ring);
    if (!q || !k || !v) return fail(KV_E_ARG, "q, k and v are required");
    const int64_t D = ctx->D;
    if (n_new > 1 && (q_stride < c.n_head * D || k_stride < c.n_head_kv * D || v_stride < c.n_head_kv * D))
        return fail(KV_E_ARG, "row strides shorter than a token's heads");
    if (c.qk_norm == 1 && (!q_norm_w || !k_norm_w)) return fail(KV_E_ARG, "qk_norm needs q_norm_w and k_norm_w");
    if (c.qk_norm == 2 && !q_norm_w) return fail(KV_E_ARG, "the nGPT norm needs q_norm_w (Q's per-channel scale)");
    int rc = ensure_device(ctx);
    if (rc) return rc;
    rc = flush_pending(ctx);
    if (rc) return rc;

    Pending pd;
    pd.on = true;
    pd.layer = layer;
    pd.n_past = n_past;
    pd.n_new = n_new;
    pd.q = q; pd.k = k; pd.v = v;
    pd.q_stride = q_stride; pd.k_stride = k_stride; pd.v_stride = v_stride;
    pd.qn = q_norm_w; pd.kn = k_norm_w;
    pd.qb = q_bias; pd.kb = k_bias; pd.vb = v_bias;
    pd.st = to_stream(stream);
    ctx->last_layer = layer;
    ctx->last_n_past = n_past;
    ctx->last_n_new = n_new;
    if (n_new == 1 && ctx->r <= kvb::attn_rows() && !ctx->ring && c.qk_norm != 2) {
        // one token: the attention kernels do the append themselves (same bits);
        // any other call on this context first performs it with the append kernel
        ctx->pend = pd;
        return KV_OK;
    }
    return run_append(ctx, pd);
}

namespace {

// Chunks whose keys go beyond this take the exact two passes: the one-pass
// kernel rounds unnormalised weights to F16 while ggml rounds the normalised
// ones, which at long context fall in F16's subnormal range -- measured on
// the oracle, rel-L2 3e-4 at 16k keys, 7e-4 at 64k, 1.3e-3 at 131k (the
// tolerance is 1e-3).
constexpr int64_t kOnePassKeys = 32768;

// Chunked-prefill attention on the tensor cores: the one-pass attention kernel,
// then the fold of pairs split over CTAs; past kOnePassKeys keys the exact
// passes instead (statistics kernel, statistics fold, output kernel, fold)
// (kv_prefill.cu).  A pair is (KV head,
// block of two 128-row query tiles); the pairs' key tiles, laid end to end, are
// cut into C equal ranges; C is the SM count, lowered until no range holds more
// than prefill_max_segments() pairs.  The one pass at head_dim 128 runs on CTA
// pairs (2-CTA clusters, tcgen05 cta_group::2): a block holds four tiles and a
// range goes to a CTA pair, C at most half the SM count.
// the caller's mask of kv_attend_mask (ptr nullptr: the implicit causal mask)
struct MaskArg {
    const void *ptr = nullptr;
    int64_t stride = 0;
    bool f16 = false;
    bool flash = false;
};

int prefill(kv_ctx *ctx, const CUtensorMap &km, const CUtensorMap &vm, const CUtensorMap *km32, int64_t n_past,
            int32_t n_new, float *dst, int64_t dst_stride, int dst_head0, const MaskArg &mk, cudaStream_t st)
{
    kvb::PrefillParams pp{};
    // the exact two passes reproduce the default branch's rounding at long
    // contexts; the flash-attn branch is one online softmax at any length
    pp.mode = !mk.flash && n_past + n_new > kOnePassKeys ? 2 : 0;
    // the one pass runs on CTA pairs where the layer has that kernel's K map
    const bool cta2 = km32 && pp.mode == 0;
    pp.hkv = ctx->hkv_loc;
    pp.r = ctx->r;
    pp.hq_loc = ctx->hq_loc;
    pp.D = ctx->D;
    pp.n_past = n_past;
    pp.n_new = n_new;
    pp.tb = ctx->pf_tb;
    pp.nt = cta2 ? 4 : kvb::prefill_tiles(ctx->pf_D);
    pp.dv = ctx->D;
    pp.nblk = (n_new + pp.nt * pp.tb - 1) / (pp.nt * pp.tb);
    std::vector<int64_t> nt(pp.nblk);
    pp.s_all = 0;
    for (int b = 0; b < pp.nblk; b++) {
        nt[b] = (n_past + (mk.ptr ? (int64_t)n_new : std::min<int64_t>(n_new, (int64_t)(pp.nt * (b + 1)) * pp.tb)) +
                 127) / 128;
        pp.s_all += nt[b];
    }
    const int64_t W = (int64_t)pp.hkv * pp.s_all;
    const int kseg = kvb::prefill_max_segments();
    // the pairs' starts, to count the segments of each range
    std::vector<int64_t> start((size_t)pp.hkv * pp.nblk + 1, 0);
    for (int pr = 0; pr < pp.hkv * pp.nblk; pr++) start[pr + 1] = start[pr] + nt[pr % pp.nblk];
    // work ranges: one a CTA, or one a CTA pair
    int C = (int)std::min<int64_t>(cta2 ? ctx->sm_count / 2 : ctx->sm_count, W);
    for (;; C = std::max(1, C * 3 / 4)) {
        int worst = 0;
        for (int cc = 0; cc < C; cc++) {
            const int64_t lo = (int64_t)cc * W / C, hi = (int64_t)(cc + 1) * W / C;
            const auto a = std::upper_bound(start.begin(), start.end(), lo) - start.begin() - 1;
            const auto b = std::upper_bound(start.begin(), start.end(), hi - 1) - start.begin() - 1;
            worst = std::max(worst, (int)(b - a + 1));
        }
        if (worst <= kseg || C == 1) break;
    }
    pp.n_cta = C;
    pp.kseg = kseg;
    pp.scale = ctx->scale;
    pp.mask = mk.ptr;
    pp.mask_stride = mk.stride;
    pp.mask_f16 = mk.f16 ? 1 : 0;
    pp.mask_vec = mk.ptr && reinterpret_cast<uintptr_t>(mk.ptr) % 16 == 0 &&
                  (mk.stride * (mk.f16 ? 2 : 4)) % 16 == 0;
    pp.flash = mk.flash ? 1 : 0;
    pp.pstat = ctx->pf_stat;
    pp.pout = ctx->pf_out;
    pp.rstat = ctx->pf_rstat;
    pp.out = dst;
    pp.out_stride = dst_stride;
    pp.out_head0 = dst_head0;
    pp.err = ctx->err;
    pp.limit_ns = ctx->limit_ns;
    static const char *what[5] = {"prefill attention kernel", "prefill output fold", "prefill statistics kernel",
                                  "prefill statistics fold", "prefill output kernel"};
    static const int one_pass[] = {0, 1}, exact[] = {2, 3, 4, 1};
    const int *seq = pp.mode ? exact : one_pass;
    const int nseq = pp.mode ? 4 : 2;
    for (int n = 0; n < nseq; n++) {
        const int which = seq[n];
        const int kid = (which == 1 || which == 3) ? KV_K_PFOLD : (which == 0 && cta2) ? KV_K_PREFILL2 : KV_K_PREFILL;
        const int rc = launch(ctx, kid, st, what[which], [&] {
            return which == 0 && cta2 ? kvb::launch_prefill_pair(ctx->qmap, *km32, vm, pp, st)
                                      : kvb::launch_prefill(ctx->pf_D, which, ctx->qmap, km, vm, pp, st);
        });
        if (rc) return rc;
    }
    return KV_OK;
}

}  // namespace

static int attend_impl(kv_ctx *ctx, int32_t layer, int64_t n_past, int32_t n_new, const MaskArg &mk_in, float *out,
                void *stream)
{
    if (!ctx) return fail(KV_E_ARG, "NULL context");
    if (!out) return fail(KV_E_ARG, "out is NULL");
    if (layer != ctx->last_layer || n_past != ctx->last_n_past || n_new != ctx->last_n_new)
        return fail(KV_E_STATE, "kv_attend(layer %d, n_past %lld, n_new %d) does not follow kv_append of the same rows",
                    layer, (long long)n_past, n_new);
    int rc = ensure_device(ctx);
    if (rc) return rc;
    const kv_config &c = ctx->cfg;
    const cudaStream_t st = to_stream(stream);
    // the deferred single-token append runs inside the attention kernels when it
    // belongs to this call and stream; otherwise it is performed now
    const bool fused = ctx->pend.on && ctx->pend.layer == layer && ctx->pend.n_past == n_past &&
                       ctx->pend.n_new == 1 && n_new == 1 && ctx->pend.st == st;
    const Pending pd = ctx->pend;
    if (fused) ctx->pend.on = false;
    else {
        rc = flush_pending(ctx);
        if (rc) return rc;
    }
    const int64_t D = ctx->D;
    // a ring cache attends over its cells in use: the kernels see them as keys
    // [0, n_kv), the new tokens' rows among them, under a mask (the caller's,
    // or dory's visibility built here) or, for one token, every key
    const int64_t n_kv = ctx->ring ? std::min<int64_t>(ctx->ring, n_past + n_new) : n_past + n_new;
    const int64_t kpast = n_kv - n_new;   // the kernels' n_past
    MaskArg mk = mk_in;
    if (mk.ptr && mk.stride < n_kv)
        return fail(KV_E_ARG, "mask_stride %lld < the %lld keys attended", (long long)mk.stride, (long long)n_kv);
    bool all_keys = false;
    if (ctx->ring && !mk.ptr) {
        if (n_new == 1) {
            all_keys = true;
        } else {
            KV_CUDA(kvb::launch_ring_mask(ctx->ring_mask, ctx->rows, ctx->ring, n_past, n_new, n_kv, st));
            mk.ptr = ctx->ring_mask;
            mk.stride = ctx->rows;
            mk.f16 = true;
        }
    }
    const bool sharded = c.n_shards > 1;
    const bool direct = !sharded || n_new == 1;
    float *dst = direct ? out : ctx->local_out;
    const int64_t dst_stride = direct ? (int64_t)c.n_head * D : (int64_t)ctx->hq_loc * D;
    const int dst_head0 = direct ? ctx->hq0 : 0;

    kvb::AttnParams ap{};
    ap.hkv = ctx->hkv_loc;
    ap.r = ctx->r;
    ap.hq_loc = ctx->hq_loc;
    ap.hq0 = ctx->hq0;
    ap.hkv0 = ctx->hkv0;
    ap.n_kv = n_kv;
    ap.n_past = kpast;
    {
        // clusters need the CTAs resident together with the cooperative
        // launch's guarantee off: the cooperative attribute keeps the plain grid
        const DecodeShape ds = decode_shape_for(ctx->dec_sms, ctx->hkv_loc, n_kv,
                                                ctx->coop ? nullptr : ctx->max_clusters, ctx->force_q,
                                                ctx->min_keys);
        ap.n_cta = ds.n_cta;
        ap.cq = ds.cq;
        ap.ncl = ds.ncl;
    }
    ap.l2pf = ctx->l2pf >= 0 ? ctx->l2pf : l2pf_default(ctx->hkv_loc, n_kv, ap.n_cta);
    ap.scale = ctx->scale;
    ap.fused = fused ? 1 : 0;
    ap.q = pd.q;
    ap.k = pd.k;
    ap.v = pd.v;
    ap.q_stride = pd.q_stride;
    ap.q_norm_w = pd.qn;
    ap.k_norm_w = pd.kn;
    ap.q_bias = pd.qb;
    ap.k_bias = pd.kb;
    ap.v_bias = pd.vb;
    ap.qk_norm = c.qk_norm;
    ap.n_rot = c.n_rot;
    ap.rope_mode = c.rope_mode;
    ap.eps = c.rms_eps;
    ap.rope = ctx->rope;
    ap.kc = ctx->k_layer(layer);
    ap.vc = ctx->v_layer(layer);
    ap.qbuf = ctx->qbuf;
    ap.S = ctx->S;
    ap.stats = ctx->stats;
    ap.acc = ctx->acc;
    ap.counters = ctx->ctl;
    ap.nonfin = ctx->ctl + ctx->hkv_loc;
    ap.hz_row = (ctx->hz_stream == st && ctx->hz_layer == layer) ? ctx->hz_row : -1;
    ap.err = ctx->err;
    ap.limit_ns = ctx->limit_ns;
    ap.inject = ctx->inject;
    ctx->inject = 0;
    ap.out = dst;
    ap.out_stride = dst_stride;
    ap.out_head0 = dst_head0;
    ap.mask = mk.ptr;
    ap.mask_stride = mk.stride;
    ap.mask_f16 = mk.f16 ? 1 : 0;
    ap.flash = mk.flash ? 1 : 0;
    ap.all_keys = all_keys ? 1 : 0;
    ap.wait_first = ctx->ring ? 1 : 0;
    const bool via_peers = sharded && ctx->peers && n_new == 1 && ctx->r <= kvb::attn_rows() &&
                           !(!fused && ctx->pf && n_new * ctx->r >= 32);
    ap.n_peers = via_peers ? c.n_shards : 0;
    ap.xpull = ctx->xpull ? 1 : 0;
    ap.shard = c.shard;
    ap.rx_stride = ctx->rx_stride;
    ap.xticket = ctx->ctl + 2 * ctx->hkv_loc;
    for (int g = 0; g < kvb::kMaxShards; g++) {
        ap.rx[g] = via_peers ? ctx->peer_rx[g] : nullptr;
    }
    if (ap.n_cta > ctx->max_cta) return fail(KV_E_RANGE, "internal: %d CTAs > %d", ap.n_cta, ctx->max_cta);
    kvb::attn_split(ap, ctx->hkv_loc, n_kv);
    if ((int64_t)ap.n_cta * ap.S_tiles * kvb::attn_tile_scores() > ctx->S_floats)
        return fail(KV_E_RANGE, "internal: score scratch too small for %d CTAs x %lld tiles", ap.n_cta,
                    (long long)ap.S_tiles);

    const int rows = n_new * ctx->r;
    const int rows_per = kvb::attn_rows();
    const CUtensorMap &km = ctx->kmaps[layer], &vm = ctx->vmaps[layer];
    if (!fused && ctx->pf && rows >= 32) {
        const bool padded = !ctx->pf_kmaps.empty();   // head_dim 96 on the 128 kernel
        rc = prefill(ctx, padded ? ctx->pf_kmaps[layer] : km, padded ? ctx->pf_vmaps[layer] : vm,
                     ctx->pf2_kmaps.empty() ? nullptr : &ctx->pf2_kmaps[layer], kpast, n_new, dst, dst_stride,
                     dst_head0, mk, st);
        if (rc) return rc;
    }
    for (int row0 = 0; row0 < rows && !(!fused && ctx->pf && rows >= 32); row0 += rows_per) {
        ap.row0 = row0;
        ap.nrows = std::min(rows_per, rows - row0);
        if (++ctx->epoch == 0) {
            // the tag wrapped: no slot may carry an old launch's tag 1
            KV_CUDA(cudaMemsetAsync(ctx->stats, 0, (size_t)ctx->max_cta * 2u * 8u * 2u * sizeof(unsigned long long), st));
            ctx->epoch = 1;
        }
        ap.epoch = ctx->epoch;
#ifdef KV_PHASE_STAMPS
        ap.stamps = ctx->stamps + (size_t)(ctx->stamp_next++ % kv_ctx::kStampRing) * ctx->max_cta * kvb::kStampSlots;
#endif
        rc = launch(ctx, KV_K_ATTN, st, "attention kernel",
                    [&] { return kvb::launch_attn(ctx->D, km, vm, ap, st, true, ctx->coop); });
        if (rc) return rc;
        ap.hz_row = -1;   // row groups after the first do not write the cache
    }
    ctx->hz_stream = st;
    ctx->hz_layer = fused ? layer : -1;
    ctx->hz_row = fused ? n_past : -1;

    if (sharded && !via_peers) {
        NcclApi &api = nccl();
        const size_t cols = (size_t)ctx->hq_loc * D;
        int nr;
        if (direct) {
            // in place: this shard's heads already sit at out + shard*cols
            nr = api.AllGather(out + (size_t)c.shard * cols, out, cols, kNcclFloat32, ctx->comm, st);
        } else {
            nr = api.AllGather(ctx->local_out, ctx->gathered, (size_t)n_new * cols, kNcclFloat32, ctx->comm, st);
        }
        if (nr != 0) return fail(KV_E_COMM, "ncclAllGather: %s", api.GetErrorString ? api.GetErrorString(nr) : "error");
        if (!direct) {
            rc = launch(ctx, KV_K_GATHER, st, "unshard kernel", [&] {
                return kvb::launch_unshard(out, (int64_t)c.n_head * D, ctx->gathered, c.n_shards, n_new, (int)cols, st);
            });
            if (rc) return rc;
        }
    }
    return KV_OK;
}

int kv_attend(kv_ctx *ctx, int32_t layer, int64_t n_past, int32_t n_new, float *out, void *stream)
{
    if (!ctx) return fail(KV_E_ARG, "NULL context");
    MaskArg mk;
    mk.flash = ctx->cfg.flash_attn != 0;   // the session's branch (use_flash_attn)
    return guarded("kv_attend", [&] { return attend_impl(ctx, layer, n_past, n_new, mk, out, stream); });
}

int kv_attend_mask(kv_ctx *ctx, int32_t layer, int64_t n_past, int32_t n_new, const void *mask, int32_t mask_type,
                   int64_t mask_stride, uint32_t flags, float *out, void *stream)
{
    if (mask_type != KV_MASK_F32 && mask_type != KV_MASK_F16)
        return fail(KV_E_ARG, "unknown mask type %d", mask_type);
    if ((flags & ~(uint32_t)KV_ATTN_FLASH) != 0) return fail(KV_E_ARG, "unknown flags 0x%x", flags);
    MaskArg mk;
    mk.ptr = mask;
    mk.stride = mask ? mask_stride : 0;
    mk.f16 = mask_type == KV_MASK_F16;
    mk.flash = (flags & KV_ATTN_FLASH) != 0 || (ctx && ctx->cfg.flash_attn != 0);
    return guarded("kv_attend_mask", [&] { return attend_impl(ctx, layer, n_past, n_new, mk, out, stream); });
}

int kv_forward(kv_ctx *ctx, int64_t n_past, int32_t n_new,
               const float *q, int64_t q_stride, const float *k, int64_t k_stride,
               const float *v, int64_t v_stride, int64_t in_layer_stride,
               const float *q_norm_w, const float *k_norm_w, int64_t norm_layer_stride,
               float *out, int64_t out_layer_stride, void *stream)
{
    if (!ctx) return fail(KV_E_ARG, "NULL context");
    for (int l = 0; l < ctx->cfg.n_layer; l++) {
        const int64_t io = (int64_t)l * in_layer_stride;
        const int64_t no = (int64_t)l * norm_layer_stride;
        int rc = kv_append(ctx, l, n_past, n_new, q + io, q_stride, k + io, k_stride, v + io, v_stride,
                           q_norm_w ? q_norm_w + no : nullptr, k_norm_w ? k_norm_w + no : nullptr, stream);
        if (rc) return rc;
        rc = kv_attend(ctx, l, n_past, n_new, out + (int64_t)l * out_layer_stride, stream);
        if (rc) return rc;
    }
    return KV_OK;
}

static int rows_io(kv_ctx *ctx, int32_t layer, int32_t which, int64_t row0, int64_t nrows, void *host, bool to_host)
{
    if (!ctx || !host) return fail(KV_E_ARG, "NULL argument");
    if (layer < 0 || layer >= ctx->cfg.n_layer || (which != 0 && which != 1))
        return fail(KV_E_ARG, "bad layer or which");
    if (row0 < 0 || nrows < 0 || row0 > ctx->rows || nrows > ctx->rows - row0)
        return fail(KV_E_RANGE, "rows outside the cache");
    int rc = ensure_device(ctx);
    if (rc) return rc;
    rc = flush_pending(ctx);
    if (rc) return rc;
    __half *base = (which == 0 ? ctx->k_layer(layer) : ctx->v_layer(layer)) + row0 * (int64_t)ctx->hkv_loc * ctx->D;
    const size_t bytes = (size_t)nrows * ctx->hkv_loc * ctx->D * sizeof(__half);
    if (bytes == 0) return KV_OK;
    KV_CUDA(cudaDeviceSynchronize());
    if (to_host) KV_CUDA(cudaMemcpy(host, base, bytes, cudaMemcpyDeviceToHost));
    else KV_CUDA(cudaMemcpy(base, host, bytes, cudaMemcpyHostToDevice));
    return KV_OK;
}

int kv_export_rows(kv_ctx *ctx, int32_t layer, int32_t which, int64_t row0, int64_t nrows, uint16_t *host_dst)
{
    return rows_io(ctx, layer, which, row0, nrows, host_dst, true);
}

int kv_import_rows(kv_ctx *ctx, int32_t layer, int32_t which, int64_t row0, int64_t nrows, const uint16_t *host_src)
{
    return rows_io(ctx, layer, which, row0, nrows, const_cast<uint16_t *>(host_src), false);
}

int kv_comm_unique_id(void *id_out)
{
    if (!id_out) return fail(KV_E_ARG, "id_out is NULL");
    NcclApi &api = nccl();
    if (!api.GetUniqueId) return fail(KV_E_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    NcclId id;
    const int rc = api.GetUniqueId(&id);
    if (rc != 0) return fail(KV_E_COMM, "ncclGetUniqueId failed (%d)", rc);
    std::memcpy(id_out, id.internal, sizeof(id.internal));
    return KV_OK;
}

const char *kv_strerror(int code)
{
    switch (code) {
    case KV_OK: return "ok";
    case KV_E_ARG: return "invalid argument";
    case KV_E_OOM: return "device out of memory";
    case KV_E_RANGE: return "row range out of bounds";
    case KV_E_CUDA: return "CUDA error";
    case KV_E_COMM: return "collective error";
    case KV_E_TIMEOUT: return "device wait timed out";
    case KV_E_STATE: return "call order violated";
    case KV_E_UNSUPPORTED: return "unsupported";
    default: return "unknown error";
    }
}

const char *kv_last_error(void) { return g_last_error; }

int kv_status(kv_ctx *ctx, void *stream)
{
    if (!ctx) return fail(KV_E_ARG, "NULL context");
    int rc = ensure_device(ctx);
    if (rc) return rc;
    rc = flush_pending(ctx);
    if (rc) return rc;
    KV_CUDA(cudaStreamSynchronize(to_stream(stream)));
    unsigned word = 0;
    KV_CUDA(cudaMemcpy(&word, ctx->err, sizeof(word), cudaMemcpyDeviceToHost));
    if (word == 0) return KV_OK;
    // a CTA that left early never counted itself in: restart the per-head
    // tickets and clear the output accumulators
    KV_CUDA(cudaMemset(ctx->ctl, 0, (2u * (size_t)ctx->hkv_loc + 1u) * sizeof(unsigned)));
    KV_CUDA(cudaMemset(ctx->acc, 0, (size_t)ctx->hkv_loc * 8u * (size_t)ctx->D * sizeof(long long)));
    KV_CUDA(cudaMemset(ctx->err, 0, sizeof(unsigned)));
    return fail(KV_E_TIMEOUT, "a device-side wait expired (error word 0x%x); the outputs of that call are invalid",
                word);
}

int kv_debug_inject(kv_ctx *ctx, int32_t what, uint64_t limit_ns)
{
    if (!ctx) return fail(KV_E_ARG, "NULL context");
    if (what != 0 && what != 1) return fail(KV_E_ARG, "unknown injection %d", what);
    ctx->inject = what;
    if (limit_ns) ctx->limit_ns = limit_ns;
    return KV_OK;
}

// ---- kv_bench.h -------------------------------------------------------------

int kv_fill_synthetic(kv_ctx *ctx, uint64_t seed, uint64_t stream_base, int64_t row0, int64_t nrows, void *stream)
{
    if (!ctx) return fail(KV_E_ARG, "NULL context");
    if (row0 < 0 || nrows < 0 || row0 > ctx->rows || nrows > ctx->rows - row0)
        return fail(KV_E_RANGE, "rows outside the cache");
    int rc = ensure_device(ctx);
    if (rc) return rc;
    rc = flush_pending(ctx);
    if (rc) return rc;
    kvb::FillParams p;
    p.cache = ctx->cache;
    p.n_layer = ctx->cfg.n_layer;
    p.D = ctx->D;
    p.hkv_loc = ctx->hkv_loc;
    p.hkv_total = ctx->cfg.n_head_kv;
    p.hkv0 = ctx->hkv0;
    p.n_ctx = ctx->rows;
    p.row0 = row0;
    p.nrows = nrows;
    p.seed = seed;
    p.stream_base = stream_base;
    KV_CUDA(kvb::launch_fill(p, to_stream(stream)));
    return KV_OK;
}

int kv_gen_normal_device(float *dst, uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n, void *cuda_stream)
{
    if (!dst || n < 0) return fail(KV_E_ARG, "bad argument");
    KV_CUDA(kvb::launch_gen_normal(dst, seed, stream, idx0, n, to_stream(cuda_stream)));
    return KV_OK;
}

int kv_profile_enable(kv_ctx *ctx, int on)
{
    if (!ctx) return fail(KV_E_ARG, "NULL context");
    ctx->prof_on = on != 0;
    return KV_OK;
}

int kv_profile_reset(kv_ctx *ctx)
{
    if (!ctx) return fail(KV_E_ARG, "NULL context");
    for (auto &r : ctx->recs) cudaEventSynchronize(r.b);
    try {
        ctx->ev_pool.reserve(ctx->ev_pool.size() + 2 * ctx->recs.size());
        for (auto &r : ctx->recs) {
            ctx->ev_pool.push_back(r.a);
            ctx->ev_pool.push_back(r.b);
        }
    } catch (const std::bad_alloc &) {   // no room to pool them: release the events instead
        for (auto &r : ctx->recs) {
            cudaEventDestroy(r.a);
            cudaEventDestroy(r.b);
        }
    }
    ctx->recs.clear();
    return KV_OK;
}

int kv_profile_read(kv_ctx *ctx, int32_t kernel, int64_t *launches, double *total_ms)
{
    if (!ctx || kernel < 0 || kernel >= KV_K_COUNT) return fail(KV_E_ARG, "bad argument");
    int64_t n = 0;
    double ms = 0.0;
    for (auto &r : ctx->recs) {
        if (r.k != kernel) continue;
        KV_CUDA(cudaEventSynchronize(r.b));
        float t = 0.0f;
        KV_CUDA(cudaEventElapsedTime(&t, r.a, r.b));
        n++;
        ms += t;
    }
    if (launches) *launches = n;
    if (total_ms) *total_ms = ms;
    return KV_OK;
}

const char *kv_kernel_name(int32_t kernel)
{
    static const char *names[KV_K_COUNT] = {"kv_append", "kv_attn", "kv_prefill", "kv_prefill_fold", "kv_unshard",
                                            "kv_prefill_pair"};
    return (kernel >= 0 && kernel < KV_K_COUNT) ? names[kernel] : "?";
}

int64_t kv_launch_count(const kv_ctx *ctx) { return ctx ? ctx->launches.load() : 0; }

#ifdef KV_PHASE_STAMPS
// Measurement builds only: copies the stamp ring ([ring][max_cta][slots]
// globaltimer values) to host_dst and returns the number of launches stamped
// so far (launch i sits in ring slot i % ring); *ring and *max_cta describe it.
int64_t kv_debug_stamps(kv_ctx *ctx, unsigned long long *host_dst, int32_t *ring, int32_t *max_cta)
{
    if (!ctx || !ring || !max_cta) return -1;
    if (ensure_device(ctx)) return -1;
    *ring = kv_ctx::kStampRing;
    *max_cta = ctx->max_cta;
    if (host_dst) {   // (NULL: the sizes only)
        cudaDeviceSynchronize();
        cudaMemcpy(host_dst, ctx->stamps, (size_t)kv_ctx::kStampRing * ctx->max_cta * kvb::kStampSlots * 8u,
                   cudaMemcpyDeviceToHost);
    }
    return ctx->stamp_next;
}
#else
int64_t kv_debug_stamps(kv_ctx *ctx, unsigned long long *host_dst, int32_t *ring, int32_t *max_cta)
{
    (void)ctx;
    (void)host_dst;
    (void)ring;
    (void)max_cta;
    return (int64_t)fail(KV_E_UNSUPPORTED, "this library was built without KV_PHASE_STAMPS (build.py --stamps)");
}
#endif

int kv_rope_table_host(const kv_config *cfg, int64_t pos0, int64_t npos, float *out)
{
    if (!cfg || !out || pos0 < 0 || npos < 0) return fail(KV_E_ARG, "bad argument");
    return guarded("kv_rope_table_host", [&] {
        std::string why;
        if (!shape_ok(cfg, why)) return fail(KV_E_ARG, "%s", why.c_str());
        if (cfg->n_rot == 0 || npos == 0) return KV_OK;
        RopeSpec rs{cfg->n_rot, cfg->rope_base, cfg->rope_freq_scale, cfg->rope_attn_factor, cfg->rope_ext_factor,
                    cfg->rope_beta_fast, cfg->rope_beta_slow, cfg->n_ctx_orig, cfg->rope_freq_factors};
        rope_rows(rs, pos0, pos0 + npos, out);
        return KV_OK;
    });
}

int kv_decode_shape(int32_t sm_count, int32_t n_kv_heads_local, int64_t n_kv, const int32_t *max_clusters,
                    int32_t *n_cta, int32_t *cluster_ctas, int32_t *clusters_per_head)
{
    if (!n_cta || !cluster_ctas || !clusters_per_head || sm_count <= 0 || n_kv_heads_local <= 0 || n_kv <= 0)
        return fail(KV_E_ARG, "bad argument");
    int mc[kvb::kMaxClusterCtas + 1] = {};
    if (max_clusters)
        for (int q = 2; q <= kvb::kMaxClusterCtas; q++) mc[q] = max_clusters[q];
    const DecodeShape d = decode_shape_for(sm_count, n_kv_heads_local, n_kv, max_clusters ? mc : nullptr, 0);
    *n_cta = d.n_cta;
    *cluster_ctas = d.cq;
    *clusters_per_head = d.ncl;
    return KV_OK;
}

int kv_decode_grid_fits(int32_t sm_count, int32_t blocks_per_sm, int32_t n_cta)
{
    return decode_grid_fits(sm_count, blocks_per_sm, n_cta) ? 1 : 0;
}

int kv_decode_ctas(int32_t sm_count, int32_t n_kv_heads_local, int64_t n_kv, int32_t *n_cta)
{
    if (!n_cta || sm_count <= 0 || n_kv_heads_local <= 0 || n_kv <= 0) return fail(KV_E_ARG, "bad argument");
    *n_cta = decode_ctas_for(sm_count, n_kv_heads_local, n_kv);
    return KV_OK;
}

int kv_shard_geometry(const kv_config *cfg, int32_t shard, int32_t *q_head0, int32_t *n_q_heads,
                      int32_t *kv_head0, int32_t *n_kv_heads)
{
    if (!cfg) return fail(KV_E_ARG, "NULL cfg");
    std::string why;
    if (!shape_ok(cfg, why)) return fail(KV_E_ARG, "%s", why.c_str());
    const int ns = cfg->n_shards <= 1 ? 1 : cfg->n_shards;
    if (shard < 0 || shard >= ns) return fail(KV_E_ARG, "shard out of range");
    const int hkv = cfg->n_head_kv / ns, r = cfg->n_head / cfg->n_head_kv;
    if (q_head0) *q_head0 = shard * hkv * r;
    if (n_q_heads) *n_q_heads = hkv * r;
    if (kv_head0) *kv_head0 = shard * hkv;
    if (n_kv_heads) *n_kv_heads = hkv;
    return KV_OK;
}

}  // extern "C"
