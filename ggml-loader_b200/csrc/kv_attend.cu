// kv_attend.cu -- attention of kv_attend: one TMA-fed, tensor-core kernel per
// layer (and per group of <= 8 query rows), chained to its neighbours with
// programmatic dependent launch.
//
// Numerics: the reference's default attention branch (src/model.cpp:1416-1445):
// scores = F16(q) . K accumulated in F32, softmax with the global max and sum,
// p = F16(expf(s - max) * (1/sum)), out = p . V accumulated in F32.  ggml rounds
// the *normalised* p to F16 (its mul_mat converts the F32 operand), so no p can
// be formed before the head's global max and sum are known: the kernel runs a K
// phase, a per-head statistics exchange, then a V phase.
//
// Work split: the layer's Hkv*n_kv (head, key) rows, head-major, are cut into C
// equal contiguous ranges, one CTA each (hkv <= C <= SMs, one CTA per SM, so
// all CTAs are resident together), every SM streams the same number of bytes
// and a CTA spans at most two heads (two "segments"); C is a multiple of the
// heads, so that no CTA straddles two, when that idles at most 5 % of the SMs.
//
// attn_decode_kernel
//   * warp 8 streams the range's K tiles (128 keys; 64-wide boxes with 128-byte
//     swizzle, 32-wide with 64-byte swizzle at head_dim 96) and straight after
//     them its V tiles through one NS-stage mbarrier ring (cp.async.bulk.tensor),
//     so HBM never waits for the phase change;
//   * K phase: warps 0-7 take 16 keys of a tile each and compute S = K . Q^T with
//     mma.m16n8k16 (F16 x F16 -> F32; the GQA group's query rows are N <= 8).
//     Scores go to per-CTA scratch in the order the V phase reads them back,
//     running max / sum of exp stay in registers;
//   * decode (one new token) performs the append: every CTA rotates (and
//     RMS-normalises, qwen3) the query rows of its heads, the CTA that owns a
//     head's new row rotates the K row, writes K and V to the cache and patches
//     them into its staged tiles -- bit-identical to kv_append;
//   * statistics: each CTA publishes its (max, sum) per (segment, row) and counts
//     itself in on a per-head ticket, then waits (bounded) for the other CTAs of
//     its heads while the producer keeps filling the ring with V;
//   * V phase: p = F16(expf(s - M) / Z) formed directly as the mma B fragment,
//     O^T += V^T . P^T (ldmatrix.trans); rows past the valid keys are zeroed so
//     stale data never reaches the sum; the scores come back through a
//     per-thread cp.async ring;
//   * output: each (CTA, segment) partial is added into a per-head fixed-point
//     accumulator (2^-40) with 64-bit integer atomics -- exact, so the result
//     does not depend on the order CTAs finish -- and the head's last CTA
//     converts it to F32, writes the output and clears the accumulator.
// Every wait is bounded (limit_ns): an expired wait sets the error word read by
// kv_status, and the CTA drains its own tile loads before leaving.
#include <math.h>

#include <algorithm>

#include "kv_internal.h"
#include "kv_sm100.cuh"

namespace kvb {
namespace {

using namespace sm100;

// Phase stamps for measurement builds (-DKV_PHASE_STAMPS): one %globaltimer
// value per (CTA, phase) into AttnParams::stamps; nothing in other builds.
#ifdef KV_PHASE_STAMPS
#define KV_STAMP(cond, i)                                                                  \
    do {                                                                                   \
        if (p.stamps && (cond)) p.stamps[(int64_t)blockIdx.x * kStampSlots + (i)] = globaltimer(); \
    } while (0)
#else
#define KV_STAMP(cond, i) do { } while (0)
#endif

constexpr int kTK = 128;         // keys per tile (8 warps x 16)
constexpr int kConsumers = 256;  // warps 0-7
constexpr int kThreads = 288;    // + producer warp 8
constexpr int kRows = 8;         // query rows per launch (mma N)
constexpr int kSD = 4;           // depth of the per-thread score ring of the V phase
constexpr int kTileScores = 8 * kRows * 16;   // floats of score scratch per tile
constexpr int kMaxSpan = 160;  // CTAs one head may span (launches have at most this many CTAs)
constexpr float kFix = 1099511627776.0f;      // 2^40: output accumulator scale
constexpr float kUnfix = 1.0f / 1099511627776.0f;

template <int D> struct G4;
template <> struct G4<64>  { static constexpr int BW = 64, NS = 11; };
template <> struct G4<96>  { static constexpr int BW = 32, NS = 6; };
// (4 stages: 128 KB in flight an SM keeps HBM busy; a fifth only lengthens the
// queue the statistics poll and the query loads wait behind -- 128k: 92.7 ->
// 90.7 us a layer, 32k: 28.9 -> 28.8)
template <> struct G4<128> { static constexpr int BW = 64, NS = 4; };
template <> struct G4<256> { static constexpr int BW = 64, NS = 2; };   // 64 KB stages; the V-phase buffer takes 66 KB

template <int BW>
__device__ __forceinline__ uint32_t swz(int row, int chunk)
{
    if constexpr (BW == 64) return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
    else return (uint32_t)(row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4));
}

// ---- the balanced split -----------------------------------------------------
struct Range {
    int h0;
    int64_t s0, e0, e1;
    int nt0, nt;
};

__device__ __forceinline__ Range cta_range(int c, int64_t n_kv, int hkv, int C)
{
    const int64_t T = (int64_t)hkv * n_kv;
    const int64_t lo = (int64_t)c * T / C, hi = (int64_t)(c + 1) * T / C;
    Range g;
    g.h0 = (int)(lo / n_kv);
    g.s0 = lo - (int64_t)g.h0 * n_kv;
    g.e0 = min(n_kv, hi - (int64_t)g.h0 * n_kv);
    g.e1 = hi > (int64_t)(g.h0 + 1) * n_kv ? hi - (int64_t)(g.h0 + 1) * n_kv : 0;
    g.nt0 = (int)((g.e0 - g.s0 + kTK - 1) / kTK);
    g.nt = g.nt0 + (int)((g.e1 + kTK - 1) / kTK);
    return g;
}

__device__ __forceinline__ void tile_of(const Range &g, int i, int &h, int64_t &k0, int64_t &kend)
{
    if (i < g.nt0) { h = g.h0; k0 = g.s0 + (int64_t)i * kTK; kend = g.e0; }
    else { h = g.h0 + 1; k0 = (int64_t)(i - g.nt0) * kTK; kend = g.e1; }
}

// the caller's additive mask at (token, key)
__device__ __forceinline__ float mask_at(const AttnParams &p, int tok, int64_t key)
{
    const int64_t i = (int64_t)tok * p.mask_stride + key;
    return p.mask_f16 ? __half2float(__ldg(reinterpret_cast<const __half *>(p.mask) + i))
                      : __ldg(reinterpret_cast<const float *>(p.mask) + i);
}

// index of the (CTA, segment) statistics of local head h held by CTA cc
__device__ __forceinline__ int64_t part_slot(const AttnParams &p, int h, int cc)
{
    return (int64_t)cc * 2 + (cc == p.span_a[h] ? p.span_slot[h] : 0);
}

// ---- the fused single-token append ---------------------------------------------
// (cos, sin) entries of this lane's dims at the new position: the table is
// written once at kv_alloc, so this may run before griddepcontrol.wait.
template <int D>
__device__ __forceinline__ void rope_prefetch(const AttnParams &p, float2 (&csr)[(D + 31) / 32])
{
    const int lane = threadIdx.x & 31, half = p.n_rot >> 1;
    const float2 *cs = p.rope + p.n_past * (int64_t)half;
#pragma unroll
    for (int e = 0; e < (D + 31) / 32; e++) {
        const int i = lane + 32 * e;
        csr[e] = make_float2(1.0f, 0.0f);
        if (i < p.n_rot) csr[e] = __ldg(cs + (p.rope_mode == 2 ? (i < half ? i : i - half) : (i >> 1)));
    }
}

// One warp turns one head vector (D floats at src) into its rotated, optionally
// RMS-normalised form in xs[] (shared), with the separately rounded arithmetic of
// kv_append (kv_append.cu) so the bits agree.
template <int D>
__device__ void warp_rotate(const float *src, const float *bias, const float *gamma, const AttnParams &p, float *xs,
                            float *tmp, const float2 (&csr)[(D + 31) / 32])
{
    constexpr int E = (D + 31) / 32;
    const int lane = threadIdx.x & 31;
    float x[E], w[E];
#pragma unroll
    for (int e = 0; e < E; e++) {
        const int i = lane + 32 * e;
        x[e] = i < D ? __ldg(src + i) : 0.0f;
        if (bias && i < D) x[e] = __fadd_rn(x[e], __ldg(bias + i));   // the projection bias, first
        w[e] = (gamma && i < D) ? __ldg(gamma + i) : 1.0f;
    }
#pragma unroll
    for (int e = 0; e < E; e++)
        if (lane + 32 * e < D) tmp[lane + 32 * e] = gamma ? __fmul_rn(x[e], x[e]) : x[e];
    __syncwarp();
    if (gamma) {
        float sc = 0.0f;
        if (lane == 0) {   // sequential double sum of the rounded squares
            double sum = 0.0;
            for (int i = 0; i < D; i++) sum = __dadd_rn(sum, (double)tmp[i]);
            const float mean = __double2float_rn(__ddiv_rn(sum, (double)D));
            sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
        }
        sc = __shfl_sync(0xffffffffu, sc, 0);
        __syncwarp();
#pragma unroll
        for (int e = 0; e < E; e++)
            if (lane + 32 * e < D) tmp[lane + 32 * e] = __fmul_rn(__fmul_rn(x[e], sc), w[e]);
        __syncwarp();
    }
    const int half = p.n_rot >> 1;
#pragma unroll
    for (int e = 0; e < E; e++) {
        const int i = lane + 32 * e;
        if (i >= D) break;
        float v = tmp[i];
        if (i < p.n_rot) {
            const float2 c = csr[e];
            if (p.rope_mode == 2) {
                if (i < half) v = __fsub_rn(__fmul_rn(tmp[i], c.x), __fmul_rn(tmp[i + half], c.y));
                else v = __fadd_rn(__fmul_rn(tmp[i - half], c.y), __fmul_rn(tmp[i], c.x));
            } else {
                if ((i & 1) == 0) v = __fsub_rn(__fmul_rn(tmp[i], c.x), __fmul_rn(tmp[i + 1], c.y));
                else v = __fadd_rn(__fmul_rn(tmp[i - 1], c.y), __fmul_rn(tmp[i], c.x));
            }
        }
        xs[i] = v;
    }
    __syncwarp();
}

// Store one F16 cache row (row `key` of the staged tile) into the swizzled boxes.
template <int D, int BW>
__device__ __forceinline__ void patch_row(unsigned char *stage, int key, const __half *row16)
{
    constexpr int CPB = BW / 8;            // 16-byte chunks per box row
    constexpr uint32_t kSub = kTK * BW * 2;
    const int lane = threadIdx.x & 31;
    for (int cidx = lane; cidx < D / 8; cidx += 32) {
        const uint4 v = *reinterpret_cast<const uint4 *>(row16 + cidx * 8);
        *reinterpret_cast<uint4 *>(stage + (cidx / CPB) * kSub + swz<BW>(key, cidx % CPB)) = v;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
}

// ---- shared memory -------------------------------------------------------------
template <int D>
struct Smem {
    static constexpr int BW = G4<D>::BW, NB = D / BW, NS = G4<D>::NS;
    static constexpr uint32_t kSub = kTK * BW * 2, kStage = kSub * NB;
    static constexpr int RED_LD = D + 4;
    static constexpr size_t ring = (size_t)NS * kStage;
    // K phase: rotated q [2 heads][8 rows][D] + per-warp scratch [8][D];
    // V phase: per-warp partial outputs [8 warps][8 rows][RED_LD]
    static constexpr size_t uni_k = (size_t)(2 * kRows + 8) * D * 4;
    static constexpr size_t uni_v = (size_t)8 * kRows * RED_LD * 4;
    static constexpr size_t uni = uni_k > uni_v ? uni_k : uni_v;
    static constexpr size_t o_uni = ring;
    static constexpr size_t o_sS = o_uni + uni;                            // [kSD][256][4] floats
    static constexpr size_t o_bar = o_sS + (size_t)kSD * kConsumers * 16;  // full[NS], empty[NS]
    static constexpr size_t o_redm = o_bar + (size_t)2 * NS * 8;           // [2][8 warps][8 rows]
    static constexpr size_t o_redz = o_redm + 2 * 8 * kRows * 4;
    static constexpr size_t o_row = o_redz + 2 * 8 * kRows * 4;            // rowM[2][8], rowInv[2][8]
    static constexpr size_t o_kf = o_row + 4 * kRows * 4;                  // [D] f32
    static constexpr size_t o_knew = o_kf + (size_t)D * 4;                 // [D] f16
    static constexpr size_t o_vnew = o_knew + (size_t)D * 2;               // [D] f16
    static constexpr size_t o_flags = o_vnew + (size_t)D * 2;              // abort, last(seg 0), last(seg 1), collector
    // cluster exchange (kMaxQ > 1): the cluster's (max, sum) per (rank, row),
    // two transaction barriers (statistics, partial outputs) and the leader's
    // receive buffer for the other ranks' partial outputs [kMaxQ-1][8 rows][D]
    static constexpr int kMaxQ = D <= 128 ? 8 : 1;
    static constexpr size_t o_cst = o_flags + 16;                          // [kMaxQ][8] float2
    static constexpr size_t o_cbar = o_cst + (size_t)kMaxQ * kRows * 8;   // [2] u64
    static constexpr size_t o_crecv = (o_cbar + 16 + 15) / 16 * 16;
    static constexpr size_t bytes = o_crecv + (size_t)(kMaxQ - 1) * kRows * D * 4;
    static_assert(bytes <= 227 * 1024, "shared memory of the attention kernel");
    static_assert(o_cst % 16 == 0 && o_cbar % 8 == 0 && o_crecv % 16 == 0, "aligned cluster regions");
    static_assert(kStage % 1024 == 0, "ring stages stay 1024-byte aligned");
    // the staged new rows and the scratch blocks are read with 16-byte vector loads
    static_assert(o_sS % 16 == 0 && o_kf % 16 == 0 && o_knew % 16 == 0 && o_vnew % 16 == 0 && o_redm % 16 == 0,
                  "16-byte aligned shared regions");
};

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// MASKED: the instance for the caller's mask or a ring's single token (every
// key visible); FLASH: the flash-attn branch; CL: cluster mode (launched with
// clusters of p.cq CTAs).  The plain causal default-branch instance is
// compiled without any of them.
template <int D, bool MASKED, bool FLASH, bool CL>
__global__ void __launch_bounds__(kThreads, 1) attn_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                    const __grid_constant__ CUtensorMap vmap,
                                                                    const AttnParams p)
{
    using L = Smem<D>;
    constexpr int BW = L::BW, NB = L::NB, NS = L::NS, KC = D / 16, DT = D / 16, RED_LD = L::RED_LD;
    constexpr uint32_t kSub = L::kSub, kStage = L::kStage;

    extern __shared__ __align__(1024) unsigned char smem[];
    float *qs = reinterpret_cast<float *>(smem + L::o_uni);                 // K phase
    float *tmp = qs + 2 * kRows * D;
    float *red = reinterpret_cast<float *>(smem + L::o_uni);                // V phase
    float *sS = reinterpret_cast<float *>(smem + L::o_sS);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::o_bar);
    uint64_t *empty = full + NS;
    float *red_m = reinterpret_cast<float *>(smem + L::o_redm);
    float *red_z = reinterpret_cast<float *>(smem + L::o_redz);
    float *rowM = reinterpret_cast<float *>(smem + L::o_row);
    float *rowInv = rowM + 2 * kRows;
    float *kf = reinterpret_cast<float *>(smem + L::o_kf);
    __half *knew = reinterpret_cast<__half *>(smem + L::o_knew);
    __half *vnew = reinterpret_cast<__half *>(smem + L::o_vnew);
    volatile int *flags = reinterpret_cast<volatile int *>(smem + L::o_flags);
    float2 *cst = reinterpret_cast<float2 *>(smem + L::o_cst);
    uint64_t *cbar = reinterpret_cast<uint64_t *>(smem + L::o_cbar);
    float *crecv = reinterpret_cast<float *>(smem + L::o_crecv);
    // cluster mode (p.cq > 1): CTAs c of one cluster cover one head; rank 0 leads
    constexpr bool clus = CL && L::kMaxQ > 1;   // the plain instances carry no cluster code
    const uint32_t crank = clus ? cluster_rank() : 0u;

    const int c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Range g = cta_range(c, p.n_kv, p.hkv, p.n_cta);
    const bool two = g.nt > g.nt0;
    const bool s_local = g.nt <= kSD;   // the range's scores fit the V phase's staging ring
    // decode: this CTA owns head h0's new row when its first segment ends the head
    const bool owns_new = p.fused && g.e0 == p.n_kv;
    const int it_new = owns_new ? (int)((p.n_past - g.s0) / kTK) : -1;

    if (tid == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 8);
        }
        flags[0] = 0;
        flags[1] = 0;
        flags[2] = 0;
        if (clus) {
            // statistics: every rank's 8 rows; partial outputs: the other
            // ranks' rows (leader only) -- counted as transaction bytes
            mbar_init(&cbar[0], 1);
            mbar_init(&cbar[1], 1);
            mbar_arrive_expect_tx(&cbar[0], (uint32_t)((p.cq - 1) * kRows * 8));
            if (crank == 0) mbar_arrive_expect_tx(&cbar[1], (uint32_t)((p.cq - 1) * p.nrows * D * 4));
        }
        fence_mbar_init();
    }
    __syncthreads();
    // no rank may store into another before its barriers are initialised
    if (clus) cluster_sync_all();
    KV_STAMP(tid == 0, 0);   // entry

    // ---- producer: K tiles 0..nt-1, then V tiles 0..nt-1, one ring ----
    if (warp == 8) {
        int issued = 0;
        if (lane == 0) {
            prefetch_tmap(&kmap);
            prefetch_tmap(&vmap);
            const int total = 2 * g.nt;
            bool waited = false;
            const uint64_t pol = policy_evict_first();   // K/V are read once per launch
            for (int j = 0; j < total; j++) {
                if (p.inject == 1 && j == 1) break;   // test hook: withhold tile 1
                const int s = j % NS;
                // the two waits for a free stage that last longest -- behind the
                // previous kernel's tail and behind the statistics exchange --
                // keep HBM busy: the next l2pf tiles go to L2 first
                if (((j == NS && (p.l2pf & 0x100)) || (j == g.nt + NS && (p.l2pf & 0x200))) && (p.l2pf & 0xff))
                    for (int t = j; t < total && t < j + (p.l2pf & 0xff); t++) {
                        const bool tv = t >= g.nt;
                        int h2;
                        int64_t k2, e2;
                        tile_of(g, tv ? t - g.nt : t, h2, k2, e2);
#pragma unroll
                        for (int b = 0; b < NB; b++) tma_prefetch_3d(tv ? &vmap : &kmap, b * BW, h2, (int)k2);
                    }
                if (j >= NS && !mbar_wait(&empty[s], ((j / NS) - 1) & 1, p.limit_ns)) {
                    atomicOr(p.err, 2u);
                    flags[0] = 1;
                    break;
                }
                if (flags[0]) break;
                const bool isv = j >= g.nt;
                int h;
                int64_t k0, kend;
                tile_of(g, isv ? j - g.nt : j, h, k0, kend);
                // rows the previous kernel may still write (a multi-token
                // append's rows, or the row a fused launch of this layer adds)
                // need its completion; every older kernel has completed,
                // since the previous one let this one start only after its
                // own griddepcontrol.wait
                if (!waited && (p.wait_first || (!p.fused && k0 + kTK > p.n_past) ||
                                (p.hz_row >= k0 && p.hz_row < k0 + kTK))) {
                    pdl_wait();
                    waited = true;
                }
                mbar_arrive_expect_tx(&full[s], kStage);
                if (j == 0) KV_STAMP(true, 10);   // first tile issued
                if (j == NS) KV_STAMP(true, 11);  // first tile past the ring depth issued
#pragma unroll
                for (int b = 0; b < NB; b++)
                    tma_load_3d_hint(smem + s * kStage + b * kSub, isv ? &vmap : &kmap, &full[s], b * BW, h, (int)k0,
                                     pol);
                issued = j + 1;
            }
            if (!waited) pdl_wait();   // complete only after the previous kernel
        }
        // the CTA leaves together; if the consumers gave up, tiles they never
        // took may still be landing: wait for the last load of every slot
        named_sync(2, kThreads);
        if (lane == 0 && flags[0])
            for (int j = issued > NS ? issued - NS : 0; j < issued; j++)
                mbar_wait(&full[j % NS], (j / NS) & 1, p.limit_ns);
        __syncwarp();
        if (clus) {   // every thread of the cluster takes part in its exit barrier
            cluster_arrive();
            cluster_wait();
        }
        return;
    }

    // ======================= K phase =======================
    const int gq = lane >> 2, cq = lane & 3;
    const int R = p.nrows;
    const int row_a = 2 * cq, row_b = 2 * cq + 1;
    const int tok_a = (p.row0 + min(row_a, R - 1)) / p.r, tok_b = (p.row0 + min(row_b, R - 1)) / p.r;
    // the last visible key of each row: the causal bound, or every key with a mask
    const bool masked = MASKED && p.mask;
    const bool flash = FLASH;
    const bool all = masked || (MASKED && p.all_keys);
    const int64_t lim_a = all ? p.n_kv : p.n_past + tok_a;
    const int64_t lim_b = all ? p.n_kv : p.n_past + tok_b;
    float *const Scta = p.S + (int64_t)c * p.S_tiles * kTileScores;

    float2 csr[(D + 31) / 32];
    if (p.fused) {
        rope_prefetch<D>(p, csr);
        // the query rows (and the new K row) into L2 while the previous kernel
        // finishes: L2 is coherent, so a row it still writes is read fresh below
        const int nq = R * (two ? 2 : 1);
        for (int it = warp; it < nq + (owns_new ? 1 : 0); it += 8)
            if (lane < D / 32) {
                const float *src = it < nq ? p.q + (int64_t)((p.row0 + it % R) / p.r) * p.q_stride +
                                                 (int64_t)(p.hq0 + (g.h0 + it / R) * p.r + (p.row0 + it % R) % p.r) * D
                                           : p.k + (int64_t)(p.hkv0 + g.h0) * D;
                l2_prefetch(src + lane * 32);
            }
    }
    pdl_wait();   // inputs, qbuf and the rows below may come from the previous kernel
    pdl_launch_dependents();   // only now: the next kernel may rely on every kernel before this one
    KV_STAMP(tid == 0, 1);   // griddepcontrol.wait returned

    // decode: rotate the query rows of both heads and the new K row, one item per warp
    if (p.fused) {
        const int nq = R * (two ? 2 : 1);
        for (int it = warp; it < nq + (owns_new ? 1 : 0); it += 8) {
            if (it < nq) {
                const int hs = it / R, row = p.row0 + it % R;
                const float *src = p.q + (int64_t)(row / p.r) * p.q_stride +
                                   (int64_t)(p.hq0 + (g.h0 + hs) * p.r + row % p.r) * D;
                const float *bq = p.q_bias ? p.q_bias + (int64_t)(p.hq0 + (g.h0 + hs) * p.r + row % p.r) * D
                                           : nullptr;
                warp_rotate<D>(src, bq, p.qk_norm ? p.q_norm_w : nullptr, p, qs + (hs * kRows + it % R) * D,
                               tmp + warp * D, csr);
            } else {
                warp_rotate<D>(p.k + (int64_t)(p.hkv0 + g.h0) * D,
                               p.k_bias ? p.k_bias + (int64_t)(p.hkv0 + g.h0) * D : nullptr,
                               p.qk_norm ? p.k_norm_w : nullptr, p, kf, tmp + warp * D, csr);
                __half *dst = p.kc + (p.n_past * (int64_t)p.hkv + g.h0) * D;
                for (int i = lane; i < D; i += 32) {
                    const __half h16 = __float2half_rn(kf[i]);
                    knew[i] = h16;
                    dst[i] = h16;
                }
            }
        }
        named_sync(1, kConsumers);
    }
    KV_STAMP(tid == 0, 2);   // query rows rotated

    // B fragments (Q^T): column n = query row gq, k = dims
    uint32_t bq[KC][2];
    auto load_q = [&](int hs) {
        const bool ok = gq < R;
        if (p.fused) {
#pragma unroll
            for (int kc = 0; kc < KC; kc++) {
                const float *qr = qs + (hs * kRows + (ok ? gq : 0)) * D + kc * 16 + 2 * cq;
                bq[kc][0] = ok ? pack_half2(__float2half_rn(qr[0]), __float2half_rn(qr[1])) : 0u;
                bq[kc][1] = ok ? pack_half2(__float2half_rn(qr[8]), __float2half_rn(qr[9])) : 0u;
            }
        } else {
            const int row = p.row0 + (ok ? gq : 0), h = g.h0 + hs;
            const __half *qrow = p.qbuf + ((int64_t)(row / p.r) * p.hq_loc + (int64_t)h * p.r + row % p.r) * D;
#pragma unroll
            for (int kc = 0; kc < KC; kc++) {
                const uint32_t lo = *reinterpret_cast<const uint32_t *>(qrow + kc * 16 + 2 * cq);
                const uint32_t hi = *reinterpret_cast<const uint32_t *>(qrow + kc * 16 + 2 * cq + 8);
                bq[kc][0] = ok ? lo : 0u;
                bq[kc][1] = ok ? hi : 0u;
            }
        }
    };
    load_q(0);

    float ma = -INFINITY, mb = -INFINITY, ma0 = -INFINITY, mb0 = -INFINITY;
    float za = 0.0f, zb = 0.0f, za0 = 0.0f, zb0 = 0.0f;
    bool aborted = false;
    const uint32_t ring = smem_addr(smem);
    {
        const int mi = lane >> 3;
        const int arow = warp * 16 + (lane & 7) + (mi & 1) * 8;
        // where this lane's four scores land in the warp's 128-float block: the
        // V phase's lane (row, c') reads keys 2c'+{0,1}, 2c'+8+{0,1} as one float4
        const int so_a = (row_a * 4 + (gq >> 1)) * 4 + (gq & 1);
        const int so_b = (row_b * 4 + (gq >> 1)) * 4 + (gq & 1);

        auto upd = [&](float &m, float &z, float s0, float s1) {
            const float mn = fmaxf(m, fmaxf(s0, s1));
            const float base = mn == -INFINITY ? 0.0f : mn;
            z = z * __expf(m - base) + __expf(s0 - base) + __expf(s1 - base);
            m = mn;
        };

        for (int i = 0; i < g.nt; i++) {
            if (i == g.nt0) {
                ma0 = ma; mb0 = mb; za0 = za; zb0 = zb;
                ma = mb = -INFINITY;
                za = zb = 0.0f;
                load_q(1);
            }
            const int s = i % NS;
            int h;
            int64_t k0, kend;
            tile_of(g, i, h, k0, kend);
            // (key gq, row 2cq), (key gq, row 2cq+1), (key gq+8, row 2cq), (key gq+8, row 2cq+1)
            const int64_t key0 = k0 + warp * 16 + gq, key1 = key0 + 8;
            const bool v0 = key0 < kend, v1 = key1 < kend;
            // the caller's mask: loaded before the tile wait, which hides the latency
            float mk[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (masked) {
                if (v0) {
                    mk[0] = mask_at(p, tok_a, key0);
                    mk[1] = mask_at(p, tok_b, key0);
                }
                if (v1) {
                    mk[2] = mask_at(p, tok_a, key1);
                    mk[3] = mask_at(p, tok_b, key1);
                }
            }
            const bool ok = mbar_wait(&full[s], (i / NS) & 1, p.limit_ns);
            if (__any_sync(0xffffffffu, !ok)) {
                if (lane == 0) {
                    atomicOr(p.err, 1u);
                    flags[0] = 1;
                }
                aborted = true;
                break;
            }
            if (i == it_new && (int)((p.n_past - k0) >> 4) == warp)
                patch_row<D, BW>(smem + s * kStage, (int)(p.n_past - k0), knew);

            float acc0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, acc1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int kc = 0; kc < KC; kc++) {
                const int dim0 = kc * 16 + (mi >> 1) * 8;
                const uint32_t addr = ring + s * kStage + (dim0 / BW) * kSub + swz<BW>(arow, (dim0 % BW) >> 3);
                uint32_t a0, a1, a2, a3;
                ldsm_x4(addr, a0, a1, a2, a3);
                if (kc & 1) mma_16816(acc1, a0, a1, a2, a3, bq[kc][0], bq[kc][1]);
                else mma_16816(acc0, a0, a1, a2, a3, bq[kc][0], bq[kc][1]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);

            // s = dot*scale (+ mask), rounded separately as ggml_soft_max_ext does
            auto score = [&](float dot, bool vis, float m) {
                return vis ? (masked ? __fadd_rn(__fmul_rn(dot, p.scale), m) : __fmul_rn(dot, p.scale)) : -INFINITY;
            };
            const float sa0 = score(acc0[0] + acc1[0], v0 && key0 <= lim_a, mk[0]);
            const float sb0 = score(acc0[1] + acc1[1], v0 && key0 <= lim_b, mk[1]);
            const float sa1 = score(acc0[2] + acc1[2], v1 && key1 <= lim_a, mk[2]);
            const float sb1 = score(acc0[3] + acc1[3], v1 && key1 <= lim_b, mk[3]);
            // a range of at most kSD tiles keeps its scores in the V phase's
            // staging ring (the same layout per tile): no global round trip
            float *Sw = (s_local ? sS + (i % kSD) * (kConsumers * 4) : Scta + (int64_t)i * kTileScores) + warp * 128;
            if (row_a < R) {
                if (v0) Sw[so_a] = sa0;
                if (v1) Sw[so_a + 2] = sa1;
                upd(ma, za, sa0, sa1);
            }
            if (row_b < R) {
                if (v0) Sw[so_b] = sb0;
                if (v1) Sw[so_b + 2] = sb1;
                upd(mb, zb, sb0, sb1);
            }
        }
    }

    // ======================= statistics =======================
    // (max, sum) per (segment, row): the 8 lanes of a row pair, then the 8 warps
    KV_STAMP(tid == 0, 3);   // warp 0's K loop done
    {
        const float m_s[2][2] = {{two ? ma0 : ma, two ? mb0 : mb}, {ma, mb}};
        const float z_s[2][2] = {{two ? za0 : za, two ? zb0 : zb}, {za, zb}};
#pragma unroll
        for (int sl = 0; sl < 2; sl++)
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const float m = aborted ? -INFINITY : m_s[sl][rr];
                float M = m;
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
                float z = (m == -INFINITY) ? 0.0f : z_s[sl][rr] * __expf(m - M);
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
                if (gq == 0) {
                    red_m[(sl * 8 + warp) * kRows + 2 * cq + rr] = M;
                    red_z[(sl * 8 + warp) * kRows + 2 * cq + rr] = z;
                }
            }
    }
    aborted = named_sync_or(1, kConsumers, aborted);
    // publish: one 16-byte slot per (CTA, segment, row) holding (max, sum), each
    // word tagged with this launch's epoch, so a reader needs no fence or ticket
    // -- a slot is valid once both tags match
    if (tid < 2 * kRows) {
        const int sl = tid / kRows, row = tid % kRows;
        float mw[8], zw[8];
#pragma unroll
        for (int w = 0; w < 8; w++) {
            mw[w] = red_m[(sl * 8 + w) * kRows + row];
            zw[w] = red_z[(sl * 8 + w) * kRows + row];
        }
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; w++) M = fmaxf(M, mw[w]);
        // the 8 warps' sums (F32: this slot is on the head's critical path;
        // the rounding is ~1e-7 of Z)
        float Z = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++)
            if (mw[w] != -INFINITY) Z = fmaf(zw[w], __expf(mw[w] - M), Z);
        // an aborted CTA publishes empty statistics, so no other CTA waits for it
        const float Mp = aborted ? -INFINITY : M, Zp = aborted ? 0.0f : (float)Z;
        if (clus) {
            // row `row` of rank crank: here with a plain store, into every
            // other rank counted on its statistics barrier
            if (sl == 0) {
                cst[crank * kRows + row] = make_float2(Mp, Zp);
                const uint32_t la = smem_addr(cst + crank * kRows + row), lb = smem_addr(&cbar[0]);
                for (int q = 0; q < p.cq; q++)
                    if (q != (int)crank) st_async_v2(mapa(la, (uint32_t)q), Mp, Zp, mapa(lb, (uint32_t)q));
            }
        } else {
            const unsigned long long tag = (unsigned long long)p.epoch << 32;
            st_volatile_v2(p.stats + 2 * (((int64_t)c * 2 + sl) * kRows + row), tag | __float_as_uint(Mp),
                           tag | __float_as_uint(Zp));
        }
    }
    // the leader's last store into another rank's shared memory is behind it;
    // this rank's own row is seen by the warps that combine the rows
    bool c_arrived = false;
    if (clus) {
        named_sync(1, kConsumers);
        if (crank == 0) {
            cluster_arrive();
            c_arrived = true;
        }
    }
    KV_STAMP(tid == 0, 4);   // statistics published
    // decode: the new V row of head h0 goes to the cache now, while others finish
    if (owns_new && warp == 7) {
        const float *src = p.v + (int64_t)(p.hkv0 + g.h0) * D;
        const float *bv = p.v_bias ? p.v_bias + (int64_t)(p.hkv0 + g.h0) * D : nullptr;
        __half *dst = p.vc + (p.n_past * (int64_t)p.hkv + g.h0) * D;
        for (int i = lane; i < D; i += 32) {
            const __half h16 = __float2half_rn(bv ? __fadd_rn(__ldg(src + i), __ldg(bv + i)) : __ldg(src + i));
            vnew[i] = h16;
            dst[i] = h16;
        }
    }

    // global max and 1/sum of each (segment, query row): warp w polls the slots
    // of row w of every CTA of its heads (all loads in flight at once; spans of
    // up to kPU*32 CTAs) until every tag shows this launch, bounded by limit_ns
    bool late = false;
    // cluster mode: the cluster's (max, sum) of row `warp` from its ranks' rows
    bool cdone = false;   // the cluster covers the whole head: statistics known
    if (clus && !aborted && warp < R) {
        const bool ok = mbar_wait(&cbar[0], 0, p.limit_ns);
        float mq = -INFINITY, zq = 0.0f;
        if (ok && lane < p.cq) {
            const float2 v = cst[lane * kRows + warp];
            mq = v.x;
            zq = v.y;
        }
        float M = mq;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float Z = mq == -INFINITY ? 0.0f : zq * __expf(mq - M);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) Z += __shfl_xor_sync(0xffffffffu, Z, o);
        if (!__all_sync(0xffffffffu, ok)) {
            late = true;
            if (lane == 0) {
                atomicOr(p.err, 4u);
                flags[0] = 1;
            }
        } else if (p.ncl == 1) {
            if (lane == 0) {
                rowM[warp] = M;
                rowInv[warp] = Z > 0.0f ? __fdiv_rn(1.0f, Z) : 0.0f;
            }
            cdone = true;
        } else if (crank == 0 && lane == 0) {
            // one slot per (cluster, row), tagged as the CTA slots
            const unsigned long long tag = (unsigned long long)p.epoch << 32;
            st_volatile_v2(p.stats + 2 * (((int64_t)(c / p.cq) * 2) * kRows + warp), tag | __float_as_uint(M),
                           tag | __float_as_uint(Z));
        }
    }
    if (!aborted && !late && !cdone) {
        constexpr int kPU = kMaxSpan / 32;
        float mm[2][kPU], zz[2][kPU];
        unsigned pend = 0u;
        int ca[2], cb[2];
#pragma unroll
        for (int sl = 0; sl < 2; sl++) {
            const int h = g.h0 + sl;
            const bool act = warp < R && (sl == 0 || two);
            // the parties: the head's CTAs, or its clusters in cluster mode
            ca[sl] = act ? (clus ? h * p.ncl : p.span_a[h]) : 0;
            cb[sl] = act ? (clus ? h * p.ncl + p.ncl - 1 : p.span_b[h]) : -1;
#pragma unroll
            for (int u = 0; u < kPU; u++) {
                mm[sl][u] = -INFINITY;
                zz[sl][u] = 0.0f;
                if (ca[sl] + lane + 32 * u <= cb[sl]) pend |= 1u << (sl * kPU + u);
            }
        }
        const unsigned ep = p.epoch;
        const uint64_t t_start = globaltimer();
        for (;;) {
            // every pending slot's load goes out before any is checked: one L2
            // round trip a poll, however many CTAs span the head
            unsigned long long w0[2][kPU], w1[2][kPU];
#pragma unroll
            for (int sl = 0; sl < 2; sl++)
#pragma unroll
                for (int u = 0; u < kPU; u++) {
                    w0[sl][u] = w1[sl][u] = 0ull;
                    if (pend & (1u << (sl * kPU + u))) {
                        const int cc = ca[sl] + lane + 32 * u;
                        const int64_t slot = clus ? (int64_t)cc * 2 : part_slot(p, g.h0 + sl, cc);
                        ld_volatile_v2(p.stats + 2 * (slot * kRows + warp), w0[sl][u], w1[sl][u]);
                    }
                }
#pragma unroll
            for (int sl = 0; sl < 2; sl++)
#pragma unroll
                for (int u = 0; u < kPU; u++) {
                    const unsigned bit = 1u << (sl * kPU + u);
                    if ((pend & bit) && (unsigned)(w0[sl][u] >> 32) == ep && (unsigned)(w1[sl][u] >> 32) == ep) {
                        mm[sl][u] = __uint_as_float((unsigned)w0[sl][u]);
                        zz[sl][u] = __uint_as_float((unsigned)w1[sl][u]);
                        pend &= ~bit;
                    }
                }
            if (!__any_sync(0xffffffffu, pend != 0u)) break;
            if (globaltimer() - t_start > p.limit_ns) {
                late = true;
                break;
            }
        }
        late = __any_sync(0xffffffffu, late);
        if (!late) {
#pragma unroll
            for (int sl = 0; sl < 2; sl++) {
                float M = -INFINITY;
#pragma unroll
                for (int u = 0; u < kPU; u++) M = fmaxf(M, mm[sl][u]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
                float Z = 0.0f;
#pragma unroll
                for (int u = 0; u < kPU; u++)
                    if (mm[sl][u] != -INFINITY) Z += zz[sl][u] * __expf(mm[sl][u] - M);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) Z += __shfl_xor_sync(0xffffffffu, Z, o);
                if (lane == 0) {
                    rowM[sl * kRows + warp] = M;
                    rowInv[sl * kRows + warp] = Z > 0.0f ? __fdiv_rn(1.0f, Z) : 0.0f;
                }
            }
        } else if (lane == 0) {
            atomicOr(p.err, 4u);
            flags[0] = 1;
        }
    }
    aborted = named_sync_or(1, kConsumers, aborted || late);
    KV_STAMP(tid == 0, 5);   // global statistics known

    // ======================= V phase =======================
    float oacc[DT][4];
#pragma unroll
    for (int dt = 0; dt < DT; dt++) oacc[dt][0] = oacc[dt][1] = oacc[dt][2] = oacc[dt][3] = 0.0f;

    // scores of tile i for this lane: one float4 of the warp's block, through a
    // kSD-deep per-thread cp.async ring
    const float *Sl = Scta + warp * 128 + (gq * 4 + cq) * 4;
    float *stg = sS + tid * 4;
    auto stage_s = [&](int i) {
        if (s_local) {   // already in place; an empty group keeps the wait counts
            cp_async_commit();
            return;
        }
        if (i < g.nt && gq < R) cp_async_16(stg + (i % kSD) * (kConsumers * 4), Sl + (int64_t)i * kTileScores);
        cp_async_commit();
    };
    if (!aborted)
        for (int i = 0; i < kSD - 1; i++) stage_s(i);

    // the head's final values into out and, with KV-head shards, into every
    // peer's receive buffer; the CTA that writes the shard's last local head
    // then collects the peers' heads.  value_of(idx, row, dd) gives element
    // idx = row * D + dd; each thread takes the idx it took in the sums before.
    auto emit_head = [&](int h, auto &&value_of) {
        const int par = (int)(p.epoch & 1u);
        for (int idx = tid; idx < R * D; idx += kConsumers) {
            const int row = idx / D, dd = idx - row * D;
            const float val = value_of(idx, row, dd);
            const int qrow = p.row0 + row;
            const int64_t o = (int64_t)(qrow / p.r) * p.out_stride + (int64_t)(p.out_head0 + h * p.r + qrow % p.r) * D + dd;
            p.out[o] = val;
            // KV-head shards: the same value, tagged with this launch, into
            // every peer's receive buffer (NVLink stores; no fence or flag:
            // the reader checks each word's tag)
            const unsigned long long word = ((unsigned long long)p.epoch << 32) | __float_as_uint(val);
            if (p.xpull) {
                if (p.n_peers > 1) p.rx[p.shard][par * p.rx_stride + o] = word;
            } else {
                for (int gg = 0; gg < p.n_peers; gg++)
                    if (gg != p.shard) p.rx[gg][par * p.rx_stride + o] = word;
            }
        }
        if (p.n_peers > 1) {
            named_sync(1, kConsumers);
            // count the head in; the CTA that converts the last local head
            // collects the peers' heads
            // (a shard of one KV head: its converter is the collector, no ticket)
            if (tid == 0) flags[3] = p.hkv == 1 || atomicAdd(p.xticket, 1u) == (unsigned)(p.hkv - 1);
            named_sync(1, kConsumers);
            if (flags[3]) {
                KV_STAMP(tid == 0, 8);   // collector starts polling the peers' words
                // every column outside this shard's, once its word carries
                // this launch's tag; a thread keeps up to kXW words' loads in
                // flight per poll
                const int cols = p.hkv * p.r * D;   // this shard's columns (every shard has as many)
                // push: the peers' words sit in this shard's buffer; pull: in
                // the buffer of the shard that owns the column
                auto word_at = [&](int o) -> const unsigned long long * {
                    return (p.xpull ? p.rx[o / cols] : p.rx[p.shard]) + par * p.rx_stride + o;
                };
                const int lo = p.out_head0 * D, all = p.n_peers * cols;
                const unsigned ep = p.epoch;
                bool xlate = false;
                const uint64_t t0 = globaltimer();
                // up to kXW words a thread in one batch: at 8 shards every peer
                // column of a 4-head group (3584 words) in one poll round trip
                constexpr int kXW = 16;
                for (int base = 0; base < all && !xlate; base += kXW * kConsumers) {
                    unsigned pend = 0u;
#pragma unroll
                    for (int u = 0; u < kXW; u++) {
                        const int o = base + u * kConsumers + tid;
                        if (o < all && (o < lo || o >= lo + cols)) pend |= 1u << u;
                    }
                    while (pend) {
                        unsigned long long w[kXW];
#pragma unroll
                        for (int u = 0; u < kXW; u++)   // all loads out before any is used
                            w[u] = (pend & (1u << u)) ? ld_volatile_u64(word_at(base + u * kConsumers + tid)) : 0ull;
#pragma unroll
                        for (int u = 0; u < kXW; u++)
                            if ((pend & (1u << u)) && (unsigned)(w[u] >> 32) == ep) {
                                p.out[base + u * kConsumers + tid] = __uint_as_float((unsigned)w[u]);
                                pend &= ~(1u << u);
                            }
                        if (pend && globaltimer() - t0 > p.limit_ns) {
                            xlate = true;
                            break;
                        }
                    }
                }
                if (named_sync_or(1, kConsumers, xlate) && tid == 0) atomicOr(p.err, 8u);
                KV_STAMP(tid == 0, 9);   // collector done
                if (tid == 0 && p.hkv > 1) *p.xticket = 0u;
            }
        }
    };

    // this CTA's partial output of segment sl: into the head's fixed-point
    // accumulator, whose last CTA converts and writes the output; in cluster
    // mode first into the cluster leader's shared memory, and the leader adds
    // the ranks' rows in rank order (the head's output when its one cluster
    // covers it, else the cluster's rows go to the accumulator)
    auto flush_out = [&](int sl) {
        if (named_sync_or(1, kConsumers, aborted)) {
            aborted = true;
            return;
        }
        const int h = g.h0 + sl;
#pragma unroll
        for (int dt = 0; dt < DT; dt++) {
            float *rw = red + (warp * kRows) * RED_LD + dt * 16 + gq;
            rw[(2 * cq) * RED_LD] = oacc[dt][0];
            rw[(2 * cq + 1) * RED_LD] = oacc[dt][1];
            rw[(2 * cq) * RED_LD + 8] = oacc[dt][2];
            rw[(2 * cq + 1) * RED_LD + 8] = oacc[dt][3];
            oacc[dt][0] = oacc[dt][1] = oacc[dt][2] = oacc[dt][3] = 0.0f;
        }
        named_sync(1, kConsumers);
        if (clus) {
            if (crank != 0) {
                // the rank's rows (the 8 warps' sum; flash: normalised) into
                // the leader, counted on its output barrier
                const uint32_t lb = mapa(smem_addr(&cbar[1]), 0u);
                for (int i4 = tid; i4 < R * D / 4; i4 += kConsumers) {
                    const int idx = i4 * 4, row = idx / D, dd = idx - row * D;
                    float4 v = *reinterpret_cast<const float4 *>(red + row * RED_LD + dd);
#pragma unroll
                    for (int w = 1; w < 8; w++) {
                        const float4 x = *reinterpret_cast<const float4 *>(red + (w * kRows + row) * RED_LD + dd);
                        v.x += x.x;
                        v.y += x.y;
                        v.z += x.z;
                        v.w += x.w;
                    }
                    if (flash) {
                        const float iz = rowInv[row];
                        v.x = __fmul_rn(v.x, iz);
                        v.y = __fmul_rn(v.y, iz);
                        v.z = __fmul_rn(v.z, iz);
                        v.w = __fmul_rn(v.w, iz);
                    }
                    st_async_v4(mapa(smem_addr(crecv + ((crank - 1) * kRows + row) * D + dd), 0u), v, lb);
                }
                // its last store into another rank is behind it
                __syncwarp();
                cluster_arrive();
                c_arrived = true;
                return;
            }
            const bool got = mbar_wait(&cbar[1], 0, p.limit_ns);
            if (named_sync_or(1, kConsumers, !got)) {
                if (tid == 0) {
                    atomicOr(p.err, 16u);
                    flags[0] = 1;
                }
                aborted = true;
                return;
            }
            // the cluster's rows, kept in warp 0's slot of each element (the
            // thread that sums an element is the one that reads it later)
            for (int idx = tid; idx < R * D; idx += kConsumers) {
                const int row = idx / D, dd = idx - row * D;
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < 8; w++) sum += red[(w * kRows + row) * RED_LD + dd];
                if (flash) sum = __fmul_rn(sum, rowInv[row]);
                for (int q = 1; q < p.cq; q++) sum += crecv[((q - 1) * kRows + row) * D + dd];
                red[row * RED_LD + dd] = sum;
            }
            if (p.ncl == 1) {
                KV_STAMP(tid == 0, 7);   // the cluster's rows summed
                emit_head(h, [&](int, int row, int dd) {
                    const float v = red[row * RED_LD + dd];
                    return isfinite(v) ? v : __int_as_float(0x7fc00000);
                });
                return;
            }
        }
        long long *acc = p.acc + (int64_t)h * kRows * D;
        unsigned bad = 0u;   // rows with a non-finite partial
        for (int idx = tid; idx < R * D; idx += kConsumers) {
            const int row = idx / D, dd = idx - row * D;
            float sum;
            if (clus) {
                sum = red[row * RED_LD + dd];
            } else {
                sum = 0.0f;
#pragma unroll
                for (int w = 0; w < 8; w++) sum += red[(w * kRows + row) * RED_LD + dd];
                if (flash) sum = __fmul_rn(sum, rowInv[sl * kRows + row]);   // flash: normalised here
            }
            if (isfinite(sum))
                atomicAdd(reinterpret_cast<unsigned long long *>(acc + idx),
                          (unsigned long long)__float2ll_rn(__fmul_rn(sum, kFix)));
            else
                bad |= 1u << row;
        }
        if (bad) atomicOr(&p.nonfin[h], bad);
        // the CTA's atomics, ordered by the barrier, are released by the ticket
        // (cumulativity); the last CTA's ticket acquires every other CTA's
        named_sync(1, kConsumers);
        if (tid == 0) {
            const unsigned parties = clus ? (unsigned)p.ncl : (unsigned)(p.span_b[h] - p.span_a[h] + 1);
            flags[1 + sl] = atom_add_acq_rel_gpu(&p.counters[h], 1u) == parties - 1u;
        }
        named_sync(1, kConsumers);
        KV_STAMP(tid == 0, 7);   // partial added, ticket taken
        if (flags[1 + sl]) {
            const unsigned nan_rows = __ldcg(&p.nonfin[h]);
            emit_head(h, [&](int idx, int row, int) {
                const long long v = __ldcg(acc + idx);
                acc[idx] = 0;
                return (nan_rows >> row) & 1u ? __int_as_float(0x7fc00000) : __fmul_rn(__ll2float_rn(v), kUnfix);
            });
            if (tid == 0) {
                p.counters[h] = 0u;
                p.nonfin[h] = 0u;
            }
        }
    };

    for (int i = 0; i < g.nt; i++) {
        if (i == g.nt0 && i > 0) flush_out(0);
        if (aborted) continue;   // keep step with the other warps' barriers
        const int j = g.nt + i, s = j % NS;
        stage_s(i + kSD - 1);
        const bool ok = mbar_wait(&full[s], (j / NS) & 1, p.limit_ns);
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) {
                atomicOr(p.err, 1u);
                flags[0] = 1;
            }
            aborted = true;
            continue;
        }
        int h;
        int64_t k0, kend;
        tile_of(g, i, h, k0, kend);
        const int sl = i < g.nt0 ? 0 : 1;
        const int n_valid = (int)min((int64_t)kTK, kend - k0);
        const int kw = warp * 16;
        unsigned char *stage = smem + s * kStage;

        if (kw + 16 > n_valid) {   // rows past the valid keys: zero, so 0 * stale never reaches the sum
            const int zr0 = max(kw, n_valid);
            constexpr int CPR = BW / 8;
            for (int idx = lane; idx < (kw + 16 - zr0) * NB * CPR; idx += 32) {
                const int rr = zr0 + idx / (NB * CPR), rest = idx % (NB * CPR);
                *reinterpret_cast<uint4 *>(stage + (rest / CPR) * kSub + (BW == 64 ? rr * 128 : rr * 64) +
                                           (rest % CPR) * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
        }
        if (i == it_new && (int)((p.n_past - k0) >> 4) == warp) patch_row<D, BW>(stage, (int)(p.n_past - k0), vnew);

        cp_async_wait<kSD - 1>();
        const float4 sv = *reinterpret_cast<const float4 *>(stg + (i % kSD) * (kConsumers * 4));
        const float sc[4] = {sv.x, sv.y, sv.z, sv.w};
        const float M = rowM[sl * kRows + gq], inv = rowInv[sl * kRows + gq];
        __half pv[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int kk = kw + 2 * cq + (e & 1) + 8 * (e >> 1);
            const bool valid = gq < R && kk < n_valid;
            // default branch: F16(exp(s - M) * (1/Z)), ggml's rounding of the
            // normalised weight; flash branch: F16(exp(s - M)), scaled by 1/Z at
            // the output, and 0 for a row without a visible key
            const float pe = flash ? (M == -INFINITY ? 0.0f : expf(sc[e] - M)) : __fmul_rn(expf(sc[e] - M), inv);
            pv[e] = valid ? __float2half_rn(pe) : __ushort_as_half((unsigned short)0);
        }
        const uint32_t b0 = pack_half2(pv[0], pv[1]), b1 = pack_half2(pv[2], pv[3]);

        const int mi = lane >> 3;
        const int krow = kw + (lane & 7) + (mi >> 1) * 8;
#pragma unroll
        for (int dt = 0; dt < DT; dt++) {
            const int dim0 = dt * 16 + (mi & 1) * 8;
            const uint32_t addr = ring + s * kStage + (dim0 / BW) * kSub + swz<BW>(krow, (dim0 % BW) >> 3);
            uint32_t a0, a1, a2, a3;
            ldsm_x4_t(addr, a0, a1, a2, a3);
            mma_16816(oacc[dt], a0, a1, a2, a3, b0, b1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    cp_async_wait<0>();
    KV_STAMP(tid == 0, 6);   // warp 0's V loop done
    flush_out(two ? 1 : 0);
    // every consumer has read its scores (flush_out opens with a barrier): the
    // scratch is dead until the next launch rewrites it, so it leaves L2
    // without a write-back (dropping it before the output's atomics instead
    // measured 1.3 % slower on config 2: the drops queue with the atomics)
    if (!s_local)
        for (int ln = tid; ln < g.nt * (kTileScores / 32); ln += kConsumers) l2_discard(Scta + ln * 32);
    named_sync(2, kThreads);
    KV_STAMP(tid == 0, 12);   // exit
    if (clus) {
        // no rank leaves while another may still store into its shared
        // memory: every transaction counted here has landed, and every thread
        // of the cluster is past its last store into another rank
        __syncwarp();
        if (!c_arrived) cluster_arrive();
        if (tid == 0) {
            mbar_wait(&cbar[0], 0, p.limit_ns);
            if (crank == 0) mbar_wait(&cbar[1], 0, p.limit_ns);
        }
        __syncwarp();
        cluster_wait();
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int D, bool CL>
cudaError_t prep_cl()
{
    const int b = (int)Smem<D>::bytes;
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<D, false, false, CL>, cudaFuncAttributeMaxDynamicSharedMemorySize, b);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_decode_kernel<D, false, true, CL>, cudaFuncAttributeMaxDynamicSharedMemorySize, b);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_decode_kernel<D, true, false, CL>, cudaFuncAttributeMaxDynamicSharedMemorySize, b);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_decode_kernel<D, true, true, CL>, cudaFuncAttributeMaxDynamicSharedMemorySize, b);
    return e;
}

template <int D>
cudaError_t prep()
{
    cudaError_t e = prep_cl<D, false>();
    if (e == cudaSuccess && Smem<D>::kMaxQ > 1) e = prep_cl<D, Smem<D>::kMaxQ != 1>();
    return e;
}

template <int D>
cudaError_t occupancy(int *blocks)
{
    // the fewest resident CTAs an SM takes among the four instances
    int b[4] = {0, 0, 0, 0};
    const size_t sm = Smem<D>::bytes;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b[0], attn_decode_kernel<D, false, false, false>, kThreads, sm);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b[1], attn_decode_kernel<D, false, true, false>, kThreads, sm);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b[2], attn_decode_kernel<D, true, false, false>, kThreads, sm);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b[3], attn_decode_kernel<D, true, true, false>, kThreads, sm);
    *blocks = std::min(std::min(b[0], b[1]), std::min(b[2], b[3]));
    return e;
}

template <int D>
cudaError_t launch(const CUtensorMap &kmap, const CUtensorMap &vmap, const AttnParams &p, cudaStream_t st, bool pdl,
                   bool coop)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)p.n_cta);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Smem<D>::bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[3];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (coop) {
        attr[na].id = cudaLaunchAttributeCooperative;
        attr[na].val.cooperative = 1;
        na++;
    }
    if (p.cq > 1) {
        if (Smem<D>::kMaxQ < p.cq || p.n_cta % p.cq) return cudaErrorInvalidValue;
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)p.cq;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    const bool m = p.mask || p.all_keys;
    if (p.cq > 1) {
        constexpr bool C = Smem<D>::kMaxQ > 1;   // (the launch was refused above otherwise)
        if (m && p.flash) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, true, true, C>, kmap, vmap, p);
        if (m) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, true, false, C>, kmap, vmap, p);
        if (p.flash) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, false, true, C>, kmap, vmap, p);
        return cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, false, false, C>, kmap, vmap, p);
    }
    if (m && p.flash) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, true, true, false>, kmap, vmap, p);
    if (m) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, true, false, false>, kmap, vmap, p);
    if (p.flash) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, false, true, false>, kmap, vmap, p);
    return cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, false, false, false>, kmap, vmap, p);
}

}  // namespace

int attn_rows() { return kRows; }
int attn_tile_keys() { return kTK; }
int attn_box_width(int D) { return D == 96 ? 32 : 64; }
int attn_tile_scores() { return kTileScores; }
int attn_max_ctas() { return kMaxSpan; }

cudaError_t attn_prepare(int D)
{
    switch (D) {
    case 64: return prep<64>();
    case 96: return prep<96>();
    case 128: return prep<128>();
    case 256: return prep<256>();
    default: return cudaErrorInvalidValue;
    }
}

template <int D>
cudaError_t cluster_occupancy(int q, int *clusters)
{
    *clusters = 0;
    if (Smem<D>::kMaxQ < q) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(q * 32));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Smem<D>::bytes;
    cudaLaunchAttribute a[1];
    a[0].id = cudaLaunchAttributeClusterDimension;
    a[0].val.clusterDim.x = (unsigned)q;
    a[0].val.clusterDim.y = 1;
    a[0].val.clusterDim.z = 1;
    cfg.attrs = a;
    cfg.numAttrs = 1;
    int n[4] = {0, 0, 0, 0};
    cudaError_t e = cudaOccupancyMaxActiveClusters(&n[0], attn_decode_kernel<D, false, false, true>, &cfg);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n[1], attn_decode_kernel<D, false, true, true>, &cfg);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n[2], attn_decode_kernel<D, true, false, true>, &cfg);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n[3], attn_decode_kernel<D, true, true, true>, &cfg);
    if (e == cudaSuccess) *clusters = std::min(std::min(n[0], n[1]), std::min(n[2], n[3]));
    return e;
}

cudaError_t attn_cluster_occupancy(int D, int q, int *clusters)
{
    switch (D) {
    case 64: return cluster_occupancy<64>(q, clusters);
    case 96: return cluster_occupancy<96>(q, clusters);
    case 128: return cluster_occupancy<128>(q, clusters);
    default: *clusters = 0; return cudaSuccess;
    }
}

cudaError_t attn_occupancy(int D, int *blocks_per_sm)
{
    switch (D) {
    case 64: return occupancy<64>(blocks_per_sm);
    case 96: return occupancy<96>(blocks_per_sm);
    case 128: return occupancy<128>(blocks_per_sm);
    case 256: return occupancy<256>(blocks_per_sm);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_attn(int D, const CUtensorMap &kmap, const CUtensorMap &vmap, const AttnParams &p,
                        cudaStream_t st, bool pdl, bool coop)
{
    if (p.nrows < 1 || p.nrows > kRows) return cudaErrorInvalidValue;
    switch (D) {
    case 64: return launch<64>(kmap, vmap, p, st, pdl, coop);
    case 96: return launch<96>(kmap, vmap, p, st, pdl, coop);
    case 128: return launch<128>(kmap, vmap, p, st, pdl, coop);
    case 256: return launch<256>(kmap, vmap, p, st, pdl, coop);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace kvb
