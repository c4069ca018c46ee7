// kv_prefill.cu -- attention of a multi-token chunk (prefill) on the 5th-
// generation tensor cores: tcgen05.mma with TMEM accumulators, operands staged
// in shared memory by TMA.
//
// What it computes: the reference's attention branch (src/model.cpp:1416-1445)
// for n_new query tokens: S = F16(q) . K (F32 accumulation), causal mask (key <=
// n_past + token), scale, softmax over the keys, O = P . V with the weights P
// rounded to F16 (ggml converts the mul_mat operand to the F16 vec-dot type).
//
// How: one pass over the keys with an online softmax.  Per query row the kernel
// keeps a running maximum m (log2 units: s * log2 e), the F32 sum l of
// 2^(s*log2e - m) and O = sum F16(2^(s*log2e - m)) . V in TMEM; the output is
// O / l.  ggml rounds the normalised weight exp(s - M) / Z to F16 instead; the
// two roundings differ by at most one F16 ulp of each weight (2^-11 relative),
// far inside the attention tolerance.  m is raised lazily: only when a tile's
// maximum exceeds it by more than 2^8 are l and the row of O rescaled, so the
// weights stay <= 256 (exact range of F16) and O is rarely read back.  exp is
// 2^x on the SFU (ex2.approx, a few F32 ulps from expf).
//
// Work: query rows are packed GQA-group-major: a 128-row tile holds tb =
// floor(128 / r) tokens x the r query heads of one KV head (row = token*r +
// head), and a CTA holds two such tiles, A and B (2*tb consecutive tokens), so
// a K/V tile staged once feeds four MMAs.  At head_dim 256 a CTA holds one
// tile (PL<256>::NT): O takes 256 TMEM columns and a K or V tile 64 KB.  A "pair" is (KV head, block of 2*tb
// tokens); its keys are the tiles of 128 keys up to the block's last visible
// key.  The pairs' tiles, laid end to end, are cut into C equal ranges (one CTA
// each, C <= SMs); a range holds one or more "segments" (the part of one pair
// it covers).  A pair that one segment covers is written to the output by the
// kernel; otherwise each segment leaves its (m, l, O) rows in scratch and
// prefill_out_fold merges them (weights 2^(m_i - max m), CTAs in order).
//
// prefill_kernel<D> (384 threads):
//   warp 0     TMA: the pair's two Q tiles, then K and V tiles into mbarrier rings
//   warps 1,10,11  MMA issuers (one thread each; warp 1 also owns TMEM), in
//              sub-tiles of 64 keys (half a K/V tile).  TMEM columns: two S
//              buffers per query tile (64 F32 columns each; P, F16 pairs,
//              overwrites the first 32 columns of its S), then O_A, O_B (D
//              each).  Warp 1 issues S_A, warp 10 S_B -- sub-tile i+2 into the
//              buffer of i once PV(i) has read its P (barrier o_ready), so the
//              tensor cores compute S two sub-tiles ahead of the softmax --
//              and warp 11 issues PV_A(i), PV_B(i) as the softmax reports P.
//              One thread's tcgen05.mma issue rate, not the tensor cores, bounds
//              these narrow MMAs, hence three issuers
//   warps 2-5  softmax of tile A, warps 6-9 of tile B: one query row per thread,
//              a sub-tile's 64 keys read with tcgen05.ld; P written back with
//              tcgen05.st; the rare O rescale (after the previous P . V, which
//              o_ready reports); at a segment's end O out
// prefill_out_fold   merges the segments of pairs split over CTAs
// With the caller's additive mask (kv_attend_mask) every pair covers all keys,
// the mask is added to each score (acc + mask/scale, so s*log2e = acc*cs +
// mask*log2e) and the causal bound is not applied; the flash-attn branch runs
// the one-pass mode at any length and gives 0 for a row without a visible key
// (the default branch: NaN, as ggml's soft_max of an all -inf row).
// Every wait is bounded (limit_ns) and gives up when the CTA's abort flag is
// set; the CTA drains its TMA loads and MMAs and frees TMEM before leaving.
#include <math.h>

#include "kv_internal.h"
#include "kv_sm100.cuh"

namespace kvb {
namespace {

using namespace sm100;

constexpr int kGW = 4;                         // softmax warps per query tile
constexpr int kPThreads = 32 * (4 + 2 * kGW);  // TMA warp, three MMA issuers, two softmax groups
constexpr uint32_t kBox = 128 * 128;           // one [128 rows][64 halves] swizzled box
constexpr uint32_t kTmO = 256;                 // TMEM column of O_A (O_B follows at +D)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazy = 8.0f;                  // raise m only past 2^8 growth
// kernel modes: one pass (online softmax), or the exact two passes for long
// contexts: statistics (S, row max and sum), then output (ggml's normalised p)
constexpr int kOnePass = 0, kStats = 1, kExact = 2;

template <int D>
struct PL {
    // query tiles a CTA holds: two (A, B) up to head_dim 128; one at 256, where
    // O takes 256 TMEM columns and a 128-key K or V tile 64 KB of shared memory
    static constexpr int NT = D == 256 ? 1 : 2;
    static constexpr int NB = D / 64;                        // boxes per Q/K/V row
    static constexpr uint32_t kTile = (uint32_t)NB * kBox;   // 128 rows x D halves
    static constexpr int KS = D == 256 ? 1 : D == 128 ? 3 : 6;   // K ring
    static constexpr int VS = D == 256 ? 1 : D == 128 ? 2 : 5;   // V ring
    static constexpr size_t o_q = 0;                         // Q tiles A (, B)
    static constexpr size_t o_k = o_q + NT * (size_t)kTile;
    static constexpr size_t o_v = o_k + (size_t)KS * kTile;
    static constexpr size_t o_bar = o_v + (size_t)VS * kTile;
    // q_full, q_empty, k_full[KS], k_empty[KS], v_full[VS], v_empty[VS],
    // s_full[2][2], p_full[2][2], o_ready[2][2], o_full, o_empty, drain[3]
    static constexpr int NBAR = 2 + 2 * KS + 2 * VS + 12 + 5;
    static constexpr size_t o_tm = o_bar + (size_t)NBAR * 8;
    static constexpr size_t o_flags = o_tm + 16;
    static constexpr size_t bytes = o_flags + 16;
    static_assert(bytes <= 227 * 1024, "shared memory of the prefill kernel");
};

// ---- the caller's mask -----------------------------------------------------------
// v[e] (raw dots of keys kb + e, e < nvis) += mask[tok][kb + e] / scale; 16-byte
// loads when the rows allow them (mask_vec), else one element at a time
__device__ __forceinline__ void add_mask(const PrefillParams &p, int tok, int64_t kb, int nvis, float mscl,
                                         uint32_t (&v)[64])
{
    const int64_t base = (int64_t)tok * p.mask_stride + kb;
    if (p.mask_vec && nvis == 64) {
        if (p.mask_f16) {
            const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const __half *>(p.mask) + base);
            uint4 u[8];
#pragma unroll
            for (int q = 0; q < 8; q++) u[q] = __ldg(src + q);
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const uint32_t w4[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w4[t]));
                    v[8 * q + 2 * t] = __float_as_uint(fmaf(f.x, mscl, __uint_as_float(v[8 * q + 2 * t])));
                    v[8 * q + 2 * t + 1] = __float_as_uint(fmaf(f.y, mscl, __uint_as_float(v[8 * q + 2 * t + 1])));
                }
            }
        } else {
            const float4 *src = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p.mask) + base);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float4 f[8];
#pragma unroll
                for (int q = 0; q < 8; q++) f[q] = __ldg(src + 8 * h + q);
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const int e = 32 * h + 4 * q;
                    v[e] = __float_as_uint(fmaf(f[q].x, mscl, __uint_as_float(v[e])));
                    v[e + 1] = __float_as_uint(fmaf(f[q].y, mscl, __uint_as_float(v[e + 1])));
                    v[e + 2] = __float_as_uint(fmaf(f[q].z, mscl, __uint_as_float(v[e + 2])));
                    v[e + 3] = __float_as_uint(fmaf(f[q].w, mscl, __uint_as_float(v[e + 3])));
                }
            }
        }
        return;
    }
#pragma unroll
    for (int e = 0; e < 64; e++)
        if (e < nvis) {
            const float m = p.mask_f16 ? __half2float(__ldg(reinterpret_cast<const __half *>(p.mask) + base + e))
                                       : __ldg(reinterpret_cast<const float *>(p.mask) + base + e);
            v[e] = __float_as_uint(fmaf(m, mscl, __uint_as_float(v[e])));
        }
}

// output scale of a row without a visible key: 0 in the flash-attn branch,
// NaN in the default one (ggml's soft_max of an all -inf row)
__device__ __forceinline__ float no_key_scale(const PrefillParams &p)
{
    return p.flash ? 0.0f : __int_as_float(0x7fc00000);
}

// ---- the work split ------------------------------------------------------------
// key tiles of block b (tokens [nt*b*tb, nt*(b+1)*tb), nt the query tiles a CTA holds)
__device__ __forceinline__ int nt_of(const PrefillParams &p, int b)
{
    // keys [0, last): the causal bound of the block's last token, or all keys with a mask
    const int64_t last = p.n_past + (p.mask ? (int64_t)p.n_new
                                            : min((int64_t)p.n_new, (int64_t)(p.nt * (b + 1)) * p.tb));
    return (int)((last + 127) / 128);
}

__device__ __forceinline__ int64_t pair_start(const PrefillParams &p, int pair)
{
    const int kvh = pair / p.nblk, b = pair % p.nblk;
    int64_t x = (int64_t)kvh * p.s_all;
    for (int bb = 0; bb < b; bb++) x += nt_of(p, bb);
    return x;
}

// pair holding flattened tile x
__device__ __forceinline__ int pair_of(const PrefillParams &p, int64_t x)
{
    const int kvh = (int)(x / p.s_all);
    int64_t rem = x - (int64_t)kvh * p.s_all;
    int b = 0;
    for (; b < p.nblk - 1; b++) {
        const int n = nt_of(p, b);
        if (rem < n) break;
        rem -= n;
    }
    return kvh * p.nblk + b;
}

__device__ __forceinline__ int64_t cta_lo(const PrefillParams &p, int c)
{
    return (int64_t)c * ((int64_t)p.hkv * p.s_all) / p.n_cta;
}

// segment k of CTA c: pair, its tiles [t0, t1)
struct Seg {
    int pair, t0, t1;
};

template <class F>
__device__ __forceinline__ void for_segments(const PrefillParams &p, int c, F &&f)
{
    int64_t x = cta_lo(p, c);
    const int64_t hi = cta_lo(p, c + 1);
    int k = 0;
    while (x < hi && k < p.kseg) {
        Seg s;
        s.pair = pair_of(p, x);
        const int64_t ps = pair_start(p, s.pair);
        const int64_t pe = ps + nt_of(p, s.pair % p.nblk);
        const int64_t e = min(hi, pe);
        s.t0 = (int)(x - ps);
        s.t1 = (int)(e - ps);
        if (!f(k, s)) return;
        x = e;
        k++;
    }
}

__device__ __forceinline__ void give_up(const PrefillParams &p, volatile int *flags, unsigned bit)
{
    if (!flags[0]) {
        atomicOr(p.err, bit);
        flags[0] = 1;
    }
}

// CTAs [ca, cb] hold pair `pair`
__device__ __forceinline__ void pair_ctas(const PrefillParams &p, int pair, int &ca, int &cb)
{
    const int64_t W = (int64_t)p.hkv * p.s_all;
    const int64_t x0 = pair_start(p, pair), x1 = x0 + nt_of(p, pair % p.nblk) - 1;
    // the CTA holding tile x: the largest c with floor(c W / C) <= x
    auto cta_of = [&](int64_t x) { return (int)(((x + 1) * p.n_cta - 1) / W); };
    ca = cta_of(x0);
    cb = cta_of(x1);
}

// ---------------------------------------------------------------------------
// softmax arithmetic: three-input max and packed F32 pairs (sm_100)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float max3(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ uint64_t pk2(float lo, float hi)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ float2 up2(uint64_t v)
{
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}

// (a.x*b.x + c.x, a.y*b.y + c.y), each rounded once
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// 12 warps put 3 on each of the SM's four 16K-register quarters: at most 168
// registers a thread
template <int D, int MODE, bool MASKED>
__global__ void __launch_bounds__(kPThreads, 1) prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                 const __grid_constant__ CUtensorMap kmap,
                                                                 const __grid_constant__ CUtensorMap vmap,
                                                                 const PrefillParams p)
{
    using L = PL<D>;
    constexpr int NB = L::NB, KS = L::KS, VS = L::VS;
    constexpr uint32_t kTile = L::kTile;
    constexpr int NT = L::NT;
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L::o_bar);
    uint64_t *q_full = bar, *q_empty = bar + 1;
    uint64_t *k_full = bar + 2, *k_empty = k_full + KS;
    uint64_t *v_full = k_empty + KS, *v_empty = v_full + VS;
    uint64_t *s_full = v_empty + VS;   // [tile g][buffer]: S_g of a sub-tile is in TMEM
    uint64_t *p_full = s_full + 4;     // [tile g][buffer]: P_g of a sub-tile is in TMEM
    uint64_t *o_ready = p_full + 4;    // [tile g][buffer]: the P_g . V of a sub-tile has completed
    uint64_t *o_full = o_ready + 4, *o_empty = o_full + 1;
    uint64_t *drain = o_empty + 1;     // [issuer]
    uint32_t *tm_slot = reinterpret_cast<uint32_t *>(smem + L::o_tm);
    volatile int *flags = reinterpret_cast<volatile int *>(smem + L::o_flags);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, c = blockIdx.x;
    int issued_q = 0, issued_k = 0, issued_v = 0;   // TMA loads issued (warp 0, lane 0)

    if (tid == 0) {
        for (int i = 0; i < L::NBAR; i++) {
            // a softmax group's warps arrive on its p_full, both groups' on
            // o_empty; both S issuers commit to k_empty and q_empty
            const uint64_t *bi = &bar[i];
            const bool two = bi == q_empty || (bi >= k_empty && bi < k_empty + KS);
            mbar_init(&bar[i], (bi >= p_full && bi < p_full + 4) ? kGW : bi == o_empty ? NT * kGW : two ? NT : 1);
        }
        flags[0] = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tm_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tm_slot;
    // launched programmatically: the set-up above overlapped the previous
    // kernel (the append that wrote the Q tiles and the new K/V rows)
    pdl_wait();
    pdl_launch_dependents();   // the fold may start its set-up (it waits for this grid)

    if (warp == 0) {
        // ================= TMA =================
        if (lane == 0) {
            prefetch_tmap(&qmap);
            prefetch_tmap(&kmap);
            if (MODE != kStats) prefetch_tmap(&vmap);
            const uint32_t qbytes = (uint32_t)(p.r * p.tb) * 128u * NB;   // one Q tile (zero fill counts)
            for_segments(p, c, [&](int k, const Seg &sg) {
                const int kvh = sg.pair / p.nblk, b = sg.pair % p.nblk;
                if (k > 0 && !mbar_wait_ab(q_empty, (k - 1) & 1, p.limit_ns, flags)) {
                    give_up(p, flags, 2u);
                    return false;
                }
                mbar_arrive_expect_tx(q_full, NT * qbytes);
#pragma unroll
                for (int g = 0; g < NT; g++)
#pragma unroll
                    for (int bx = 0; bx < NB; bx++)
                        tma_load_3d(smem + L::o_q + g * kTile + bx * kBox, &qmap, q_full, bx * 64, kvh * p.r,
                                    (NT * b + g) * p.tb);
                issued_q++;
                for (int t = sg.t0; t < sg.t1; t++) {
                    const int s = issued_k % KS;
                    if (issued_k >= KS && !mbar_wait_ab(&k_empty[s], ((issued_k / KS) - 1) & 1, p.limit_ns, flags)) {
                        give_up(p, flags, 2u);
                        return false;
                    }
                    mbar_arrive_expect_tx(&k_full[s], kTile);
#pragma unroll
                    for (int bx = 0; bx < NB; bx++)
                        tma_load_3d(smem + L::o_k + s * kTile + bx * kBox, &kmap, &k_full[s], bx * 64, kvh, t * 128);
                    issued_k++;
                    if constexpr (MODE != kStats) {
                        const int sv = issued_v % VS;
                        if (issued_v >= VS &&
                            !mbar_wait_ab(&v_empty[sv], ((issued_v / VS) - 1) & 1, p.limit_ns, flags)) {
                            give_up(p, flags, 2u);
                            return false;
                        }
                        mbar_arrive_expect_tx(&v_full[sv], kTile);
#pragma unroll
                        for (int bx = 0; bx < NB; bx++)
                            tma_load_3d(smem + L::o_v + sv * kTile + bx * kBox, &vmap, &v_full[sv], bx * 64, kvh,
                                        t * 128);
                        issued_v++;
                    }
                }
                return true;
            });
        }
    } else if (warp == 1 || warp >= 2 + 2 * kGW) {
        // ================= MMA issue =================
        // Sub-tile i = 64 keys (half of K/V tile i/2; i counts across
        // segments), S buffer i&1.  Three issuing warps, since one thread's
        // tcgen05.mma issue, not the tensor cores, limits narrow MMAs:
        //   S issuer of tile g (warps 1, 10): S_g(i) once PV_g(i-2) has read
        //     the buffer's P (o_ready) -- so S runs two sub-tiles ahead
        //   PV issuer (warp 11): PV_A(i), PV_B(i) once the softmax reports P
        const int role = warp == 1 ? 0 : warp - (1 + 2 * kGW);   // 0: S_A, 1: S_B, 2: PV
        if (lane == 0) {
            constexpr uint32_t idS = idesc_f16_f32(128, 64, false);
            constexpr uint32_t idO = idesc_f16_f32(128, D, true);
            const uint32_t sq = smem_addr(smem + L::o_q), sk = smem_addr(smem + L::o_k);
            const uint32_t sv = smem_addr(smem + L::o_v);
            bool ok = true;
            auto wt = [&](uint64_t *b, uint32_t par) {
                if (ok && !mbar_wait_ab(b, par, p.limit_ns, flags)) {
                    give_up(p, flags, 1u);
                    ok = false;
                }
                return ok;
            };
            int i = 0;   // sub-tiles consumed
            if (role < NT) {
                const int g = role;
                for_segments(p, c, [&](int k, const Seg &sg) {
                    const int i1 = i + 2 * (sg.t1 - sg.t0);
                    if (!wt(q_full, k & 1)) return false;
                    for (; i < i1; i++) {
                        const int tile = i >> 1;
                        if (!(i & 1) && !wt(&k_full[tile % KS], (tile / KS) & 1)) return false;
                        // the buffer is free once PV_g(i-2) has read its P (the
                        // statistics pass: once the softmax has read S_g(i-2))
                        if (i >= 2 && !wt(MODE == kStats ? &p_full[g * 2 + (i & 1)] : &o_ready[g * 2 + (i & 1)],
                                          ((i - 2) >> 1) & 1))
                            return false;
                        tc_fence_after();
                        // S_g(i) = Q_g . K(64 of the tile's 128 rows)^T
                        const uint32_t kt = sk + (tile % KS) * kTile + (i & 1) * 8192;
#pragma unroll
                        for (int kk = 0; kk < D / 16; kk++) {
                            const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
                            umma_ss(tmem + g * 128 + (i & 1) * 64, sdesc_k_sw128(sq + g * kTile + off),
                                    sdesc_k_sw128(kt + off), idS, kk > 0);
                        }
                        umma_commit(&s_full[g * 2 + (i & 1)]);
                        if (i & 1) umma_commit(&k_empty[tile % KS]);   // both halves of the K tile read
                        if (i == i1 - 1) umma_commit(q_empty);
                    }
                    return true;
                });
            } else if (role == 2 && MODE != kStats) {
                for_segments(p, c, [&](int k, const Seg &sg) {
                    const int i0 = i, i1 = i + 2 * (sg.t1 - sg.t0);
                    for (; i < i1; i++) {
                        const int tile = i >> 1;
#pragma unroll
                        for (int g = 0; g < NT; g++) {
                            if (!wt(&p_full[g * 2 + (i & 1)], (i >> 1) & 1)) return false;
                            if (g == 0 && !(i & 1) && !wt(&v_full[tile % VS], (tile / VS) & 1)) return false;
                            if (g == 0 && i == i0 && k > 0 && !wt(o_empty, (k - 1) & 1)) return false;
                            tc_fence_after();
                            // O_g (+)= P_g(i) . V(64 of the tile's 128 rows)
                            const uint32_t vt = sv + (tile % VS) * kTile + (i & 1) * 8192;
#pragma unroll
                            for (int kk = 0; kk < 4; kk++) {   // 16 keys per step: 8 packed P columns
                                const uint64_t bd = sdesc_mn_sw128(vt + kk * 2048, kBox);
                                umma_ts(tmem + kTmO + g * D, tmem + g * 128 + (i & 1) * 64 + kk * 8, bd, idO,
                                        !(i == i0 && kk == 0));
                            }
                            umma_commit(&o_ready[g * 2 + (i & 1)]);
                        }
                        if (i & 1) umma_commit(&v_empty[tile % VS]);   // both halves of the V tile read
                        if (i == i1 - 1) umma_commit(o_full);
                    }
                    return true;
                });
            }
            // every MMA this thread issued has completed before TMEM is freed
            umma_commit(&drain[role]);
            mbar_wait(&drain[role], 0, p.limit_ns);
        }
    } else {
        // ================= softmax / epilogue =================
        // group grp (0: tile A, 1: tile B) of kGW warps; warp w reaches TMEM
        // lanes 32*(w%4) .. +31, one query row per thread, 64 keys a sub-tile
        const int grp = (warp - 2) / kGW;
        if (grp < NT) {   // (one query tile at head_dim 256: group B is idle)
        const int q4 = warp & 3;
        const int row = q4 * 32 + lane;           // query row of the tile = token*r + head
        const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
        const uint32_t tS = trow + grp * 128, tO = trow + kTmO + grp * D;
        const int tok_in = row / p.r, hd = row - tok_in * p.r;
        const bool row_ok = tok_in < p.tb;
        const float cs = p.scale * kLog2e;        // s * log2 e = acc * cs
        const uint64_t cs2 = pk2(cs, cs);
        int i = 0;
        for_segments(p, c, [&](int k, const Seg &sg) {
            const int b = sg.pair % p.nblk, kvh = sg.pair / p.nblk;
            const int tok = (NT * b + grp) * p.tb + tok_in;
            const bool valid = row_ok && tok < p.n_new;
            const int64_t lim = !valid ? -1 : p.mask ? p.n_past + p.n_new - 1 : p.n_past + tok;   // last visible key
            const float mscl = p.mask ? __fdiv_rn(1.0f, p.scale) : 0.0f;   // mask / scale adds to the raw dot
            const int i0 = i, i1 = i + 2 * (sg.t1 - sg.t0);
            float m = -INFINITY, l = 0.0f;   // one pass: running max (log2 units), sum; statistics: raw max, sum
            float nMx = 0.0f, inv = 0.0f;     // exact pass: -M * log2 e and 1/Z of the row
            if constexpr (MODE == kExact) {
                if (valid) {
                    const float2 st = p.rstat[(int64_t)sg.pair * 256 + grp * 128 + row];
                    nMx = -st.x * kLog2e;
                    inv = st.y;
                }
            }
            for (; i < i1; i++) {
                const int bf = i & 1;
                if (!mbar_wait_ab(&s_full[grp * 2 + bf], (i >> 1) & 1, p.limit_ns, flags)) {
                    give_up(p, flags, 1u);
                    return false;
                }
                tc_fence_after();
                uint32_t v[64];
                tmem_ld32(tS + bf * 64, *reinterpret_cast<uint32_t(*)[32]>(v));
                tmem_ld32(tS + bf * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
                tmem_wait_ld();
                if constexpr (MODE == kStats) {   // S is in registers: the buffer may be refilled
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&p_full[grp * 2 + bf]);
                }
                const int64_t kb = (int64_t)(2 * sg.t0 + (i - i0)) * 64;   // first key of the sub-tile
                const int nvis = (int)max((int64_t)0, min((int64_t)64, lim - kb + 1));
                const bool full = __all_sync(0xffffffffu, nvis == 64);
                if (!full) {
#pragma unroll
                    for (int e = 0; e < 64; e++)
                        if (e >= nvis) v[e] = __float_as_uint(-INFINITY);
                }
                if constexpr (MASKED)   // (a separate instance: the causal one keeps its registers)
                    if (valid) add_mask(p, tok, kb, nvis, mscl, v);
                float mx = 0.0f;
                if constexpr (MODE != kExact) {
                    float m4[4];
#pragma unroll
                    for (int a = 0; a < 4; a++) m4[a] = fmaxf(__uint_as_float(v[a]), __uint_as_float(v[4 + a]));
#pragma unroll
                    for (int e = 8; e < 64; e += 8)
#pragma unroll
                        for (int a = 0; a < 4; a++)
                            m4[a] = max3(m4[a], __uint_as_float(v[e + a]), __uint_as_float(v[e + 4 + a]));
                    mx = max3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
                }
                if constexpr (MODE == kStats) {
                    // running raw max and sum of 2^((acc - max) * cs), exact online rescale
                    const float nmax = fmaxf(m, mx);
                    if (nmax != -INFINITY) {
                        const float nb = -nmax * cs;
                        const uint64_t nb2 = pk2(nb, nb);
                        uint64_t s2[2] = {0ull, 0ull};
#pragma unroll
                        for (int e = 0; e < 32; e++) {
                            const float2 xy = up2(fma2(pk2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])),
                                                       cs2, nb2));
                            s2[e & 1] = add2(s2[e & 1], pk2(ex2_approx(xy.x), ex2_approx(xy.y)));
                        }
                        const float2 sa = up2(add2(s2[0], s2[1]));
                        l = (m == -INFINITY ? 0.0f : l * ex2_approx(fmaf(m, cs, nb))) + (sa.x + sa.y);
                        m = nmax;
                    }
                    continue;
                }
                float f = 1.0f;
                bool resc = false;
                uint64_t nm2;
                if constexpr (MODE == kOnePass) {
                    const float xm = mx * cs;
                    if (xm > m + kLazy) {   // never for a sub-tile without visible keys (xm = -inf)
                        f = ex2_approx(m - xm);   // 0 while m = -inf
                        resc = m != -INFINITY;
                        l *= f;
                        m = xm;
                    }
                    // p = 2^(acc*cs - m): masked keys hold -inf (2^-inf = 0); rows
                    // without a visible key yet have m = -inf and every key masked
                    const float nm = m == -INFINITY ? 0.0f : -m;
                    nm2 = pk2(nm, nm);
                } else {
                    nm2 = pk2(nMx, nMx);   // p = F16(2^(acc*cs - M*log2e) * (1/Z)), ggml's rounding
                }
                uint64_t s2[2] = {0ull, 0ull};
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    uint32_t pkd[16];
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        const float2 xy = up2(fma2(pk2(__uint_as_float(v[u * 32 + 2 * e]),
                                                       __uint_as_float(v[u * 32 + 2 * e + 1])), cs2, nm2));
                        float x0 = ex2_approx(xy.x), x1 = ex2_approx(xy.y);
                        if constexpr (MODE == kOnePass) {
                            s2[e & 1] = add2(s2[e & 1], pk2(x0, x1));
                        } else {
                            x0 = __fmul_rn(x0, inv);
                            x1 = __fmul_rn(x1, inv);
                        }
                        const __half2 h2 = __floats2half2_rn(x0, x1);
                        pkd[e] = *reinterpret_cast<const uint32_t *>(&h2);
                    }
                    // keys 32u .. 32u+31 -> packed columns 16u .. 16u+15 of the buffer
                    tmem_st16(tS + bf * 64 + u * 16, pkd);
                }
                if constexpr (MODE == kOnePass) {
                    const float2 sa = up2(add2(s2[0], s2[1]));
                    l += sa.x + sa.y;
                    // O holds this segment's earlier sub-tiles: once the last P . V
                    // into it has completed, scale the raised rows (before P(i) is
                    // reported, so before PV(i) adds to O)
                    if (i > i0 && __any_sync(0xffffffffu, resc)) {
                        if (!mbar_wait_ab(&o_ready[grp * 2 + ((i - 1) & 1)], ((i - 1) >> 1) & 1, p.limit_ns, flags)) {
                            give_up(p, flags, 1u);
                            return false;
                        }
                        tc_fence_after();
                        const float fo = resc ? f : 1.0f;
#pragma unroll 1
                        for (int ch = 0; ch < D / 16; ch++) {
                            uint32_t o[16];
                            tmem_ld16(tO + ch * 16, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int e = 0; e < 16; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * fo);
                            tmem_st16(tO + ch * 16, o);
                        }
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[grp * 2 + bf]);
            }
            const bool whole = sg.t0 == 0 && sg.t1 == nt_of(p, b);   // no other CTA holds this pair
            const int64_t slot = (((int64_t)c * p.kseg + k) * p.nt + grp) * 128 + row;
            if constexpr (MODE == kStats) {
                // (max in scaled units, sum) of every segment, split or not
                reinterpret_cast<float2 *>(p.pstat)[slot] =
                    make_float2(m == -INFINITY ? -INFINITY : __fmul_rn(m, p.scale), l);
                return true;
            }
            // ---- the segment's output ----
            if (!mbar_wait_ab(o_full, k & 1, p.limit_ns, flags)) {
                give_up(p, flags, 1u);
                return false;
            }
            tc_fence_after();
            // (the caller's rows hold dv-wide heads; head_dim 96 runs here as 128
            // with zero-filled columns 96-127, which are not written out)
            float *dst = p.out + (int64_t)tok * p.out_stride + (int64_t)(p.out_head0 + kvh * p.r + hd) * p.dv;
            float scl = 1.0f;   // the exact pass's O is final (p carries 1/Z)
            if (whole) {
                if (MODE == kOnePass) scl = l > 0.0f ? __fdiv_rn(1.0f, l) : no_key_scale(p);
            } else {
                if (MODE == kOnePass) reinterpret_cast<float2 *>(p.pstat)[slot] = make_float2(m, l);
                dst = p.pout + slot * D;
            }
            // a split segment's rows stay in L2 (evict-last) for the fold, past the
            // K/V tiles other CTAs stream meanwhile
            const uint64_t pol = policy_evict_last();
#pragma unroll 1
            for (int ch = 0; ch < p.dv / 32; ch++) {
                uint32_t o[32];
                tmem_ld32(tO + ch * 32, o);
                tmem_wait_ld();
                if (valid)
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        const float4 val = make_float4(__uint_as_float(o[4 * q]) * scl, __uint_as_float(o[4 * q + 1]) * scl,
                                                       __uint_as_float(o[4 * q + 2]) * scl,
                                                       __uint_as_float(o[4 * q + 3]) * scl);
                        if (whole) *reinterpret_cast<float4 *>(dst + ch * 32 + 4 * q) = val;
                        else st_v4_hint(dst + ch * 32 + 4 * q, val, pol);
                    }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_empty);
            return true;
        });
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0 && lane == 0 && flags[0]) {
        // the CTA gave up: loads nobody waited for may still be landing
        for (int j = issued_k > KS ? issued_k - KS : 0; j < issued_k; j++)
            mbar_wait(&k_full[j % KS], (j / KS) & 1, p.limit_ns);
        if constexpr (MODE != kStats)
            for (int j = issued_v > VS ? issued_v - VS : 0; j < issued_v; j++)
                mbar_wait(&v_full[j % VS], (j / VS) & 1, p.limit_ns);
        if (issued_q > 0) mbar_wait(q_full, (issued_q - 1) & 1, p.limit_ns);
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// the CTA-pair form (tcgen05 cta_group::2) of the one-pass kernel, head_dim 128
// ---------------------------------------------------------------------------
// A 2-CTA cluster holds four query tiles of one KV head (a block of 4 tb
// tokens): the even CTA tiles 0 and 1 (A, B), the odd CTA tiles 2 and 3.  The
// even CTA's three MMA-issuing warps drive both SMs' tensor cores with M = 256
// instructions -- rows 0-127 from the even CTA's tile, 128-255 from the odd
// CTA's -- so one instruction does what two did in prefill_kernel, whose
// sub-tile rate the MMA issue bounds.  Each CTA stages half of every K and V
// tile: K's keys 32*rank .. +31 of both 64-key sub-tiles (B's N = 64 keys split
// 32/32), V's dims 64*rank .. +63 (N = 128 split 64/64).  Both CTAs' TMA loads
// complete on the even CTA's full barriers; the issuers' commits arrive on
// both CTAs' barriers (empty slots, S ready, P . V done); both CTAs' softmax
// warps report P and the free O on the even CTA's barriers.  Each CTA's
// softmax and epilogue handle its own 256 rows, as in prefill_kernel.
struct PL2 {
    static constexpr int NT = 2;                          // query tiles a CTA holds (4 a pair)
    static constexpr int KS = 6, VS = 4;                  // half-tile rings
    static constexpr uint32_t kQTile = 2 * kBox;          // 128 rows x 128 halves
    static constexpr uint32_t kKBox = 32 * 128;           // [32 keys][64 halves]
    static constexpr uint32_t kKHalf = 4 * kKBox;         // [2 sub-tiles][2 dim boxes][32 keys][64 halves]
    static constexpr uint32_t kVHalf = kBox;              // [128 keys][this CTA's 64 dims]
    static constexpr size_t o_q = 0;
    static constexpr size_t o_k = o_q + NT * (size_t)kQTile;
    static constexpr size_t o_v = o_k + (size_t)KS * kKHalf;
    static constexpr size_t o_bar = o_v + (size_t)VS * kVHalf;
    // as PL: q_full, q_empty, k_full[KS], k_empty[KS], v_full[VS], v_empty[VS],
    // s_full[2][2], p_full[2][2], o_ready[2][2], o_full, o_empty, drain[3]
    static constexpr int NBAR = 2 + 2 * KS + 2 * VS + 12 + 5;
    static constexpr size_t o_tm = o_bar + (size_t)NBAR * 8;
    static constexpr size_t o_flags = o_tm + 16;
    static constexpr size_t bytes = o_flags + 16;
    static_assert(bytes <= 227 * 1024, "shared memory of the pair kernel");
    static_assert(o_k % 1024 == 0 && o_v % 1024 == 0 && kKBox % 1024 == 0, "swizzled boxes 1024-byte aligned");
};

template <bool MASKED>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    prefill2_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap32,
                    const __grid_constant__ CUtensorMap vmap, const PrefillParams p)
{
    constexpr int D = 128;
    using L = PL2;
    constexpr int KS = L::KS, VS = L::VS, NT = L::NT;
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L::o_bar);
    uint64_t *q_full = bar, *q_empty = bar + 1;
    uint64_t *k_full = bar + 2, *k_empty = k_full + KS;
    uint64_t *v_full = k_empty + KS, *v_empty = v_full + VS;
    uint64_t *s_full = v_empty + VS;
    uint64_t *p_full = s_full + 4;
    uint64_t *o_ready = p_full + 4;
    uint64_t *o_full = o_ready + 4, *o_empty = o_full + 1;
    uint64_t *drain = o_empty + 1;
    uint32_t *tm_slot = reinterpret_cast<uint32_t *>(smem + L::o_tm);
    volatile int *flags = reinterpret_cast<volatile int *>(smem + L::o_flags);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank = (int)cluster_rank(), c = blockIdx.x >> 1;   // c: the pair's work range
    // the even CTA's barrier at the offset of `b` (shared::cluster address)
    auto lead = [&](uint64_t *b) { return mapa(smem_addr(b), 0); };
    int issued_q = 0, issued_k = 0, issued_v = 0;

    if (tid == 0) {
        for (int i = 0; i < L::NBAR; i++) {
            // the even CTA's full barriers count its own expect_tx arrival; its
            // p_full the softmax warps of a tile group of both CTAs, its o_empty
            // every epilogue warp of both; k_empty and q_empty get the commits of
            // both S issuers
            const uint64_t *bi = &bar[i];
            const bool two = bi == q_empty || (bi >= k_empty && bi < k_empty + KS);
            mbar_init(&bar[i], (bi >= p_full && bi < p_full + 4) ? 2 * kGW : bi == o_empty ? 2 * NT * kGW : two ? 2 : 1);
        }
        flags[0] = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc2(tm_slot, 512);
        tmem_relinquish2();
    }
    tc_fence_before();
    __syncthreads();
    // neither CTA signals the other's barriers before both are initialised
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = *tm_slot;
    pdl_wait();   // (as prefill_kernel)
    pdl_launch_dependents();

    if (warp == 0) {
        // ================= TMA (both CTAs: this CTA's halves) =================
        if (lane == 0) {
            prefetch_tmap(&qmap);
            prefetch_tmap(&kmap32);
            prefetch_tmap(&vmap);
            const uint32_t qbytes = (uint32_t)(p.r * p.tb) * 128u * 2u;   // one Q tile (zero fill counts)
            for_segments(p, c, [&](int k, const Seg &sg) {
                const int kvh = sg.pair / p.nblk, b = sg.pair % p.nblk;
                if (k > 0 && !mbar_wait_ab(q_empty, (k - 1) & 1, p.limit_ns, flags)) {
                    give_up(p, flags, 2u);
                    return false;
                }
                if (rank == 0) mbar_arrive_expect_tx(q_full, 2 * NT * qbytes);
#pragma unroll
                for (int g = 0; g < NT; g++)
#pragma unroll
                    for (int bx = 0; bx < 2; bx++)
                        tma_load_3d_pair(smem + L::o_q + g * L::kQTile + bx * kBox, &qmap, lead(q_full), bx * 64,
                                         kvh * p.r, (4 * b + 2 * rank + g) * p.tb);
                issued_q++;
                for (int t = sg.t0; t < sg.t1; t++) {
                    const int s = issued_k % KS;
                    if (issued_k >= KS && !mbar_wait_ab(&k_empty[s], ((issued_k / KS) - 1) & 1, p.limit_ns, flags)) {
                        give_up(p, flags, 2u);
                        return false;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&k_full[s], 2 * L::kKHalf);
#pragma unroll
                    for (int sub = 0; sub < 2; sub++)
#pragma unroll
                        for (int bx = 0; bx < 2; bx++)
                            tma_load_3d_pair(smem + L::o_k + s * L::kKHalf + (2 * sub + bx) * L::kKBox, &kmap32,
                                             lead(&k_full[s]), bx * 64, kvh, t * 128 + sub * 64 + rank * 32);
                    issued_k++;
                    const int sv = issued_v % VS;
                    if (issued_v >= VS && !mbar_wait_ab(&v_empty[sv], ((issued_v / VS) - 1) & 1, p.limit_ns, flags)) {
                        give_up(p, flags, 2u);
                        return false;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&v_full[sv], 2 * L::kVHalf);
                    tma_load_3d_pair(smem + L::o_v + sv * L::kVHalf, &vmap, lead(&v_full[sv]), rank * 64, kvh,
                                     t * 128);
                    issued_v++;
                }
                return true;
            });
        }
    } else if (warp == 1 || warp >= 2 + 2 * kGW) {
        // ================= MMA issue (even CTA) =================
        const int role = warp == 1 ? 0 : warp - (1 + 2 * kGW);   // 0: S_A, 1: S_B, 2: PV
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idS = idesc_f16_f32(256, 64, false);
            constexpr uint32_t idO = idesc_f16_f32(256, D, true);
            const uint32_t sq = smem_addr(smem + L::o_q), sk = smem_addr(smem + L::o_k);
            const uint32_t sv = smem_addr(smem + L::o_v);
            bool ok = true;
            auto wt = [&](uint64_t *b, uint32_t par) {
                if (ok && !mbar_wait_ab(b, par, p.limit_ns, flags)) {
                    give_up(p, flags, 1u);
                    ok = false;
                }
                return ok;
            };
            int i = 0;
            if (role < NT) {
                const int g = role;
                for_segments(p, c, [&](int k, const Seg &sg) {
                    const int i1 = i + 2 * (sg.t1 - sg.t0);
                    if (!wt(q_full, k & 1)) return false;
                    for (; i < i1; i++) {
                        const int tile = i >> 1;
                        if (!(i & 1) && !wt(&k_full[tile % KS], (tile / KS) & 1)) return false;
                        if (i >= 2 && !wt(&o_ready[g * 2 + (i & 1)], ((i - 2) >> 1) & 1)) return false;
                        tc_fence_after();
                        // S_g(i) (both CTAs' rows) = Q_g . K(sub-tile i&1: 32 keys in each CTA)^T
                        const uint32_t kt = sk + (tile % KS) * L::kKHalf + (i & 1) * 2 * L::kKBox;
#pragma unroll
                        for (int kk = 0; kk < D / 16; kk++) {
                            umma_ss2(tmem + g * 128 + (i & 1) * 64,
                                     sdesc_k_sw128(sq + g * L::kQTile + (kk >> 2) * kBox + (kk & 3) * 32),
                                     sdesc_k_sw128(kt + (kk >> 2) * L::kKBox + (kk & 3) * 32), idS, kk > 0);
                        }
                        umma_commit2_mc(&s_full[g * 2 + (i & 1)], 3);
                        if (i & 1) umma_commit2_mc(&k_empty[tile % KS], 3);
                        if (i == i1 - 1) umma_commit2_mc(q_empty, 3);
                    }
                    return true;
                });
            } else if (role == 2) {
                for_segments(p, c, [&](int k, const Seg &sg) {
                    const int i0 = i, i1 = i + 2 * (sg.t1 - sg.t0);
                    for (; i < i1; i++) {
                        const int tile = i >> 1;
#pragma unroll
                        for (int g = 0; g < NT; g++) {
                            if (!wt(&p_full[g * 2 + (i & 1)], (i >> 1) & 1)) return false;
                            if (g == 0 && !(i & 1) && !wt(&v_full[tile % VS], (tile / VS) & 1)) return false;
                            if (g == 0 && i == i0 && k > 0 && !wt(o_empty, (k - 1) & 1)) return false;
                            tc_fence_after();
                            // O_g (+)= P_g(i) . V(64 keys; 64 of the dims in each CTA)
                            const uint32_t vt = sv + (tile % VS) * L::kVHalf + (i & 1) * 8192;
#pragma unroll
                            for (int kk = 0; kk < 4; kk++)
                                umma_ts2(tmem + kTmO + g * D, tmem + g * 128 + (i & 1) * 64 + kk * 8,
                                         sdesc_mn_sw128(vt + kk * 2048, kBox), idO, !(i == i0 && kk == 0));
                            umma_commit2_mc(&o_ready[g * 2 + (i & 1)], 3);
                        }
                        if (i & 1) umma_commit2_mc(&v_empty[tile % VS], 3);
                        if (i == i1 - 1) umma_commit2_mc(o_full, 3);
                    }
                    return true;
                });
            }
            umma_commit2(&drain[role]);
            mbar_wait(&drain[role], 0, p.limit_ns);
        }
    } else {
        // ================= softmax / epilogue (both CTAs, their own rows) =================
        const int grp = (warp - 2) / kGW;
        const int gt = 2 * rank + grp;            // the tile of the pair's block
        const int q4 = warp & 3;
        const int row = q4 * 32 + lane;
        const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
        const uint32_t tS = trow + grp * 128, tO = trow + kTmO + grp * D;
        const int tok_in = row / p.r, hd = row - tok_in * p.r;
        const bool row_ok = tok_in < p.tb;
        const float cs = p.scale * kLog2e;
        const uint64_t cs2 = pk2(cs, cs);
        const uint32_t pf_lead = lead(&p_full[grp * 2]), oe_lead = lead(o_empty);
        int i = 0;
        for_segments(p, c, [&](int k, const Seg &sg) {
            const int b = sg.pair % p.nblk, kvh = sg.pair / p.nblk;
            const int tok = (4 * b + gt) * p.tb + tok_in;
            const bool valid = row_ok && tok < p.n_new;
            const int64_t lim = !valid ? -1 : p.mask ? p.n_past + p.n_new - 1 : p.n_past + tok;
            const float mscl = p.mask ? __fdiv_rn(1.0f, p.scale) : 0.0f;
            const int i0 = i, i1 = i + 2 * (sg.t1 - sg.t0);
            float m = -INFINITY, l = 0.0f;
            for (; i < i1; i++) {
                const int bf = i & 1;
                if (!mbar_wait_ab(&s_full[grp * 2 + bf], (i >> 1) & 1, p.limit_ns, flags)) {
                    give_up(p, flags, 1u);
                    return false;
                }
                tc_fence_after();
                uint32_t v[64];
                tmem_ld32(tS + bf * 64, *reinterpret_cast<uint32_t(*)[32]>(v));
                tmem_ld32(tS + bf * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
                tmem_wait_ld();
                const int64_t kb = (int64_t)(2 * sg.t0 + (i - i0)) * 64;
                const int nvis = (int)max((int64_t)0, min((int64_t)64, lim - kb + 1));
                const bool full = __all_sync(0xffffffffu, nvis == 64);
                if (!full) {
#pragma unroll
                    for (int e = 0; e < 64; e++)
                        if (e >= nvis) v[e] = __float_as_uint(-INFINITY);
                }
                if constexpr (MASKED)
                    if (valid) add_mask(p, tok, kb, nvis, mscl, v);
                float m4[4];
#pragma unroll
                for (int a = 0; a < 4; a++) m4[a] = fmaxf(__uint_as_float(v[a]), __uint_as_float(v[4 + a]));
#pragma unroll
                for (int e = 8; e < 64; e += 8)
#pragma unroll
                    for (int a = 0; a < 4; a++)
                        m4[a] = max3(m4[a], __uint_as_float(v[e + a]), __uint_as_float(v[e + 4 + a]));
                const float mx = max3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
                float f = 1.0f;
                bool resc = false;
                const float xm = mx * cs;
                if (xm > m + kLazy) {
                    f = ex2_approx(m - xm);
                    resc = m != -INFINITY;
                    l *= f;
                    m = xm;
                }
                const float nm = m == -INFINITY ? 0.0f : -m;
                const uint64_t nm2 = pk2(nm, nm);
                uint64_t s2[2] = {0ull, 0ull};
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    uint32_t pkd[16];
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        const float2 xy = up2(fma2(pk2(__uint_as_float(v[u * 32 + 2 * e]),
                                                       __uint_as_float(v[u * 32 + 2 * e + 1])), cs2, nm2));
                        const float x0 = ex2_approx(xy.x), x1 = ex2_approx(xy.y);
                        s2[e & 1] = add2(s2[e & 1], pk2(x0, x1));
                        const __half2 h2 = __floats2half2_rn(x0, x1);
                        pkd[e] = *reinterpret_cast<const uint32_t *>(&h2);
                    }
                    tmem_st16(tS + bf * 64 + u * 16, pkd);
                }
                const float2 sa = up2(add2(s2[0], s2[1]));
                l += sa.x + sa.y;
                if (i > i0 && __any_sync(0xffffffffu, resc)) {
                    if (!mbar_wait_ab(&o_ready[grp * 2 + ((i - 1) & 1)], ((i - 1) >> 1) & 1, p.limit_ns, flags)) {
                        give_up(p, flags, 1u);
                        return false;
                    }
                    tc_fence_after();
                    const float fo = resc ? f : 1.0f;
#pragma unroll 1
                    for (int ch = 0; ch < D / 16; ch++) {
                        uint32_t o[16];
                        tmem_ld16(tO + ch * 16, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * fo);
                        tmem_st16(tO + ch * 16, o);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(pf_lead + (uint32_t)(bf * 8));
            }
            const bool whole = sg.t0 == 0 && sg.t1 == nt_of(p, b);
            const int64_t slot = (((int64_t)c * p.kseg + k) * 4 + gt) * 128 + row;
            if (!mbar_wait_ab(o_full, k & 1, p.limit_ns, flags)) {
                give_up(p, flags, 1u);
                return false;
            }
            tc_fence_after();
            float *dst = p.out + (int64_t)tok * p.out_stride + (int64_t)(p.out_head0 + kvh * p.r + hd) * p.dv;
            float scl = 1.0f;
            if (whole) {
                scl = l > 0.0f ? __fdiv_rn(1.0f, l) : no_key_scale(p);
            } else {
                reinterpret_cast<float2 *>(p.pstat)[slot] = make_float2(m, l);
                dst = p.pout + slot * D;
            }
            const uint64_t pol = policy_evict_last();
#pragma unroll 1
            for (int ch = 0; ch < p.dv / 32; ch++) {
                uint32_t o[32];
                tmem_ld32(tO + ch * 32, o);
                tmem_wait_ld();
                if (valid)
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        const float4 val = make_float4(__uint_as_float(o[4 * q]) * scl, __uint_as_float(o[4 * q + 1]) * scl,
                                                       __uint_as_float(o[4 * q + 2]) * scl,
                                                       __uint_as_float(o[4 * q + 3]) * scl);
                        if (whole) *reinterpret_cast<float4 *>(dst + ch * 32 + 4 * q) = val;
                        else st_v4_hint(dst + ch * 32 + 4 * q, val, pol);
                    }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(oe_lead);
            return true;
        });
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0 && lane == 0 && rank == 0 && flags[0]) {
        // the CTA gave up: loads of either CTA nobody waited for may still be
        // landing (both CTAs' complete on these barriers)
        for (int j = issued_k > KS ? issued_k - KS : 0; j < issued_k; j++)
            mbar_wait(&k_full[j % KS], (j / KS) & 1, p.limit_ns);
        for (int j = issued_v > VS ? issued_v - VS : 0; j < issued_v; j++)
            mbar_wait(&v_full[j % VS], (j / VS) & 1, p.limit_ns);
        if (issued_q > 0) mbar_wait(q_full, (issued_q - 1) & 1, p.limit_ns);
    }
    // every MMA of the pair has completed (the issuers' drains) and every load
    // has landed before either CTA frees its tensor memory or leaves
    __syncthreads();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc2(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// the fold of split pairs
// ---------------------------------------------------------------------------
// out = sum_i 2^(m_i - M) O_i / sum_i 2^(m_i - M) l_i over the pair's segments
// (CTAs ca..cb in order; the pair is segment 0 of every CTA after ca),
// scattered to the caller's [token][head][D] rows.  One block per (pair, 16 of
// its 256 rows), 16 threads a row, D/16 floats a thread.  The statistics and
// the partial rows of four segments are loaded together (one round trip for
// the common 2-4 segments; M is raised between groups of four, rescaling what
// was summed, so the order of the sums is fixed).  The block finds the pair's
// CTAs before its grid-dependency wait, so with a programmatic launch that
// overlaps the attention kernel's tail.
template <int D>
__global__ void __launch_bounds__(256) prefill_out_fold(const PrefillParams p)
{
    constexpr int F4 = D / 64;   // float4s of a thread
    const int bpp = 8 * p.nt;    // blocks of 16 rows a pair
    const int pair = blockIdx.x / bpp, row0 = (blockIdx.x % bpp) * 16;
    __shared__ int info[3];
    if (threadIdx.x == 0) {
        int ca, cb;
        pair_ctas(p, pair, ca, cb);
        info[0] = ca;
        info[1] = cb;
        info[2] = pair - pair_of(p, cta_lo(p, ca));
    }
    __syncthreads();
    const int ca = info[0], cb = info[1], seg_a = info[2];
    pdl_wait();   // the attention kernel's partials
    if (ca == cb) return;   // one segment: the attention kernel wrote the rows
    const int rr = row0 + (int)(threadIdx.x >> 4), part = threadIdx.x & 15;
    const int grp = rr >> 7, row = rr & 127;
    const int tok_in = row / p.r, hd = row - tok_in * p.r;
    const int b = pair % p.nblk, kvh = pair / p.nblk;
    const int tok = (p.nt * b + grp) * p.tb + tok_in;
    if (grp >= p.nt || tok_in >= p.tb || tok >= p.n_new) return;
    auto slot = [&](int cc) { return (((int64_t)cc * p.kseg + (cc == ca ? seg_a : 0)) * p.nt + grp) * 128 + row; };
    if (part * F4 * 4 >= p.dv) return;   // the zero-filled columns past a 96-wide head
    float4 *dst = reinterpret_cast<float4 *>(p.out + (int64_t)tok * p.out_stride +
                                             (int64_t)(p.out_head0 + kvh * p.r + hd) * p.dv) + part * F4;
    const bool exact = p.mode == kExact;   // the segments' rows are final: their sum, CTAs in order
    const float2 *ps = reinterpret_cast<const float2 *>(p.pstat);
    const uint64_t pol = policy_evict_first();
    float M = -INFINITY, lsum = 0.0f;
    float4 acc[F4];
#pragma unroll
    for (int q = 0; q < F4; q++) acc[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int c0 = ca; c0 <= cb; c0 += 4) {
        float2 st[4];
        float4 v[4][F4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const bool in = c0 + u <= cb;
            const int64_t sl = slot(in ? c0 + u : c0);
            st[u] = in && !exact ? __ldcg(ps + sl) : make_float2(-INFINITY, 0.0f);
            const float *src = p.pout + sl * D + part * F4 * 4;
#pragma unroll
            for (int q = 0; q < F4; q++) v[u][q] = ld_cg_v4_hint(src + 4 * q, pol);   // read once: evict first
        }
        if (exact) {
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (c0 + u <= cb)
#pragma unroll
                    for (int q = 0; q < F4; q++) {
                        acc[q].x += v[u][q].x;
                        acc[q].y += v[u][q].y;
                        acc[q].z += v[u][q].z;
                        acc[q].w += v[u][q].w;
                    }
            continue;
        }
        const float mx = fmaxf(fmaxf(M, fmaxf(st[0].x, st[1].x)), fmaxf(st[2].x, st[3].x));
        if (mx > M) {   // raise M: what was summed is rescaled (never in the first group)
            const float f = M == -INFINITY ? 0.0f : exp2f(M - mx);
            lsum *= f;
#pragma unroll
            for (int q = 0; q < F4; q++) acc[q] = make_float4(acc[q].x * f, acc[q].y * f, acc[q].z * f, acc[q].w * f);
            M = mx;
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const float w = st[u].x == -INFINITY ? 0.0f : exp2f(st[u].x - M);   // no visible key: weight 0
            lsum += st[u].y * w;
#pragma unroll
            for (int q = 0; q < F4; q++) {
                acc[q].x += v[u][q].x * w;
                acc[q].y += v[u][q].y * w;
                acc[q].z += v[u][q].z * w;
                acc[q].w += v[u][q].w * w;
            }
        }
    }
    if (exact) {
#pragma unroll
        for (int q = 0; q < F4; q++) dst[q] = acc[q];
        return;
    }
    const float inv = lsum > 0.0f ? __fdiv_rn(1.0f, lsum) : no_key_scale(p);
#pragma unroll
    for (int q = 0; q < F4; q++)
        dst[q] = make_float4(acc[q].x * inv, acc[q].y * inv, acc[q].z * inv, acc[q].w * inv);
}

// (M, 1/Z) per (pair, row) for the exact output pass: M = the largest segment
// maximum, Z = sum_i l_i exp(m_i - M) in double, CTAs in order; one block per
// pair, a thread per row of its two tiles
__global__ void __launch_bounds__(256) prefill_stats_fold(const PrefillParams p)
{
    const int pair = blockIdx.x, rr = threadIdx.x, grp = rr >> 7, row = rr & 127;
    __shared__ int info[3];
    if (threadIdx.x == 0) {
        int ca, cb;
        pair_ctas(p, pair, ca, cb);
        info[0] = ca;
        info[1] = cb;
        info[2] = pair - pair_of(p, cta_lo(p, ca));
    }
    __syncthreads();
    const int ca = info[0], cb = info[1], seg_a = info[2];
    if (grp >= p.nt) return;   // (one query tile a CTA at head_dim 256)
    auto slot = [&](int cc) { return (((int64_t)cc * p.kseg + (cc == ca ? seg_a : 0)) * p.nt + grp) * 128 + row; };
    const float2 *ps = reinterpret_cast<const float2 *>(p.pstat);
    float M = -INFINITY;
    for (int cc = ca; cc <= cb; cc++) M = fmaxf(M, __ldcg(ps + slot(cc)).x);
    double Z = 0.0;
    for (int cc = ca; cc <= cb; cc++) {
        const float2 v = __ldcg(ps + slot(cc));
        if (v.x != -INFINITY) Z += (double)v.y * (double)exp2f((v.x - M) * kLog2e);
    }
    p.rstat[(int64_t)pair * 256 + rr] = make_float2(M, Z > 0.0 ? __fdiv_rn(1.0f, (float)Z) : 0.0f);
}

template <int D, bool MASKED>
cudaError_t prep_pf_m()
{
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel<D, kOnePass, MASKED>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PL<D>::bytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(prefill_kernel<D, kStats, MASKED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)PL<D>::bytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(prefill_kernel<D, kExact, MASKED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)PL<D>::bytes);
    return e;
}

template <int D>
cudaError_t prep_pf()
{
    const cudaError_t e = prep_pf_m<D, false>();
    return e == cudaSuccess ? prep_pf_m<D, true>() : e;
}

// The attention kernels are launched programmatically: their set-up (barriers,
// tensor memory, the cluster barrier) overlaps the previous kernel's tail, and
// they wait for it (griddepcontrol.wait) before any memory access it may affect.
template <class K>
cudaError_t launch_attn_early(K kernel, int n_ctas, size_t smem, cudaStream_t st, const CUtensorMap &qmap,
                              const CUtensorMap &kmap, const CUtensorMap &vmap, const PrefillParams &p)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)n_ctas);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, qmap, kmap, vmap, p);
}

template <int D, bool MASKED>
cudaError_t launch_pf_kernel(int which, const CUtensorMap &qmap, const CUtensorMap &kmap, const CUtensorMap &vmap,
                             const PrefillParams &p, cudaStream_t st)
{
    if (which == 0)
        return launch_attn_early(prefill_kernel<D, kOnePass, MASKED>, p.n_cta, PL<D>::bytes, st, qmap, kmap, vmap, p);
    if (which == 2)
        return launch_attn_early(prefill_kernel<D, kStats, MASKED>, p.n_cta, PL<D>::bytes, st, qmap, kmap, vmap, p);
    return launch_attn_early(prefill_kernel<D, kExact, MASKED>, p.n_cta, PL<D>::bytes, st, qmap, kmap, vmap, p);
}

template <int D>
cudaError_t launch_pf(int which, const CUtensorMap &qmap, const CUtensorMap &kmap, const CUtensorMap &vmap,
                      const PrefillParams &p, cudaStream_t st)
{
    switch (which) {
    case 0:
    case 2:
    case 4:
        return p.mask ? launch_pf_kernel<D, true>(which, qmap, kmap, vmap, p, st)
                      : launch_pf_kernel<D, false>(which, qmap, kmap, vmap, p, st);
    case 3: prefill_stats_fold<<<p.hkv * p.nblk, 256, 0, st>>>(p); break;
    default: {
        // the fold may be scheduled once every attention CTA has started
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(p.hkv * p.nblk * 8 * p.nt));
        cfg.blockDim = dim3(256);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, prefill_out_fold<D>, p);
    }
    }
    return cudaGetLastError();
}

}  // namespace

bool prefill_supported(int D) { return D == 64 || D == 128 || D == 256; }
int prefill_kernel_dim(int D) { return D == 96 ? 128 : D; }   // 96: the 128 kernel on zero-filled columns
int prefill_max_segments() { return 4; }

cudaError_t prefill_prepare(int D)
{
    switch (D) {
    case 64: return prep_pf<64>();
    case 128: return prep_pf<128>();
    case 256: return prep_pf<256>();
    default: return cudaSuccess;
    }
}

int prefill_tiles(int D) { return D == 256 ? PL<256>::NT : 2; }

cudaError_t prefill_pair_prepare(int *clusters)
{
    *clusters = 0;
    cudaError_t e = cudaFuncSetAttribute(prefill2_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)PL2::bytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(prefill2_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PL2::bytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = PL2::bytes;
    return cudaOccupancyMaxActiveClusters(clusters, prefill2_kernel<false>, &cfg);
}

cudaError_t launch_prefill_pair(const CUtensorMap &qmap, const CUtensorMap &kmap32, const CUtensorMap &vmap,
                                const PrefillParams &p, cudaStream_t st)
{
    // (the kernel's cluster shape is compiled in: 2 x 1 x 1)
    return p.mask ? launch_attn_early(prefill2_kernel<true>, 2 * p.n_cta, PL2::bytes, st, qmap, kmap32, vmap, p)
                  : launch_attn_early(prefill2_kernel<false>, 2 * p.n_cta, PL2::bytes, st, qmap, kmap32, vmap, p);
}

cudaError_t launch_prefill(int D, int which, const CUtensorMap &qmap, const CUtensorMap &kmap,
                           const CUtensorMap &vmap, const PrefillParams &p, cudaStream_t st)
{
    switch (D) {
    case 64: return launch_pf<64>(which, qmap, kmap, vmap, p, st);
    case 128: return launch_pf<128>(which, qmap, kmap, vmap, p, st);
    case 256: return launch_pf<256>(which, qmap, kmap, vmap, p, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace kvb
