// kv_prefill.cu -- attention of a multi-token chunk (prefill) on the 5th-
// generation tensor cores: tcgen05.mma with TMEM accumulators, operands staged
// in shared memory by TMA.
//
// Numerics: the reference's attention branch (src/model.cpp:1416-1445) for
// n_new query tokens: S = F16(q) . K (F32 accumulation), causal mask (key <=
// n_past + token), softmax with the global row max M and sum Z, p = F16(exp(s
// - M) / Z), O = p . V (F32 accumulation).  ggml rounds the normalised p to
// F16, so every p needs the final M and Z of its row: pass 1 computes S and
// the row statistics, pass 2 computes S again, forms p and accumulates P . V.
// exp is 2^(x log2 e) on the SFU (ex2.approx): within a few F32 ulps of expf,
// far inside the attention tolerance.
//
// Work: query rows are packed GQA-group-major: one 128-row tile holds tb =
// floor(128 / r) tokens x the r query heads of one KV head (row = token*r +
// head), so a K/V tile staged once serves every head of the group.  A "pair" is
// (KV head, block of tb tokens); its keys are the tiles of 128 keys up to the
// block's last visible key.  The pairs' tiles, laid end to end, are cut into C
// equal ranges (one CTA each, C <= SMs); a range holds one or more "segments"
// (the part of one pair it covers).
//
// prefill_kernel<D, OUT> (576 threads):
//   warp 0     TMA: the pair's Q tile, then K tiles (and V tiles in pass 2) into
//              mbarrier rings;
//   warp 1     TMEM owner and MMA issuer (one thread): S = Q . K^T, M=128, N=128
//              keys, K = D, into one of two 128-column TMEM buffers; in pass 2
//              also O += P . V (M=128, N=D, K=128 keys; P from TMEM, V read
//              MN-major from shared memory) into D more columns, one tile behind;
//   warps 2-17 a query row per lane and a quarter of each tile's keys per warp,
//              read from TMEM with tcgen05.ld: pass 1 keeps the running row max
//              / sum of exp; pass 2 writes p as F16 pairs back into TMEM with
//              tcgen05.st (double-buffered), the A operand of the P . V MMA,
//              and at a segment's end copies O out.
// prefill_stats_fold   (M, 1/Z) of every (pair, row) from the segments' partials
// prefill_out_fold     sum of the segments' partial outputs, scattered to out
// Every wait is bounded (limit_ns) and gives up when the CTA's abort flag is
// set; the CTA drains its TMA loads and MMAs and frees TMEM before leaving.
#include <math.h>

#include "kv_internal.h"
#include "kv_sm100.cuh"

namespace kvb {
namespace {

using namespace sm100;

constexpr int kSW = 16;                     // softmax / epilogue warps (2..17)
constexpr int kCP = 4;                      // statistics parts of a row: 2 tile groups x 2 key halves
constexpr int kPThreads = 64 + 32 * kSW;
constexpr uint32_t kBox = 128 * 128;   // one [128 rows][64 halves] swizzled box
// TMEM columns: S (two 128-column F32 buffers), O (up to 128 F32), P (two
// 64-column buffers of F16 pairs) -- 512 in all
constexpr uint32_t kTmO = 256, kTmP = 384;
constexpr float kLog2e = 1.4426950408889634f;

template <int D, bool OUT>
struct PL {
    static constexpr int NB = D / 64;                        // boxes per Q/K/V row
    static constexpr uint32_t kTile = (uint32_t)NB * kBox;   // 128 rows x D halves
    static constexpr int KS = OUT ? (D == 128 ? 3 : 6) : (D == 128 ? 6 : 12);
    static constexpr int VS = OUT ? (D == 128 ? 3 : 6) : 0;
    static constexpr size_t o_q = 0;
    static constexpr size_t o_k = o_q + kTile;
    static constexpr size_t o_v = o_k + (size_t)KS * kTile;
    static constexpr size_t o_bar = o_v + (size_t)VS * kTile;
    // q_full, q_empty, k_full[KS], k_empty[KS], v_full[VS], v_empty[VS],
    // s_full[2], s_free[2], p_full[2], p_empty[2], o_full, o_empty, drain
    static constexpr int NBAR = 2 + 2 * KS + 2 * VS + 8 + 3;
    static constexpr size_t o_tm = o_bar + (size_t)NBAR * 8;
    static constexpr size_t o_flags = o_tm + 16;
    static constexpr size_t bytes = o_flags + 16;
    static_assert(bytes <= 227 * 1024, "shared memory of the prefill kernel");
};

// ---- the work split ------------------------------------------------------------
__device__ __forceinline__ int nt_of(const PrefillParams &p, int b)
{
    const int64_t last = p.n_past + min(p.n_new, (b + 1) * p.tb);   // keys [0, last)
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

// ---------------------------------------------------------------------------
// pass 1 (OUT = false) and pass 2 (OUT = true)
// ---------------------------------------------------------------------------
template <int D, bool OUT>
__global__ void __launch_bounds__(kPThreads, 1) prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                 const __grid_constant__ CUtensorMap kmap,
                                                                 const __grid_constant__ CUtensorMap vmap,
                                                                 const PrefillParams p)
{
    using L = PL<D, OUT>;
    constexpr int NB = L::NB, KS = L::KS, VS = L::VS;
    constexpr uint32_t kTile = L::kTile;
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L::o_bar);
    uint64_t *q_full = bar, *q_empty = bar + 1;
    uint64_t *k_full = bar + 2, *k_empty = k_full + KS;
    uint64_t *v_full = k_empty + KS, *v_empty = v_full + VS;
    uint64_t *s_full = v_empty + VS, *s_free = s_full + 2;
    uint64_t *p_full = s_free + 2, *p_empty = p_full + 2;
    uint64_t *o_full = p_empty + 2, *o_empty = o_full + 1, *drain = o_empty + 1;
    uint32_t *tm_slot = reinterpret_cast<uint32_t *>(smem + L::o_tm);
    volatile int *flags = reinterpret_cast<volatile int *>(smem + L::o_flags);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, c = blockIdx.x;
    int issued_q = 0, issued_k = 0, issued_v = 0;   // TMA loads issued (warp 0, lane 0)

    if (tid == 0) {
        for (int i = 0; i < L::NBAR; i++) {
            // a tile group's 8 warps arrive on s_free and p_full, all 16 on o_empty
            const uint64_t *bi = &bar[i];
            const bool grp = bi == &s_free[0] || bi == &s_free[1] || bi == &p_full[0] || bi == &p_full[1];
            mbar_init(&bar[i], grp ? kSW / 2 : bi == o_empty ? kSW : 1);
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

    if (warp == 0) {
        // ================= TMA =================
        if (lane == 0) {
            prefetch_tmap(&qmap);
            prefetch_tmap(&kmap);
            if (OUT) prefetch_tmap(&vmap);
            const uint32_t qbytes = (uint32_t)(p.r * p.tb) * 128u * NB;
            for_segments(p, c, [&](int k, const Seg &sg) {
                const int kvh = sg.pair / p.nblk, b = sg.pair % p.nblk;
                if (k > 0 && !mbar_wait_ab(q_empty, (k - 1) & 1, p.limit_ns, flags)) {
                    give_up(p, flags, 2u);
                    return false;
                }
                mbar_arrive_expect_tx(q_full, qbytes);
#pragma unroll
                for (int bx = 0; bx < NB; bx++)
                    tma_load_3d(smem + L::o_q + bx * kBox, &qmap, q_full, bx * 64, kvh * p.r, b * p.tb);
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
                    if constexpr (OUT) {
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
    } else if (warp == 1) {
        // ================= MMA issue =================
        if (lane == 0) {
            constexpr uint32_t idS = idesc_f16_f32(128, 128, false);
            constexpr uint32_t idO = idesc_f16_f32(128, D, true);
            const uint32_t sq = smem_addr(smem + L::o_q), sk = smem_addr(smem + L::o_k);
            const uint32_t sv = smem_addr(smem + L::o_v);
            int j = 0;               // tiles issued (S)
            // tiles whose P . V is still to issue, oldest first; P . V runs two
            // tiles behind S so the next S never queues behind a P . V
            struct Pend {
                int j, seg;
                bool first, last;
            };
            Pend pq0{}, pq1{};
            int npq = 0;
            bool ok = true;
            auto issue_pv = [&](const Pend &pe) -> bool {
                const int jp = pe.j, pb = jp & 1, vs = jp % (VS > 0 ? VS : 1);
                if (!mbar_wait_ab(&p_full[pb], (jp >> 1) & 1, p.limit_ns, flags) ||
                    !mbar_wait_ab(&v_full[vs], (jp / (VS > 0 ? VS : 1)) & 1, p.limit_ns, flags) ||
                    (pe.first && pe.seg > 0 && !mbar_wait_ab(o_empty, (pe.seg - 1) & 1, p.limit_ns, flags))) {
                    give_up(p, flags, 1u);
                    return false;
                }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {   // 16 keys per step: 8 packed P columns
                    const uint64_t bd = sdesc_mn_sw128(sv + vs * kTile + kk * 2048, kBox);
                    umma_ts(tmem + kTmO, tmem + kTmP + pb * 64 + kk * 8, bd, idO, !(pe.first && kk == 0));
                }
                umma_commit(&p_empty[pb]);
                umma_commit(&v_empty[vs]);
                if (pe.last) umma_commit(o_full);
                return true;
            };
            for_segments(p, c, [&](int k, const Seg &sg) {
                if (!mbar_wait_ab(q_full, k & 1, p.limit_ns, flags)) {
                    give_up(p, flags, 1u);
                    return ok = false;
                }
                for (int t = sg.t0; t < sg.t1; t++) {
                    const int s = j % KS, sb = j & 1;
                    if (!mbar_wait_ab(&k_full[s], (j / KS) & 1, p.limit_ns, flags) ||
                        (j >= 2 && !mbar_wait_ab(&s_free[sb], ((j - 2) >> 1) & 1, p.limit_ns, flags))) {
                        give_up(p, flags, 1u);
                        return ok = false;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < D / 16; kk++) {
                        const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
                        umma_ss(tmem + sb * 128, sdesc_k_sw128(sq + off), sdesc_k_sw128(sk + s * kTile + off), idS,
                                kk > 0);
                    }
                    umma_commit(&s_full[sb]);
                    umma_commit(&k_empty[s]);
                    if (t == sg.t1 - 1) umma_commit(q_empty);
                    if constexpr (OUT) {
                        if (npq == 2) {
                            if (!issue_pv(pq0)) return ok = false;
                            pq0 = pq1;
                            npq = 1;
                        }
                        const Pend pe{j, k, t == sg.t0, t == sg.t1 - 1};
                        if (npq == 0) pq0 = pe;
                        else pq1 = pe;
                        npq++;
                    }
                    j++;
                }
                return true;
            });
            if (OUT && ok && npq > 0) ok = issue_pv(pq0);
            if (OUT && ok && npq > 1) ok = issue_pv(pq1);
            // every MMA this thread issued has completed before TMEM is freed
            umma_commit(drain);
            mbar_wait(drain, 0, p.limit_ns);
        }
    } else {
        // ================= softmax / epilogue =================
        // kSW warps: warp w reaches TMEM lanes 32*(w%4) .. +31 (its rows) and
        // takes column part (w-2)/4 of every tile (kCP parts of 128/kCP keys)
        // two groups of 8 warps take alternate tiles (group g: tiles j with j%2 == g),
        // so one group computes while the other waits on TMEM; in a group, warp w
        // has TMEM lanes 32*(w%4).. (its rows) and one half of the tile's keys
        const int sw = warp - 2, grp = sw >> 3, half = (sw >> 2) & 1;
        const int q4 = warp & 3;
        const int part = grp * 2 + half;          // statistics part of this warp
        const int row = q4 * 32 + lane;           // query row of the tile = token*r + head
        const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
        const int tok_in = row / p.r;
        const bool row_ok = tok_in < p.tb;
        constexpr int kCols = 64;                 // keys of a tile per warp
        constexpr int kLd = kCols / 32;           // tcgen05.ld x32 per tile
        const float cs = p.scale * kLog2e;        // exp(s*scale - M) = 2^(acc*cs - M*log2e)
        int j = 0;
        for_segments(p, c, [&](int k, const Seg &sg) {
            const int b = sg.pair % p.nblk;
            const int tok = b * p.tb + tok_in;
            const bool valid = row_ok && tok < p.n_new;
            const int64_t lim = valid ? p.n_past + tok : -1;   // last visible key
            float nM = 0.0f, inv = 0.0f;         // -M*log2e and 1/Z of the row (pass 2)
            if constexpr (OUT) {
                if (valid) {
                    const float2 st = p.rstat[(int64_t)sg.pair * 128 + row];
                    nM = -st.x * kLog2e;
                    inv = st.y;
                }
            }
            float am = -INFINITY, z = 0.0f;      // pass 1: running max of raw S, sum of exp
            for (int t = sg.t0; t < sg.t1; t++, j++) {
                const int sb = j & 1, pb = j & 1;
                if (sb != grp) continue;   // the other group's tile
                if (!mbar_wait_ab(&s_full[sb], (j >> 1) & 1, p.limit_ns, flags)) {
                    give_up(p, flags, 1u);
                    return false;
                }
                tc_fence_after();
                uint32_t v[kLd][32];
#pragma unroll
                for (int u = 0; u < kLd; u++) tmem_ld32(trow + sb * 128 + half * kCols + u * 32, v[u]);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[sb]);
                const int64_t kc0 = (int64_t)t * 128 + half * kCols;
                const int nvis = (int)max((int64_t)0, min((int64_t)kCols, lim - kc0 + 1));   // visible keys
                if constexpr (!OUT) {
                    float m8[8];   // eight independent max chains
#pragma unroll
                    for (int i = 0; i < 8; i++) m8[i] = -INFINITY;
                    if (nvis == kCols) {
#pragma unroll
                        for (int u = 0; u < kLd; u++)
#pragma unroll
                            for (int e = 0; e < 32; e++) m8[e & 7] = fmaxf(m8[e & 7], __uint_as_float(v[u][e]));
                    } else {
#pragma unroll
                        for (int u = 0; u < kLd; u++)
#pragma unroll
                            for (int e = 0; e < 32; e++)
                                if (u * 32 + e < nvis) m8[e & 7] = fmaxf(m8[e & 7], __uint_as_float(v[u][e]));
                    }
                    const float cm = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                                           fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
                    const float nm = fmaxf(am, cm);
                    if (nm != -INFINITY) {
                        const float nb = -nm * cs;
                        float a8[8] = {am == -INFINITY ? 0.0f : z * ex2_approx(fmaf(am, cs, nb)), 0.0f, 0.0f, 0.0f,
                                       0.0f, 0.0f, 0.0f, 0.0f};
                        if (nvis == kCols) {
#pragma unroll
                            for (int u = 0; u < kLd; u++)
#pragma unroll
                                for (int e = 0; e < 32; e++)
                                    a8[e & 7] += ex2_approx(fmaf(__uint_as_float(v[u][e]), cs, nb));
                        } else {
#pragma unroll
                            for (int u = 0; u < kLd; u++)
#pragma unroll
                                for (int e = 0; e < 32; e++) {
                                    const float x = ex2_approx(fmaf(__uint_as_float(v[u][e]), cs, nb));
                                    a8[e & 7] += u * 32 + e < nvis ? x : 0.0f;
                                }
                        }
                        z = ((a8[0] + a8[1]) + (a8[2] + a8[3])) + ((a8[4] + a8[5]) + (a8[6] + a8[7]));
                        am = nm;
                    }
                } else {
                    if (j >= 2 && !mbar_wait_ab(&p_empty[pb], ((j - 2) >> 1) & 1, p.limit_ns, flags)) {
                        give_up(p, flags, 1u);
                        return false;
                    }
#pragma unroll
                    for (int u = 0; u < kLd; u++) {
                        uint32_t pk[16];
#pragma unroll
                        for (int e = 0; e < 16; e++) {
                            float x0 = __fmul_rn(ex2_approx(fmaf(__uint_as_float(v[u][2 * e]), cs, nM)), inv);
                            float x1 = __fmul_rn(ex2_approx(fmaf(__uint_as_float(v[u][2 * e + 1]), cs, nM)), inv);
                            if (nvis < kCols) {
                                x0 = u * 32 + 2 * e < nvis ? x0 : 0.0f;
                                x1 = u * 32 + 2 * e + 1 < nvis ? x1 : 0.0f;
                            }
                            const __half2 h2 = __floats2half2_rn(x0, x1);
                            pk[e] = *reinterpret_cast<const uint32_t *>(&h2);
                        }
                        // keys part*kCols + u*32 .. +31 -> 16 packed columns of P[pb]
                        tmem_st16(trow + kTmP + pb * 64 + (half * kCols + u * 32) / 2, pk);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&p_full[pb]);
                }
            }
            if constexpr (!OUT) {
                // this part's (max, sum) of the row: max in scaled units
                float2 *ps = reinterpret_cast<float2 *>(p.pstat) + (((int64_t)c * p.kseg + k) * kCP + part) * 128 + row;
                *ps = make_float2(am == -INFINITY ? -INFINITY : __fmul_rn(am, p.scale), z);
            } else {
                if (!mbar_wait_ab(o_full, k & 1, p.limit_ns, flags)) {
                    give_up(p, flags, 1u);
                    return false;
                }
                tc_fence_after();
                constexpr int kOc = D / 4;     // output dims per warp of a lane quarter (16 or 32)
                const int oq = sw >> 2;        // 0..3
                float *po = p.pout + (((int64_t)c * p.kseg + k) * 128 + row) * D + oq * kOc;
#pragma unroll 1
                for (int ch = 0; ch < kOc / 16; ch++) {
                    uint32_t o[16];
                    tmem_ld16(trow + kTmO + oq * kOc + ch * 16, o);
                    tmem_wait_ld();
                    if (valid)
#pragma unroll
                        for (int q = 0; q < 4; q++)
                            *reinterpret_cast<uint4 *>(po + ch * 16 + 4 * q) =
                                make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(o_empty);
            }
            return true;
        });
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0 && lane == 0 && flags[0]) {
        // the CTA gave up: loads nobody waited for may still be landing
        for (int j = issued_k > KS ? issued_k - KS : 0; j < issued_k; j++)
            mbar_wait(&k_full[j % KS], (j / KS) & 1, p.limit_ns);
        if constexpr (OUT)
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
// folds
// ---------------------------------------------------------------------------
// CTAs [ca, cb] hold pair `pair`; its segment index in CTA cc
__device__ __forceinline__ void pair_ctas(const PrefillParams &p, int pair, int &ca, int &cb)
{
    const int64_t W = (int64_t)p.hkv * p.s_all;
    const int64_t x0 = pair_start(p, pair), x1 = x0 + nt_of(p, pair % p.nblk) - 1;
    auto cta_of = [&](int64_t x) {
        int cc = (int)min((int64_t)p.n_cta - 1, x * p.n_cta / W);
        while (cc + 1 < p.n_cta && cta_lo(p, cc + 1) <= x) cc++;
        while (cc > 0 && cta_lo(p, cc) > x) cc--;
        return cc;
    };
    ca = cta_of(x0);
    cb = cta_of(x1);
}

__device__ __forceinline__ int seg_index(const PrefillParams &p, int cc, int pair)
{
    return pair - pair_of(p, cta_lo(p, cc));
}

// (M, 1/Z) per (pair, row) from every segment part: one thread per row
__global__ void prefill_stats_fold(const PrefillParams p)
{
    const int pair = blockIdx.x, row = threadIdx.x;
    __shared__ int span[2];
    if (row == 0) pair_ctas(p, pair, span[0], span[1]);
    __syncthreads();
    const float2 *ps = reinterpret_cast<const float2 *>(p.pstat);
    float M = -INFINITY;
    for (int cc = span[0]; cc <= span[1]; cc++) {
        const int64_t base = ((int64_t)cc * p.kseg + seg_index(p, cc, pair)) * kCP;
        for (int q = 0; q < kCP; q++) M = fmaxf(M, ps[(base + q) * 128 + row].x);
    }
    double Z = 0.0;
    for (int cc = span[0]; cc <= span[1]; cc++) {
        const int64_t base = ((int64_t)cc * p.kseg + seg_index(p, cc, pair)) * kCP;
        for (int q = 0; q < kCP; q++) {
            const float2 v = ps[(base + q) * 128 + row];
            if (v.x != -INFINITY) Z += (double)v.y * (double)exp2f((v.x - M) * kLog2e);
        }
    }
    p.rstat[(int64_t)pair * 128 + row] = make_float2(M, Z > 0.0 ? __fdiv_rn(1.0f, (float)Z) : 0.0f);
}

// out = the sum of the pair's partial outputs (CTAs in order), scattered to the
// caller's [token][head][D] rows; one block per (pair, 8 rows), float4 per thread
__global__ void __launch_bounds__(256) prefill_out_fold(const PrefillParams p)
{
    const int pair = blockIdx.x >> 4, row0 = (blockIdx.x & 15) * 8;
    __shared__ int span[2];
    __shared__ int segi[160];
    if (threadIdx.x == 0) pair_ctas(p, pair, span[0], span[1]);
    __syncthreads();
    for (int cc = span[0] + (int)threadIdx.x; cc <= span[1]; cc += blockDim.x)
        if (cc - span[0] < 160) segi[cc - span[0]] = seg_index(p, cc, pair);
    __syncthreads();
    const int per_row = p.D / 4;
    const int b = pair % p.nblk, kvh = pair / p.nblk;
    for (int idx = threadIdx.x; idx < 8 * per_row; idx += blockDim.x) {
        const int row = row0 + idx / per_row, d4 = idx % per_row;
        const int tok_in = row / p.r, hd = row - tok_in * p.r;
        const int tok = b * p.tb + tok_in;
        if (tok_in >= p.tb || tok >= p.n_new) continue;
        float4 sum = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int cc = span[0]; cc <= span[1]; cc++) {
            const int sgi = cc - span[0] < 160 ? segi[cc - span[0]] : seg_index(p, cc, pair);
            const float4 v = __ldg(reinterpret_cast<const float4 *>(
                p.pout + (((int64_t)cc * p.kseg + sgi) * 128 + row) * p.D) + d4);
            sum.x += v.x;
            sum.y += v.y;
            sum.z += v.z;
            sum.w += v.w;
        }
        *reinterpret_cast<float4 *>(p.out + (int64_t)tok * p.out_stride + (int64_t)(p.out_head0 + kvh * p.r + hd) * p.D +
                                    4 * d4) = sum;
    }
}

template <int D>
cudaError_t prep_pf()
{
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel<D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)PL<D, false>::bytes);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(prefill_kernel<D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)PL<D, true>::bytes);
}

template <int D>
cudaError_t launch_pf(int which, const CUtensorMap &qmap, const CUtensorMap &kmap, const CUtensorMap &vmap,
                      const PrefillParams &p, cudaStream_t st)
{
    switch (which) {
    case 0:
        prefill_kernel<D, false><<<p.n_cta, kPThreads, PL<D, false>::bytes, st>>>(qmap, kmap, vmap, p);
        break;
    case 1: prefill_stats_fold<<<p.hkv * p.nblk, 128, 0, st>>>(p); break;
    case 2:
        prefill_kernel<D, true><<<p.n_cta, kPThreads, PL<D, true>::bytes, st>>>(qmap, kmap, vmap, p);
        break;
    default: prefill_out_fold<<<p.hkv * p.nblk * 16, 256, 0, st>>>(p); break;
    }
    return cudaGetLastError();
}

}  // namespace

bool prefill_supported(int D) { return D == 64 || D == 128; }
int prefill_max_segments() { return 4; }

cudaError_t prefill_prepare(int D)
{
    switch (D) {
    case 64: return prep_pf<64>();
    case 128: return prep_pf<128>();
    default: return cudaSuccess;
    }
}

cudaError_t launch_prefill(int D, int which, const CUtensorMap &qmap, const CUtensorMap &kmap,
                           const CUtensorMap &vmap, const PrefillParams &p, cudaStream_t st)
{
    switch (D) {
    case 64: return launch_pf<64>(which, qmap, kmap, vmap, p, st);
    case 128: return launch_pf<128>(which, qmap, kmap, vmap, p, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace kvb
