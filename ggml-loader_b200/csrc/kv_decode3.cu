// kv_decode3.cu -- decode attention for kv_attend: TMA-fed, tensor-core dot
// products, two passes.
//
// Same contract and numerics as the reference's default attention branch
// (src/model.cpp:1416-1445): scores = F16(q) . K in F32, softmax with the
// global max and a double sum, p rounded to F16, out = p . V in F32.  Two
// passes reproduce ggml's F16 rounding of the *normalised* p (see kv_decode.cu).
//
//  * Balanced persistent split: the layer's Hkv*n_kv (head, key) rows, head-
//    major, are cut into C equal contiguous ranges, one CTA each (C = SMs, or
//    fewer for short contexts, never fewer than the heads), so a CTA spans at
//    most two heads ("segments").
//  * TMA ring: warp 8 issues cp.async.bulk.tensor loads of 128-key tiles of one
//    head (64-wide column boxes with 128-byte swizzle; 32-wide with 64-byte
//    swizzle for head_dim 96) into an mbarrier-tracked ring of 96-128 KiB.
//  * The dot products run on the tensor cores as warp-level
//    mma.m16n8k16 (F16 x F16 -> F32): the r query rows of the GQA group (<= 8)
//    are the N=8 side, 16 keys per warp the M side, fed from the swizzled tiles
//    with ldmatrix.  F16 operands with F32 accumulation are exactly the
//    reference's mul_mat semantics (it converts Q and p to F16 too).
//  * Pass 1 (scores3): S = K.Q^T per warp block; lanes write their scaled scores
//    and keep running (max, sum exp) per query row; per-(CTA, segment) partials.
//  * Pass 2 (pv3): each lane forms its own B fragment p = F16(expf(s - max) *
//    (1/sum)) from the score tile that arrived with the V tile, and
//    O^T += V^T . P^T (V through ldmatrix.trans).  Rows past the valid keys of
//    a partial tile are zeroed in shared memory first so stale cache rows can
//    never reach the sum.  Per (CTA, segment) partial outputs; the last CTA of
//    each head adds them in CTA order (deterministic).
//  * Every mbarrier wait is bounded; an expired wait sets the error word
//    (kv_status) and the CTA leaves after draining its own tile loads.
#include <math.h>

#include "kv_internal.h"
#include "kv_sm100.cuh"

namespace kvb {
namespace {

using namespace sm100;

constexpr int kTK = 128;         // keys per tile (8 warps x 16)
constexpr int kConsumers = 256;  // warps 0-7
constexpr int kThreads = 288;    // + producer warp 8
constexpr int kRows = 8;         // query rows per launch (mma N) and scratch row stride
constexpr int kSPad = kTK + 4;   // score tile: x rounded down to 4 floats

template <int D> struct G3;
template <> struct G3<64>  { static constexpr int BW = 64, NS1 = 8, NS2 = 7; };
template <> struct G3<96>  { static constexpr int BW = 32, NS1 = 5, NS2 = 4; };
template <> struct G3<128> { static constexpr int BW = 64, NS1 = 4, NS2 = 4; };

// byte offset of (row, 16-byte chunk) inside one swizzled box of BW halves
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

__device__ __forceinline__ int64_t cta_lo(int64_t c, int64_t T, int64_t C) { return c * T / C; }

__device__ __forceinline__ Range cta_range(int c, int64_t n_kv, int hkv, int C)
{
    const int64_t T = (int64_t)hkv * n_kv;
    const int64_t lo = cta_lo(c, T, C), hi = cta_lo(c + 1, T, C);
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

__device__ __forceinline__ int cta_of(int64_t x, int64_t T, int C)
{
    int c = (int)(x * C / T);
    if (c >= C) c = C - 1;
    while (c + 1 < C && cta_lo(c + 1, T, C) <= x) c++;
    while (c > 0 && cta_lo(c, T, C) > x) c--;
    return c;
}

// CTAs [ca, cb] cover head h; all but possibly ca start inside h (segment 0);
// ca's segment for h is 1 when ca starts in the previous head.
struct HeadSpan {
    int ca, cb, slot_ca;
};

__device__ __forceinline__ HeadSpan head_span(int h, int64_t n_kv, int64_t T, int C)
{
    HeadSpan s;
    s.ca = cta_of((int64_t)h * n_kv, T, C);
    s.cb = cta_of((int64_t)(h + 1) * n_kv - 1, T, C);
    s.slot_ca = cta_lo(s.ca, T, C) < (int64_t)h * n_kv ? 1 : 0;
    return s;
}

__device__ __forceinline__ void merge_stats(float &m, double &z, float m2, double z2)
{
    if (m2 == -INFINITY) return;
    if (m == -INFINITY) { m = m2; z = z2; return; }
    if (m2 > m) { z = z * exp((double)m - (double)m2) + z2; m = m2; }
    else z += z2 * exp((double)m2 - (double)m);
}

// ---- producer ----------------------------------------------------------------
template <int NS, class Issue>
__device__ void produce(const Range &g, uint64_t *full, uint64_t *empty, volatile int *abort_flag,
                        const DecodeParams &p, Issue &&issue)
{
    int issued = 0;
    for (int i = 0; i < g.nt; i++) {
        if (p.inject == 1 && i == 1) break;   // test hook: withhold tile 1
        const int s = i % NS;
        if (i >= NS && !mbar_wait(&empty[s], ((i / NS) - 1) & 1, p.limit_ns)) {
            atomicOr(p.err, 2u);
            *abort_flag = 1;
            break;
        }
        if (*abort_flag) break;
        issue(i, s);
        issued++;
    }
    if (issued < g.nt)  // leave no tile load in flight
        for (int j = issued > NS ? issued - NS : 0; j < issued; j++) mbar_wait(&full[j % NS], (j / NS) & 1, p.limit_ns);
}

// ---------------------------------------------------------------------------
// pass 1: scores
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads, 1) scores3_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                const DecodeParams p)
{
    constexpr int BW = G3<D>::BW, NB = D / BW, NS = G3<D>::NS1, KC = D / 16;
    constexpr uint32_t kSub = kTK * BW * 2, kStage = kSub * NB;

    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NS * kStage);
    uint64_t *empty = full + NS;
    double *red_z = reinterpret_cast<double *>(empty + NS);        // [2][8 warps][8 rows]
    float *red_m = reinterpret_cast<float *>(red_z + 2 * 8 * kRows);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(red_m + 2 * 8 * kRows);

    const int c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Range g = cta_range(c, p.n_kv, p.hkv, p.n_cta);

    if (tid == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 8);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 8) {
        if (lane == 0) {
            prefetch_tmap(&kmap);
            produce<NS>(g, full, empty, abort_flag, p, [&](int i, int s) {
                int h;
                int64_t k0, kend;
                tile_of(g, i, h, k0, kend);
                mbar_arrive_expect_tx(&full[s], kStage);
#pragma unroll
                for (int b = 0; b < NB; b++)
                    tma_load_3d(smem + s * kStage + b * kSub, &kmap, &full[s], b * BW, h, (int)k0);
            });
        }
        return;
    }

    const int gq = lane >> 2, cq = lane & 3;    // fragment row group / column pair
    const int R = p.nrows;
    const int row_a = 2 * cq, row_b = 2 * cq + 1;
    const int64_t lim_a = p.n_past + (p.row0 + min(row_a, R - 1)) / p.r;
    const int64_t lim_b = p.n_past + (p.row0 + min(row_b, R - 1)) / p.r;

    // B fragments: Q^T, column n = query row gq, k = dims
    uint32_t bq[KC][2];
    auto load_q = [&](int h) {
        const bool ok = gq < R;
        const int row = p.row0 + (ok ? gq : 0);
        const __half *qrow = p.qbuf + ((int64_t)(row / p.r) * p.hq_loc + (int64_t)h * p.r + row % p.r) * D;
#pragma unroll
        for (int kc = 0; kc < KC; kc++) {
            const uint32_t lo = *reinterpret_cast<const uint32_t *>(qrow + kc * 16 + 2 * cq);
            const uint32_t hi = *reinterpret_cast<const uint32_t *>(qrow + kc * 16 + 2 * cq + 8);
            bq[kc][0] = ok ? lo : 0u;
            bq[kc][1] = ok ? hi : 0u;
        }
    };
    load_q(g.h0);

    float ma = -INFINITY, mb = -INFINITY, ma0 = -INFINITY, mb0 = -INFINITY;
    double za = 0.0, zb = 0.0, za0 = 0.0, zb0 = 0.0;
    bool aborted = false;
    const uint32_t ring = smem_addr(smem);

    auto upd = [&](float &m, double &z, float s0, float s1) {
        const float lm = fmaxf(s0, s1);
        if (lm == -INFINITY) return;
        if (lm > m) {
            if (m != -INFINITY) z *= (double)expf(m - lm);
            m = lm;
        }
        z += (double)expf(s0 - m) + (double)expf(s1 - m);
    };

    for (int i = 0; i < g.nt; i++) {
        if (i == g.nt0) {
            ma0 = ma; mb0 = mb; za0 = za; zb0 = zb;
            ma = mb = -INFINITY;
            za = zb = 0.0;
            load_q(g.h0 + 1);
        }
        const int s = i % NS;
        const bool ok = mbar_wait(&full[s], (i / NS) & 1, p.limit_ns);
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) {
                atomicOr(p.err, 1u);
                *abort_flag = 1;
            }
            aborted = true;
            break;
        }
        int h;
        int64_t k0, kend;
        tile_of(g, i, h, k0, kend);

        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int mi = lane >> 3;
        const int arow = warp * 16 + (lane & 7) + (mi & 1) * 8;
#pragma unroll
        for (int kc = 0; kc < KC; kc++) {
            const int dim0 = kc * 16 + (mi >> 1) * 8;
            const uint32_t addr = ring + s * kStage + (dim0 / BW) * kSub + swz<BW>(arow, (dim0 % BW) >> 3);
            uint32_t a0, a1, a2, a3;
            ldsm_x4(addr, a0, a1, a2, a3);
            mma_16816(acc, a0, a1, a2, a3, bq[kc][0], bq[kc][1]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);

        // acc: (key gq, row 2cq), (key gq, row 2cq+1), (key gq+8, row 2cq), (key gq+8, row 2cq+1)
        const int64_t key0 = k0 + warp * 16 + gq, key1 = key0 + 8;
        const bool v0 = key0 < kend, v1 = key1 < kend;
        const float sa0 = v0 && key0 <= lim_a ? __fmul_rn(acc[0], p.scale) : -INFINITY;
        const float sb0 = v0 && key0 <= lim_b ? __fmul_rn(acc[1], p.scale) : -INFINITY;
        const float sa1 = v1 && key1 <= lim_a ? __fmul_rn(acc[2], p.scale) : -INFINITY;
        const float sb1 = v1 && key1 <= lim_b ? __fmul_rn(acc[3], p.scale) : -INFINITY;
        float *Sa = p.S + ((int64_t)h * kRows + row_a) * p.S_stride;
        float *Sb = Sa + p.S_stride;
        if (row_a < R) {
            if (v0) Sa[key0] = sa0;
            if (v1) Sa[key1] = sa1;
            upd(ma, za, sa0, sa1);
        }
        if (row_b < R) {
            if (v0) Sb[key0] = sb0;
            if (v1) Sb[key1] = sb1;
            upd(mb, zb, sb0, sb1);
        }
    }

    // merge the 8 lanes of each row pair, then the 8 warps
    const bool two = g.nt > g.nt0;
    float m_s[2][2] = {{two ? ma0 : ma, two ? mb0 : mb}, {ma, mb}};
    double z_s[2][2] = {{two ? za0 : za, two ? zb0 : zb}, {za, zb}};
#pragma unroll
    for (int sl = 0; sl < 2; sl++)
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            float m = aborted ? -INFINITY : m_s[sl][rr];
            double z = aborted ? 0.0 : z_s[sl][rr];
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
                const double z2 = __shfl_xor_sync(0xffffffffu, z, o);
                merge_stats(m, z, m2, z2);
            }
            if (gq == 0) {
                red_m[(sl * 8 + warp) * kRows + 2 * cq + rr] = m;
                red_z[(sl * 8 + warp) * kRows + 2 * cq + rr] = z;
            }
        }
    named_sync(1, kConsumers);
    if (tid < 2 * kRows) {
        const int sl = tid / kRows, row = tid % kRows;
        float M = -INFINITY;
        double Z = 0.0;
        for (int w = 0; w < 8; w++) merge_stats(M, Z, red_m[(sl * 8 + w) * kRows + row], red_z[(sl * 8 + w) * kRows + row]);
        const int64_t pi = ((int64_t)c * 2 + sl) * kRows + row;
        p.part_m[pi] = M;
        p.part_z[pi] = Z;
    }
}

// ---------------------------------------------------------------------------
// pass 2: P.V
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads, 1) pv3_kernel(const __grid_constant__ CUtensorMap vmap,
                                                            const __grid_constant__ CUtensorMap smap,
                                                            const DecodeParams p)
{
    constexpr int BW = G3<D>::BW, NB = D / BW, NS = G3<D>::NS2, DT = D / 16;
    constexpr int RED_LD = D + 4;                          // padded row of the cross-warp sum
    constexpr uint32_t kSub = kTK * BW * 2, kStage = kSub * NB, kSBytes = kSPad * kRows * 4;

    extern __shared__ __align__(1024) unsigned char smem[];
    float *sring = reinterpret_cast<float *>(smem + NS * kStage);        // [NS][8][kSPad]
    float *red = sring + NS * kRows * kSPad;                             // [8 warps][8 rows][RED_LD]
    uint64_t *full = reinterpret_cast<uint64_t *>(red + 8 * kRows * RED_LD);
    uint64_t *empty = full + NS;
    float *rowM = reinterpret_cast<float *>(empty + NS);                // [2][8]
    float *rowInv = rowM + 2 * kRows;
    volatile int *flags = reinterpret_cast<volatile int *>(rowInv + 2 * kRows);  // abort, last, ca, cb, slot_ca

    const int c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Range g = cta_range(c, p.n_kv, p.hkv, p.n_cta);
    const int64_t T = (int64_t)p.hkv * p.n_kv;
    const int R = p.nrows;

    if (tid == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 8);
        }
        flags[0] = 0;
        flags[1] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 8) {
        if (lane == 0) {
            prefetch_tmap(&vmap);
            prefetch_tmap(&smap);
            produce<NS>(g, full, empty, flags, p, [&](int i, int s) {
                int h;
                int64_t k0, kend;
                tile_of(g, i, h, k0, kend);
                mbar_arrive_expect_tx(&full[s], kStage + kSBytes);
#pragma unroll
                for (int b = 0; b < NB; b++)
                    tma_load_3d(smem + s * kStage + b * kSub, &vmap, &full[s], b * BW, h, (int)k0);
                tma_load_2d(sring + s * kRows * kSPad, &smap, &full[s], (int)(k0 & ~(int64_t)3), h * kRows);
            });
        }
        return;
    }

    // ---- global max and 1/sum of each (segment, query row) ----
    for (int pr = warp; pr < 2 * kRows; pr += 8) {
        const int sl = pr / kRows, row = pr % kRows;
        const int h = g.h0 + sl;
        float M = -INFINITY;
        double Z = 0.0;
        if (row < R && (sl == 0 || g.nt > g.nt0)) {
            const HeadSpan hs = head_span(h, p.n_kv, T, p.n_cta);
            for (int cc = hs.ca + lane; cc <= hs.cb; cc += 32) {
                const int64_t pi = ((int64_t)cc * 2 + (cc == hs.ca ? hs.slot_ca : 0)) * kRows + row;
                merge_stats(M, Z, p.part_m[pi], p.part_z[pi]);
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float m2 = __shfl_xor_sync(0xffffffffu, M, o);
                const double z2 = __shfl_xor_sync(0xffffffffu, Z, o);
                merge_stats(M, Z, m2, z2);
            }
        }
        if (lane == 0) {
            rowM[sl * kRows + row] = M;
            rowInv[sl * kRows + row] = Z > 0.0 ? (float)(1.0 / Z) : 0.0f;
        }
    }
    named_sync(1, kConsumers);

    const int gq = lane >> 2, cq = lane & 3;
    float oacc[DT][4];
#pragma unroll
    for (int dt = 0; dt < DT; dt++) oacc[dt][0] = oacc[dt][1] = oacc[dt][2] = oacc[dt][3] = 0.0f;
    bool aborted = false;
    const uint32_t ring = smem_addr(smem);

    // sum this CTA's warps into part_o[c][sl]; the head's last CTA writes out
    auto flush = [&](int sl) -> bool {
        if (named_sync_or(1, kConsumers, aborted)) return false;
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
        for (int idx = tid; idx < R * D; idx += kConsumers) {
            const int row = idx / D, dd = idx - row * D;
            float sum = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; w++) sum += red[(w * kRows + row) * RED_LD + dd];
            p.part_o[(((int64_t)c * 2 + sl) * kRows + row) * D + dd] = sum;
        }
        __threadfence();
        named_sync(1, kConsumers);
        if (tid == 0) {
            const HeadSpan hs = head_span(h, p.n_kv, T, p.n_cta);
            flags[1] = atomicAdd(&p.counters[h], 1u) == (unsigned)(hs.cb - hs.ca);
            flags[2] = hs.ca;
            flags[3] = hs.cb;
            flags[4] = hs.slot_ca;
        }
        named_sync(1, kConsumers);
        if (flags[1]) {
            __threadfence();
            const int ca = flags[2], cb = flags[3], sca = flags[4];
            for (int idx = tid; idx < R * D; idx += kConsumers) {
                const int row = idx / D, dd = idx - row * D;
                const float *src = p.part_o + (int64_t)row * D + dd;
                float sum = __ldcg(src + ((int64_t)ca * 2 + sca) * kRows * D);
                int cc = ca + 1;
                for (; cc + 3 <= cb; cc += 4) {   // four independent loads in flight
                    const float x0 = __ldcg(src + (int64_t)(cc + 0) * 2 * kRows * D);
                    const float x1 = __ldcg(src + (int64_t)(cc + 1) * 2 * kRows * D);
                    const float x2 = __ldcg(src + (int64_t)(cc + 2) * 2 * kRows * D);
                    const float x3 = __ldcg(src + (int64_t)(cc + 3) * 2 * kRows * D);
                    sum += x0;
                    sum += x1;
                    sum += x2;
                    sum += x3;
                }
                for (; cc <= cb; cc++) sum += __ldcg(src + (int64_t)cc * 2 * kRows * D);
                const int qrow = p.row0 + row;
                p.out[(int64_t)(qrow / p.r) * p.out_stride + (int64_t)(p.out_head0 + h * p.r + qrow % p.r) * D + dd] =
                    sum;
            }
            if (tid == 0) p.counters[h] = 0u;
        }
        named_sync(1, kConsumers);
        return true;
    };

    bool flushed_ok = true;
    for (int i = 0; i < g.nt; i++) {
        if (i == g.nt0 && i > 0) flushed_ok = flush(0) && flushed_ok;
        if (aborted) continue;   // keep step with the other warps' barriers
        const int s = i % NS;
        const bool ok = mbar_wait(&full[s], (i / NS) & 1, p.limit_ns);
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

        // rows past the valid keys may hold stale cache contents: zero them so
        // that 0 * (anything) cannot reach the sum
        if (kw + 16 > n_valid) {
            const int zr0 = max(kw, n_valid);
            constexpr int CPR = BW / 8;   // 16-byte chunks per box row
            for (int idx = lane; idx < (kw + 16 - zr0) * NB * CPR; idx += 32) {
                const int rr = zr0 + idx / (NB * CPR), rest = idx % (NB * CPR);
                uint4 *dst = reinterpret_cast<uint4 *>(smem + s * kStage + (rest / CPR) * kSub +
                                                       (BW == 64 ? rr * 128 : rr * 64) + (rest % CPR) * 16);
                *dst = make_uint4(0u, 0u, 0u, 0u);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
        }

        // B fragment: p for query row gq, keys kw + {2cq, 2cq+1, 2cq+8, 2cq+9}
        const float *st = sring + s * kRows * kSPad + (k0 & 3) + gq * kSPad;
        const float M = rowM[sl * kRows + gq], inv = rowInv[sl * kRows + gq];
        __half pv[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int kk = kw + 2 * cq + (e & 1) + 8 * (e >> 1);
            const bool valid = gq < R && kk < n_valid;
            const float pe = __fmul_rn(expf(st[kk] - M), inv);
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
    if (g.nt > 0) flush(g.nt > g.nt0 ? 1 : 0);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int D>
size_t smem1()
{
    constexpr int BW = G3<D>::BW, NB = D / BW, NS = G3<D>::NS1;
    return (size_t)NS * kTK * BW * 2 * NB + 2 * NS * 8 + 2 * 8 * kRows * (8 + 4) + 16;
}

template <int D>
size_t smem2()
{
    constexpr int BW = G3<D>::BW, NB = D / BW, NS = G3<D>::NS2;
    return (size_t)NS * kTK * BW * 2 * NB + (size_t)NS * kRows * kSPad * 4 + (size_t)8 * kRows * (D + 4) * 4 +
           2 * NS * 8 + 4 * kRows * 4 + 32;
}

template <int D>
cudaError_t prep()
{
    cudaError_t e = cudaFuncSetAttribute(scores3_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1<D>());
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(pv3_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2<D>());
}

template <int D>
cudaError_t launch(int which, const CUtensorMap &kmap, const CUtensorMap &vmap, const CUtensorMap &smap,
                   const DecodeParams &p, cudaStream_t st)
{
    if (which == 0) scores3_kernel<D><<<p.n_cta, kThreads, smem1<D>(), st>>>(kmap, p);
    else pv3_kernel<D><<<p.n_cta, kThreads, smem2<D>(), st>>>(vmap, smap, p);
    return cudaGetLastError();
}

}  // namespace

int decode3_rows() { return kRows; }
int decode3_tile_keys() { return kTK; }
int decode3_box_width(int D) { return D == 96 ? 32 : 64; }

cudaError_t decode3_prepare(int D)
{
    switch (D) {
    case 64: return prep<64>();
    case 96: return prep<96>();
    case 128: return prep<128>();
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_decode3(int D, int which, const CUtensorMap &kmap, const CUtensorMap &vmap,
                           const CUtensorMap &smap, const DecodeParams &p, cudaStream_t st)
{
    if (p.nrows < 1 || p.nrows > kRows) return cudaErrorInvalidValue;
    switch (D) {
    case 64: return launch<64>(which, kmap, vmap, smap, p, st);
    case 96: return launch<96>(which, kmap, vmap, smap, p, st);
    case 128: return launch<128>(which, kmap, vmap, smap, p, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace kvb
