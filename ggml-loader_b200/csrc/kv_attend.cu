// kv_attend.cu -- decode attention of kv_attend: two TMA-fed, tensor-core,
// programmatic-dependent-launch kernels per layer.
//
// Numerics: the reference's default attention branch (src/model.cpp:1416-1445):
// scores = F16(q) . K accumulated in F32, softmax with the global max and sum,
// p = F16(expf(s - max) * (1/sum)), out = p . V accumulated in F32.  The two
// passes exist because ggml rounds the *normalised* p to F16 (its mul_mat
// converts the F32 operand), which needs the global max and sum first.
//
// Layout of the work: the layer's Hkv*n_kv (head, key) rows, head-major, are cut
// into C equal contiguous ranges, one CTA each (C <= SMs, C >= heads), so every
// SM streams the same number of bytes and a CTA spans at most two heads.
//
// attn_scores_kernel (pass 1)
//   * warp 8 streams 128-key tiles of K (64-wide boxes, 128-byte swizzle; 32-wide,
//     64-byte swizzle at head_dim 96) with cp.async.bulk.tensor into a 4-5 stage
//     mbarrier ring; warps 0-7 take 16 keys each and compute S = K . Q^T with
//     mma.m16n8k16 (F16 x F16 -> F32; the GQA group's query rows are N <= 8);
//   * decode (one new token): the kernel performs the append.  Each CTA rotates
//     (and RMS-normalises, qwen3) the query rows of both its heads up front, the
//     CTA that owns a head's new key rotates that K row, writes it to the cache
//     and patches it into its staged tile -- bit-identical to kv_append; the RoPE
//     entries are fetched before griddepcontrol.wait (the table is constant);
//   * writes the scaled scores and per-(CTA, segment, row) max / sum of exp.
// attn_pv_kernel (pass 2), a programmatic dependent of pass 1:
//   * its producer streams the V tiles of existing rows before
//     griddepcontrol.wait (V does not depend on pass 1), then the score tiles;
//   * folds the partial max/sum of its heads (host-computed CTA spans), forms
//     p = F16(expf(s-M)/Z) directly as the mma B fragment, O^T += V^T . P^T
//     (ldmatrix.trans); rows past the valid keys are zeroed first so stale rows
//     never reach the sum; writes the new V row (decode) and patches its tile;
//   * per-(CTA, segment) partial outputs; the last CTA of each head adds them in
//     CTA order (deterministic), all loads in flight, after its own loop.
// Every mbarrier wait is bounded (limit_ns): an expired wait sets the error word
// read by kv_status, and the CTA drains its own tile loads before leaving.
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

template <int D> struct G4;
template <> struct G4<64>  { static constexpr int BW = 64, NS1 = 8, NS2 = 6; };
template <> struct G4<96>  { static constexpr int BW = 32, NS1 = 5, NS2 = 4; };
template <> struct G4<128> { static constexpr int BW = 64, NS1 = 4, NS2 = 4; };

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

// index of the (CTA, segment) partial of local head h held by CTA cc
__device__ __forceinline__ int64_t part_slot(const AttnParams &p, int h, int cc)
{
    return (int64_t)cc * 2 + (cc == p.span_a[h] ? p.span_slot[h] : 0);
}

// ---- producer ----------------------------------------------------------------
template <int NS, class Issue>
__device__ void produce(int nt, int first, uint64_t *full, uint64_t *empty, volatile int *abort_flag,
                        const AttnParams &p, int &issued, Issue &&issue)
{
    for (int i = first; i < nt; i++) {
        if (p.inject == 1 && i == 1) break;   // test hook: withhold tile 1
        const int s = i % NS;
        if (i >= NS && !mbar_wait(&empty[s], ((i / NS) - 1) & 1, p.limit_ns)) {
            atomicOr(p.err, 2u);
            *abort_flag = 1;
            break;
        }
        if (*abort_flag) break;
        issue(i, s);
        issued = i + 1;
    }
}

template <int NS>
__device__ void drain(int issued, int nt, uint64_t *full, const AttnParams &p)
{
    if (issued < nt)  // leave no tile load in flight
        for (int j = issued > NS ? issued - NS : 0; j < issued; j++) mbar_wait(&full[j % NS], (j / NS) & 1, p.limit_ns);
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
__device__ void warp_rotate(const float *src, const float *gamma, const AttnParams &p, float *xs, float *tmp,
                            const float2 (&csr)[(D + 31) / 32])
{
    constexpr int E = (D + 31) / 32;
    const int lane = threadIdx.x & 31;
    float x[E], w[E];
#pragma unroll
    for (int e = 0; e < E; e++) {
        const int i = lane + 32 * e;
        x[e] = i < D ? __ldg(src + i) : 0.0f;
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

// ---------------------------------------------------------------------------
// pass 1
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads, 1) attn_scores_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                    const AttnParams p)
{
    constexpr int BW = G4<D>::BW, NB = D / BW, NS = G4<D>::NS1, KC = D / 16;
    constexpr uint32_t kSub = kTK * BW * 2, kStage = kSub * NB;

    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NS * kStage);
    uint64_t *empty = full + NS;
    float *red_m = reinterpret_cast<float *>(empty + NS);             // [2][8 warps][8 rows]
    float *red_z = red_m + 2 * 8 * kRows;
    float *qs = red_z + 2 * 8 * kRows;                                 // [2 heads][8 rows][D] rotated q
    float *tmp = qs + 2 * kRows * D;                                   // [8 warps][D]
    float *kf = tmp + 8 * D;                                           // [D] rotated new K row
    __half *knew = reinterpret_cast<__half *>(kf + D);                // [D] its F16 bits
    volatile int *abort_flag = reinterpret_cast<volatile int *>(knew + D);

    pdl_launch_dependents();
    const int c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Range g = cta_range(c, p.n_kv, p.hkv, p.n_cta);
    const bool two = g.nt > g.nt0;
    // decode: this CTA owns head h0's new key when its first segment ends the head
    const bool owns_new = p.fused && g.e0 == p.n_kv;
    const int it_new = owns_new ? (int)((p.n_past - g.s0) / kTK) : -1;

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
            int issued = 0;
            bool waited = false;
            produce<NS>(g.nt, 0, full, empty, abort_flag, p, issued, [&](int i, int s) {
                int h;
                int64_t k0, kend;
                tile_of(g, i, h, k0, kend);
                // rows >= n_past may come from the kernel before this one (a
                // multi-token append): only then is the wait needed
                if (!waited && !p.fused && k0 + kTK > p.n_past) {
                    pdl_wait();
                    waited = true;
                }
                mbar_arrive_expect_tx(&full[s], kStage);
#pragma unroll
                for (int b = 0; b < NB; b++)
                    tma_load_3d(smem + s * kStage + b * kSub, &kmap, &full[s], b * BW, h, (int)k0);
            });
            drain<NS>(issued, g.nt, full, p);
            if (!waited) pdl_wait();   // complete only after the previous kernel
        }
        return;
    }

    const int gq = lane >> 2, cq = lane & 3;
    const int R = p.nrows;
    const int row_a = 2 * cq, row_b = 2 * cq + 1;
    const int64_t lim_a = p.n_past + (p.row0 + min(row_a, R - 1)) / p.r;
    const int64_t lim_b = p.n_past + (p.row0 + min(row_b, R - 1)) / p.r;

    float2 csr[(D + 31) / 32];
    if (p.fused) rope_prefetch<D>(p, csr);
    pdl_wait();   // inputs, qbuf and the rows below may come from the previous kernel

    // decode: rotate the query rows of both heads and the new K row, one item per warp
    if (p.fused) {
        const int nq = R * (two ? 2 : 1);
        for (int it = warp; it < nq + (owns_new ? 1 : 0); it += 8) {
            if (it < nq) {
                const int hs = it / R, row = p.row0 + it % R;
                const float *src = p.q + (int64_t)(row / p.r) * p.q_stride +
                                   (int64_t)(p.hq0 + (g.h0 + hs) * p.r + row % p.r) * D;
                warp_rotate<D>(src, p.qk_norm ? p.q_norm_w : nullptr, p, qs + (hs * kRows + it % R) * D,
                               tmp + warp * D, csr);
            } else {
                warp_rotate<D>(p.k + (int64_t)(p.hkv0 + g.h0) * D, p.qk_norm ? p.k_norm_w : nullptr, p, kf,
                               tmp + warp * D, csr);
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
    const int mi = lane >> 3;
    const int arow = warp * 16 + (lane & 7) + (mi & 1) * 8;

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

        // (key gq, row 2cq), (key gq, row 2cq+1), (key gq+8, row 2cq), (key gq+8, row 2cq+1)
        const int64_t key0 = k0 + warp * 16 + gq, key1 = key0 + 8;
        const bool v0 = key0 < kend, v1 = key1 < kend;
        const float sa0 = v0 && key0 <= lim_a ? __fmul_rn(acc0[0] + acc1[0], p.scale) : -INFINITY;
        const float sb0 = v0 && key0 <= lim_b ? __fmul_rn(acc0[1] + acc1[1], p.scale) : -INFINITY;
        const float sa1 = v1 && key1 <= lim_a ? __fmul_rn(acc0[2] + acc1[2], p.scale) : -INFINITY;
        const float sb1 = v1 && key1 <= lim_b ? __fmul_rn(acc0[3] + acc1[3], p.scale) : -INFINITY;
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

    // (max, sum) per (segment, row): the 8 lanes of a row pair, then the 8 warps
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
    named_sync(1, kConsumers);
    if (tid < 2 * kRows) {
        const int sl = tid / kRows, row = tid % kRows;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; w++) M = fmaxf(M, red_m[(sl * 8 + w) * kRows + row]);
        double Z = 0.0;
#pragma unroll
        for (int w = 0; w < 8; w++) {
            const float mw = red_m[(sl * 8 + w) * kRows + row];
            if (mw != -INFINITY) Z += (double)red_z[(sl * 8 + w) * kRows + row] * (double)__expf(mw - M);
        }
        const int64_t pi = ((int64_t)c * 2 + sl) * kRows + row;
        p.part_m[pi] = M;
        p.part_z[pi] = Z;
    }
}

// ---------------------------------------------------------------------------
// pass 2
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads, 1) attn_pv_kernel(const __grid_constant__ CUtensorMap vmap,
                                                                const __grid_constant__ CUtensorMap smap,
                                                                const AttnParams p)
{
    constexpr int BW = G4<D>::BW, NB = D / BW, NS = G4<D>::NS2, DT = D / 16;
    constexpr int RED_LD = D + 4;
    constexpr uint32_t kSub = kTK * BW * 2, kStage = kSub * NB, kSBytes = kSPad * kRows * 4;

    extern __shared__ __align__(1024) unsigned char smem[];
    float *sring = reinterpret_cast<float *>(smem + NS * kStage);        // [NS][8][kSPad]
    float *red = sring + NS * kRows * kSPad;                             // [8 warps][8 rows][RED_LD]
    uint64_t *full = reinterpret_cast<uint64_t *>(red + 8 * kRows * RED_LD);
    uint64_t *empty = full + NS;
    float *rowM = reinterpret_cast<float *>(empty + NS);                // [2][8]
    float *rowInv = rowM + 2 * kRows;
    __half *vnew = reinterpret_cast<__half *>(rowInv + 2 * kRows);      // [D]
    volatile int *flags = reinterpret_cast<volatile int *>(vnew + D);   // abort, last(seg 0), last(seg 1)

    pdl_launch_dependents();
    const int c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Range g = cta_range(c, p.n_kv, p.hkv, p.n_cta);
    const bool two = g.nt > g.nt0;
    const int R = p.nrows;
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
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 8) {
        if (lane == 0) {
            prefetch_tmap(&vmap);
            prefetch_tmap(&smap);
            // V tiles of rows that existed before this step do not depend on the
            // previous kernel: stream them while it finishes
            int early = 0;
            while (early < g.nt && early < NS) {
                int h;
                int64_t k0, kend;
                tile_of(g, early, h, k0, kend);
                if (k0 + kTK > p.n_past || (p.inject == 1 && early == 1)) break;
                mbar_arrive_expect_tx(&full[early], kStage + kSBytes);
#pragma unroll
                for (int b = 0; b < NB; b++)
                    tma_load_3d(smem + early * kStage + b * kSub, &vmap, &full[early], b * BW, h, (int)k0);
                early++;
            }
            pdl_wait();   // scores and partials of pass 1 are now visible
            for (int i = 0; i < early; i++) {
                int h;
                int64_t k0, kend;
                tile_of(g, i, h, k0, kend);
                tma_load_2d(sring + i * kRows * kSPad, &smap, &full[i], (int)(k0 & ~(int64_t)3), h * kRows);
            }
            int issued = early;
            produce<NS>(g.nt, early, full, empty, flags, p, issued, [&](int i, int s) {
                int h;
                int64_t k0, kend;
                tile_of(g, i, h, k0, kend);
                mbar_arrive_expect_tx(&full[s], kStage + kSBytes);
#pragma unroll
                for (int b = 0; b < NB; b++)
                    tma_load_3d(smem + s * kStage + b * kSub, &vmap, &full[s], b * BW, h, (int)k0);
                tma_load_2d(sring + s * kRows * kSPad, &smap, &full[s], (int)(k0 & ~(int64_t)3), h * kRows);
            });
            drain<NS>(issued, g.nt, full, p);
        }
        return;
    }

    pdl_wait();
    // ---- global max and 1/sum of each (segment, query row): one warp per pair ----
    for (int pr = warp; pr < 2 * kRows; pr += 8) {
        const int sl = pr / kRows, row = pr % kRows;
        const int h = g.h0 + sl;
        float M = -INFINITY, Z = 0.0f;
        if (row < R && (sl == 0 || two)) {
            const int ca = p.span_a[h], cb = p.span_b[h];
            for (int cc = ca + lane; cc <= cb; cc += 32) M = fmaxf(M, p.part_m[part_slot(p, h, cc) * kRows + row]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            for (int cc = ca + lane; cc <= cb; cc += 32) {
                const int64_t pi = part_slot(p, h, cc) * kRows + row;
                const float mj = p.part_m[pi];
                if (mj != -INFINITY) Z += (float)p.part_z[pi] * __expf(mj - M);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) Z += __shfl_xor_sync(0xffffffffu, Z, o);
        }
        if (lane == 0) {
            rowM[sl * kRows + row] = M;
            rowInv[sl * kRows + row] = Z > 0.0f ? __fdiv_rn(1.0f, Z) : 0.0f;
        }
    }
    // decode: the new V row of head h0 goes to the cache and into its tile
    if (owns_new && warp == 7) {
        const float *src = p.v + (int64_t)(p.hkv0 + g.h0) * D;
        __half *dst = p.vc + (p.n_past * (int64_t)p.hkv + g.h0) * D;
        for (int i = lane; i < D; i += 32) {
            const __half h16 = __float2half_rn(__ldg(src + i));
            vnew[i] = h16;
            dst[i] = h16;
        }
    }
    named_sync(1, kConsumers);

    const int gq = lane >> 2, cq = lane & 3;
    float oacc[DT][4];
#pragma unroll
    for (int dt = 0; dt < DT; dt++) oacc[dt][0] = oacc[dt][1] = oacc[dt][2] = oacc[dt][3] = 0.0f;
    bool aborted = false;
    const uint32_t ring = smem_addr(smem);

    // this CTA's partial of segment sl into part_o; flags[1+sl] = last CTA of the head
    auto write_partial = [&](int sl) -> bool {
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
        if (tid == 0)
            flags[1 + sl] = atomicAdd(&p.counters[h], 1u) == (unsigned)(p.span_b[h] - p.span_a[h]);
        named_sync(1, kConsumers);
        return true;
    };

    // the head's last CTA: sum its CTAs' partials in CTA order, every load in flight
    auto combine = [&](int h) {
        __threadfence();
        const int ca = p.span_a[h], n = p.span_b[h] - ca + 1;
        const int64_t cstride = (int64_t)2 * kRows * D;
        for (int idx = tid; idx < R * D; idx += kConsumers) {
            const int row = idx / D, dd = idx - row * D;
            const float *src = p.part_o + (int64_t)row * D + dd;
            float sum = __ldcg(src + part_slot(p, h, ca) * kRows * D);
            for (int base = 1; base < n; base += 16) {
                float x[16];
#pragma unroll
                for (int u = 0; u < 16; u++) x[u] = base + u < n ? __ldcg(src + (int64_t)(ca + base + u) * cstride) : 0.0f;
#pragma unroll
                for (int u = 0; u < 16; u++) sum += x[u];
            }
            const int qrow = p.row0 + row;
            p.out[(int64_t)(qrow / p.r) * p.out_stride + (int64_t)(p.out_head0 + h * p.r + qrow % p.r) * D + dd] = sum;
        }
        if (tid == 0) p.counters[h] = 0u;
    };

    for (int i = 0; i < g.nt; i++) {
        if (i == g.nt0 && i > 0) write_partial(0);
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
    if (g.nt > 0 && write_partial(two ? 1 : 0)) {
        if (flags[1]) combine(g.h0);
        if (two && flags[2]) combine(g.h0 + 1);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int D>
size_t smem1()
{
    constexpr int BW = G4<D>::BW, NB = D / BW, NS = G4<D>::NS1;
    return (size_t)NS * kTK * BW * 2 * NB + 2 * NS * 8 + 2 * 2 * 8 * kRows * 4 + (size_t)(2 * kRows + 8 + 1) * D * 4 +
           (size_t)D * 2 + 16;
}

template <int D>
size_t smem2()
{
    constexpr int BW = G4<D>::BW, NB = D / BW, NS = G4<D>::NS2;
    return (size_t)NS * kTK * BW * 2 * NB + (size_t)NS * kRows * kSPad * 4 + (size_t)8 * kRows * (D + 4) * 4 +
           2 * NS * 8 + 4 * kRows * 4 + (size_t)D * 2 + 32;
}

template <int D>
cudaError_t prep()
{
    cudaError_t e =
        cudaFuncSetAttribute(attn_scores_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1<D>());
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(attn_pv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2<D>());
}

template <int D>
cudaError_t launch(int which, const CUtensorMap &kmap, const CUtensorMap &vmap, const CUtensorMap &smap,
                   const AttnParams &p, cudaStream_t st, bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)p.n_cta);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (which == 0) {
        cfg.dynamicSmemBytes = smem1<D>();
        return cudaLaunchKernelEx(&cfg, attn_scores_kernel<D>, kmap, p);
    }
    cfg.dynamicSmemBytes = smem2<D>();
    return cudaLaunchKernelEx(&cfg, attn_pv_kernel<D>, vmap, smap, p);
}

}  // namespace

int attn_rows() { return kRows; }
int attn_tile_keys() { return kTK; }
int attn_box_width(int D) { return D == 96 ? 32 : 64; }

cudaError_t attn_prepare(int D)
{
    switch (D) {
    case 64: return prep<64>();
    case 96: return prep<96>();
    case 128: return prep<128>();
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_attn(int D, int which, const CUtensorMap &kmap, const CUtensorMap &vmap, const CUtensorMap &smap,
                        const AttnParams &p, cudaStream_t st, bool pdl)
{
    if (p.nrows < 1 || p.nrows > kRows) return cudaErrorInvalidValue;
    switch (D) {
    case 64: return launch<64>(which, kmap, vmap, smap, p, st, pdl);
    case 96: return launch<96>(which, kmap, vmap, smap, p, st, pdl);
    case 128: return launch<128>(which, kmap, vmap, smap, p, st, pdl);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace kvb
