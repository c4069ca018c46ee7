// kv_decode.cu -- split-K decode attention on the CUDA cores, two passes.
//
// Replaces the reference's default attention branch (src/model.cpp:1416-1445):
//   KQ  = ggml_mul_mat(K, Q)                      F16 K . F16(Q), F32 accumulate
//   KQ  = ggml_soft_max_ext(KQ, mask, 1/sqrt(d))  w = s*scale (+mask); e = expf(w-max);
//                                                 p = e * (float)(1/sum_double(e))
//   KQV = ggml_mul_mat(cont(V^T), KQ)             F16 V . F16(p), F32 accumulate
// The V transpose copy (model.cpp:1439-1440) is not needed: V is read in place.
//
// Why two passes.  ggml rounds the NORMALISED probabilities p to F16 before the
// P.V product (mul_mat converts its F32 src1 to F16).  At long context p is
// ~1/n_kv, inside F16's subnormal range, so that rounding is a visible part of
// the reference's numerics (~1e-3 relative at 128k).  A one-pass online softmax
// cannot reproduce it (p is unknown until the global max and sum are), so:
//   pass 1 (scores_kernel): one CTA per (KV-head, key split).  Streams the split's
//     K rows once for all r query heads of the GQA group, writes the scaled
//     scores S (F32) and the split's (max, sum exp) partials.
//   pass 2 (pv_kernel): same grid.  Folds the partials into the global (max, sum)
//     per query row, forms p = F16(expf(S - max) * (1/sum)) exactly as the
//     reference, streams the split's V rows once for the group, and writes a
//     partial output; the last CTA of each KV head to finish sums the partials
//     in split order (deterministic) into `out`.
// Scores and partials are < 4% of the K/V bytes; K and V are each read once.
//
// Thread mapping (scores): LPK lanes share a key row, each owning CH 16-byte
// chunks (8 halves), so every warp load instruction covers whole 128-byte
// segments; the LPK partial dots are combined with xor-shuffles.
// Thread mapping (P.V): D/8 lanes own a V row's 16-byte chunks; 32/(D/8) rows
// per warp per step; the r output rows accumulate in registers.
#include <math.h>

#include "kv_internal.h"

namespace kvb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 4;

template <int D> struct Shape;
template <> struct Shape<64>  { static constexpr int CH = 1, RMAX = 8, SPLIT_MAX = 1024; };
template <> struct Shape<96>  { static constexpr int CH = 3, RMAX = 4, SPLIT_MAX = 2048; };
template <> struct Shape<128> { static constexpr int CH = 2, RMAX = 4, SPLIT_MAX = 2048; };

__device__ __forceinline__ uint4 ld_stream(const void *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ void unpack8(const uint4 &u, float f[8])
{
    const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const float2 v = __half22float2(h[e]);
        f[2 * e] = v.x;
        f[2 * e + 1] = v.y;
    }
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ double warp_sum(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// pass 1
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads) scores_kernel(const ScoresParams p)
{
    constexpr int CH = Shape<D>::CH, RMAX = Shape<D>::RMAX;
    constexpr int LPK = D / 8 / CH;      // lanes per key row
    constexpr int KPW = 32 / LPK;        // key rows per warp step
    constexpr int KPB = kWarps * KPW;    // key rows per block step
    static_assert(RMAX <= LPK, "lane j stores row j");
    extern __shared__ float smem[];
    float *qs = smem;                    // [RMAX][D]
    float *ss = smem + RMAX * D;         // [RMAX][split_len]

    const int h = blockIdx.y, s = blockIdx.x;
    const int64_t k0 = (int64_t)s * p.split_len;
    const int64_t k1 = min(k0 + (int64_t)p.split_len, p.n_kv);
    const int len = (int)(k1 - k0);
    const int R = p.nrows;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    for (int idx = tid; idx < RMAX * D; idx += kThreads) {
        const int i = idx / D, dd = idx % D;
        float v = 0.0f;
        if (i < R) {
            const int row = p.row0 + i;
            const int t = row / p.r, jj = row % p.r;
            v = __half2float(p.qbuf[((int64_t)t * p.hq_loc + (int64_t)h * p.r + jj) * D + dd]);
        }
        qs[idx] = v;
    }
    __syncthreads();

    const int j = lane % LPK, g = lane / LPK;
    float qr[RMAX][CH * 8];
#pragma unroll
    for (int i = 0; i < RMAX; i++)
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int e = 0; e < 8; e++) qr[i][c * 8 + e] = qs[i * D + (j + c * LPK) * 8 + e];
    int64_t lim[RMAX];
#pragma unroll
    for (int i = 0; i < RMAX; i++) lim[i] = p.n_past + (p.row0 + i) / p.r;

    const __half *kbase = p.kc + (int64_t)h * D;
    for (int base = 0; base < len; base += KPB * kUnroll) {
        uint4 kv[kUnroll][CH];
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            const int kk = base + u * KPB + warp * KPW + g;
            if (kk < len) {
                const __half *row = kbase + (k0 + kk) * (int64_t)p.row_elems;
#pragma unroll
                for (int c = 0; c < CH; c++) kv[u][c] = ld_stream(row + (j + c * LPK) * 8);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            const int kk = base + u * KPB + warp * KPW + g;
            float acc[RMAX];
#pragma unroll
            for (int i = 0; i < RMAX; i++) acc[i] = 0.0f;
            if (kk < len) {
#pragma unroll
                for (int c = 0; c < CH; c++) {
                    float kf[8];
                    unpack8(kv[u][c], kf);
#pragma unroll
                    for (int i = 0; i < RMAX; i++)
#pragma unroll
                        for (int e = 0; e < 8; e++) acc[i] = fmaf(qr[i][c * 8 + e], kf[e], acc[i]);
                }
            }
#pragma unroll
            for (int o = LPK / 2; o > 0; o >>= 1)
#pragma unroll
                for (int i = 0; i < RMAX; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
            if (kk < len && j < R) {
                float v = acc[0];
                int64_t lj = lim[0];
#pragma unroll
                for (int i = 1; i < RMAX; i++)
                    if (j == i) { v = acc[i]; lj = lim[i]; }
                ss[j * p.split_len + kk] = (k0 + kk <= lj) ? __fmul_rn(v, p.scale) : -INFINITY;
            }
        }
    }
    __syncthreads();

    if (warp < R) {
        const float *srow = ss + warp * p.split_len;
        float m = -INFINITY;
        for (int kk = lane; kk < len; kk += 32) m = fmaxf(m, srow[kk]);
        m = warp_max(m);
        double z = 0.0;
        if (m != -INFINITY)
            for (int kk = lane; kk < len; kk += 32) z += (double)expf(srow[kk] - m);
        z = warp_sum(z);
        if (lane == 0) {
            const int64_t pi = ((int64_t)h * p.n_splits + s) * RMAX + warp;
            p.part_m[pi] = m;
            p.part_z[pi] = z;
        }
        float *gs = p.S + ((int64_t)h * RMAX + warp) * p.S_stride + k0;
        for (int kk = lane; kk < len; kk += 32) gs[kk] = srow[kk];
    }
}

// ---------------------------------------------------------------------------
// pass 2
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads) pv_kernel(const PVParams p)
{
    constexpr int RMAX = Shape<D>::RMAX;
    constexpr int LPV = D / 8;           // lanes per V row (one 16-byte chunk each)
    constexpr int KPW = 32 / LPV;        // V rows per warp step
    constexpr int KPB = kWarps * KPW;
    constexpr int SLOTS = kWarps * KPW;
    extern __shared__ float smem[];
    __shared__ float rowM[RMAX], rowInv[RMAX];
    __shared__ int is_last;
    float *ps = smem;                    // [RMAX][split_len], later [SLOTS][RMAX][D]

    const int h = blockIdx.y, s = blockIdx.x;
    const int64_t k0 = (int64_t)s * p.split_len;
    const int64_t k1 = min(k0 + (int64_t)p.split_len, p.n_kv);
    const int len = (int)(k1 - k0);
    const int R = p.nrows;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // global max and sum of each query row from the per-split partials
    if (warp < R) {
        const float *pm = p.part_m + (int64_t)h * p.n_splits * RMAX + warp;
        const double *pz = p.part_z + (int64_t)h * p.n_splits * RMAX + warp;
        float M = -INFINITY;
        for (int jx = lane; jx < p.n_splits; jx += 32) M = fmaxf(M, pm[(int64_t)jx * RMAX]);
        M = warp_max(M);
        double Z = 0.0;
        for (int jx = lane; jx < p.n_splits; jx += 32) {
            const float mj = pm[(int64_t)jx * RMAX];
            if (mj != -INFINITY) Z += pz[(int64_t)jx * RMAX] * exp((double)mj - (double)M);
        }
        Z = warp_sum(Z);
        if (lane == 0) {
            rowM[warp] = M;
            rowInv[warp] = (float)(1.0 / Z);
        }
    }
    __syncthreads();

    // p = F16(expf(w - max) * (1/sum)), kept as the exact F32 value of that half
    for (int idx = tid; idx < R * len; idx += kThreads) {
        const int i = idx / len, kk = idx - i * len;
        const float w = p.S[((int64_t)h * RMAX + i) * p.S_stride + k0 + kk];
        const float e = expf(w - rowM[i]);
        ps[i * p.split_len + kk] = __half2float(__float2half_rn(__fmul_rn(e, rowInv[i])));
    }
    __syncthreads();

    const int g = lane / LPV, ci = lane % LPV;
    const bool lane_ok = g < KPW;
    float acc[RMAX][8];
#pragma unroll
    for (int i = 0; i < RMAX; i++)
#pragma unroll
        for (int e = 0; e < 8; e++) acc[i][e] = 0.0f;
    const __half *vbase = p.vc + (int64_t)h * D + ci * 8;
    for (int base = 0; base < len; base += KPB * kUnroll) {
        uint4 vv[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            const int kk = base + u * KPB + warp * KPW + g;
            if (lane_ok && kk < len) vv[u] = ld_stream(vbase + (k0 + kk) * (int64_t)p.row_elems);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            const int kk = base + u * KPB + warp * KPW + g;
            if (lane_ok && kk < len) {
                float vf[8];
                unpack8(vv[u], vf);
#pragma unroll
                for (int i = 0; i < RMAX; i++) {
                    if (i < R) {
                        const float pi = ps[i * p.split_len + kk];
#pragma unroll
                        for (int e = 0; e < 8; e++) acc[i][e] = fmaf(pi, vf[e], acc[i][e]);
                    }
                }
            }
        }
    }
    __syncthreads();

    float *red = smem;  // [SLOTS][RMAX][D]
    if (lane_ok) {
        const int slot = warp * KPW + g;
#pragma unroll
        for (int i = 0; i < RMAX; i++)
            if (i < R)
#pragma unroll
                for (int e = 0; e < 8; e++) red[(slot * RMAX + i) * D + ci * 8 + e] = acc[i][e];
    }
    __syncthreads();
    for (int idx = tid; idx < R * D; idx += kThreads) {
        const int i = idx / D, dd = idx - i * D;
        float sum = 0.0f;
#pragma unroll 4
        for (int sl = 0; sl < SLOTS; sl++) sum += red[(sl * RMAX + i) * D + dd];
        p.part_o[(((int64_t)h * p.n_splits + s) * RMAX + i) * D + dd] = sum;
    }

    // the last CTA of this KV head sums the split partials in split order
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = (atomicAdd(&p.counters[h], 1u) == (unsigned)(p.n_splits - 1));
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int idx = tid; idx < R * D; idx += kThreads) {
        const int i = idx / D, dd = idx - i * D;
        float sum = 0.0f;
        const float *src = p.part_o + ((int64_t)h * p.n_splits * RMAX + i) * D + dd;
        for (int jx = 0; jx < p.n_splits; jx++) sum += __ldcg(src + (int64_t)jx * RMAX * D);
        const int row = p.row0 + i;
        const int t = row / p.r, jj = row % p.r;
        p.out[(int64_t)t * p.out_stride + (int64_t)(p.out_head0 + h * p.r + jj) * D + dd] = sum;
    }
    if (tid == 0) p.counters[h] = 0u;
}

__global__ void unshard_kernel(float *out, int64_t out_stride, const float *src, int G, int n_new, int cols)
{
    const int64_t total = (int64_t)G * n_new * cols;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(idx % cols);
        const int64_t rest = idx / cols;
        const int t = (int)(rest % n_new);
        const int g = (int)(rest / n_new);
        out[(int64_t)t * out_stride + (int64_t)g * cols + c] = src[idx];
    }
}

template <int D>
cudaError_t prepare_d()
{
    cudaError_t e = cudaFuncSetAttribute(scores_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)scores_smem(D, Shape<D>::SPLIT_MAX));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(pv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)pv_smem(D, Shape<D>::SPLIT_MAX));
}

}  // namespace

int decode_rmax(int D)
{
    switch (D) {
    case 64: return Shape<64>::RMAX;
    case 96: return Shape<96>::RMAX;
    case 128: return Shape<128>::RMAX;
    default: return 0;
    }
}

int decode_split_max(int D)
{
    switch (D) {
    case 64: return Shape<64>::SPLIT_MAX;
    case 96: return Shape<96>::SPLIT_MAX;
    case 128: return Shape<128>::SPLIT_MAX;
    default: return 0;
    }
}

size_t scores_smem(int D, int split_len)
{
    const int rmax = decode_rmax(D);
    return sizeof(float) * (size_t)rmax * (size_t)(D + split_len);
}

size_t pv_smem(int D, int split_len)
{
    const int rmax = decode_rmax(D);
    const int slots = kWarps * (32 / (D / 8));
    const size_t a = (size_t)rmax * (size_t)split_len;
    const size_t b = (size_t)slots * (size_t)rmax * (size_t)D;
    return sizeof(float) * (a > b ? a : b);
}

cudaError_t decode_prepare(int D)
{
    switch (D) {
    case 64: return prepare_d<64>();
    case 96: return prepare_d<96>();
    case 128: return prepare_d<128>();
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_scores(int D, const ScoresParams &p, int hkv_loc, cudaStream_t st)
{
    const dim3 grid((unsigned)p.n_splits, (unsigned)hkv_loc);
    const size_t sm = scores_smem(D, p.split_len);
    switch (D) {
    case 64: scores_kernel<64><<<grid, kThreads, sm, st>>>(p); break;
    case 96: scores_kernel<96><<<grid, kThreads, sm, st>>>(p); break;
    case 128: scores_kernel<128><<<grid, kThreads, sm, st>>>(p); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_pv(int D, const PVParams &p, int hkv_loc, cudaStream_t st)
{
    const dim3 grid((unsigned)p.n_splits, (unsigned)hkv_loc);
    const size_t sm = pv_smem(D, p.split_len);
    switch (D) {
    case 64: pv_kernel<64><<<grid, kThreads, sm, st>>>(p); break;
    case 96: pv_kernel<96><<<grid, kThreads, sm, st>>>(p); break;
    case 128: pv_kernel<128><<<grid, kThreads, sm, st>>>(p); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_unshard(float *out, int64_t out_stride, const float *src, int G, int n_new, int cols,
                           cudaStream_t st)
{
    const int64_t total = (int64_t)G * n_new * cols;
    if (total <= 0) return cudaSuccess;
    int blocks = (int)((total + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    unshard_kernel<<<blocks, 256, 0, st>>>(out, out_stride, src, G, n_new, cols);
    return cudaGetLastError();
}

}  // namespace kvb
