// kv_append.cu -- fused QK-Norm + RoPE + F32->F16 (RNE) append of one layer.
//
// Replaces, for one layer, the reference's (src/model.cpp):
//   QKV projection bias (qwen2), ggml_add      model.cpp:1099-1102
//   per-head RMSNorm * gamma on Q and K        model.cpp:1382-1387 (rms_norm_mul 1071-1074)
//   ggml_rope_ext on Q and K                   model.cpp:1389-1404
//   ggml_cpy(K/V -> cache rows [n_past, +n_new)) model.cpp:1406-1414
// and the F16 conversion of Q that ggml_mul_mat(K, Q) performs on its F32 src1.
//
// Bit-exactness: every product and sum is a separately rounded IEEE float op
// (__fmul_rn / __fadd_rn / __fsub_rn: nothing is contracted into an FMA); the
// RMSNorm mean equals that of the sequential double sum of the float squares
// (exact_mean, with the sequential sum itself as the fallback); sqrt and the
// reciprocal are correctly rounded; the (cos, sin) table is built on the host
// with the same libm calls as the CPU path.  So the cache bytes equal the CPU
// path's.
//
// Work decomposition: a "row" is one (token, head) vector of D floats of Q, K
// or V.  D/8 threads own a row, each thread 8 consecutive elements, so a
// thread stores its 8 halves with one 16-byte st.global and a row group writes
// a contiguous D*2-byte cache segment.  32 rows per block.
#include <algorithm>

#include "kv_internal.h"
#include "kv_sm100.cuh"

namespace kvb {
namespace {

using sm100::pdl_launch_dependents;
using sm100::pdl_wait;

constexpr int kRowsPerBlock = 32;

__device__ __forceinline__ void load8(const float *src, bool vec, float x[8])
{
    if (vec) {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(src));
        const float4 b = __ldg(reinterpret_cast<const float4 *>(src) + 1);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) x[e] = __ldg(src + e);
    }
}

__device__ __forceinline__ void store8_f16(__half *dst, const float x[8])
{
    __half2 h[4];
#pragma unroll
    for (int e = 0; e < 4; e++) h[e] = __halves2half2(__float2half_rn(x[2 * e]), __float2half_rn(x[2 * e + 1]));
    *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(h);
}

// cache row of token t: its position, or the position modulo the ring's cells
// (a ring cache, dory.c:459-472)
__device__ __forceinline__ int64_t cache_row(const AppendParams &p, int t)
{
    const int64_t pos = p.n_past + t;
    return p.ring ? pos % p.ring : pos;
}

// row -> (token, kind 0 Q / 1 K / 2 V, head); false past the last row
__device__ __forceinline__ bool row_of(const AppendParams &p, int64_t row, int &t, int &kind, int &h)
{
    const int rows_per_tok = p.hq_loc + 2 * p.hkv_loc;
    t = 0;
    kind = 2;
    h = 0;
    if (row >= (int64_t)p.n_new * rows_per_tok) return false;
    const int r32 = (int)row;   // rows of one call < 2^31: 32-bit division
    t = r32 / rows_per_tok;
    const int slot = r32 - t * rows_per_tok;
    if (slot < p.hq_loc) { kind = 0; h = slot; }
    else if (slot < p.hq_loc + p.hkv_loc) { kind = 1; h = slot - p.hq_loc; }
    else { kind = 2; h = slot - p.hq_loc - p.hkv_loc; }
    return true;
}

// The mean of a row's squares exactly as ggml computes it, from the G threads'
// 8 squares each (G a power of two: the row's threads are one aligned group of
// lanes).  T = the squares summed in double as a tree (pairs within the
// thread, then the row's threads by shuffles): every term is >= 0, so T is
// within log2(8 G) * 2^-53 < 2^-49 of the exact sum.  ggml's sequential double
// sum is within (D - 1) * 2^-53 < 2^-45.9 of it.  When no float rounding
// boundary lies within 2^-44 T of T, both round to the same float and the
// mean is that float / D (D a power of two).  Returns false when the test
// cannot decide (the caller then sums sequentially).
template <int G, int D>
__device__ __forceinline__ bool exact_mean(const float (&sq)[8], float &mean)
{
    double T = (((double)sq[0] + (double)sq[1]) + ((double)sq[2] + (double)sq[3])) +
               (((double)sq[4] + (double)sq[5]) + ((double)sq[6] + (double)sq[7]));
#pragma unroll
    for (int o = 1; o < G; o <<= 1) T += __shfl_xor_sync(0xffffffffu, T, o);
    // (a warp holds whole rows: any row's inf/nan sends the warp's rows to the chain)
    if (__any_sync(0xffffffffu, !(T < INFINITY))) return false;
    if (T == 0.0) {   // every square is zero: so is the sequential sum
        mean = 0.0f;
        return true;
    }
    if (T < 0x1p-100) return false;   // keep (float)(T / D) far from the subnormal range
    const float f = __double2float_rn(T);   // positive and finite: its neighbours are +-1 ulp
    const double up = 0.5 * ((double)f + (double)__uint_as_float(__float_as_uint(f) + 1u));
    const double dn = 0.5 * ((double)f + (double)__uint_as_float(__float_as_uint(f) - 1u));
    const double tol = T * 0x1p-44;
    if (fabs(T - up) <= tol || fabs(T - dn) <= tol) return false;
    mean = f * (1.0f / (float)D);   // D is a power of two: exact
    return true;
}

template <int D>
struct AppendSmem {
    static constexpr int LDD = D + 1;   // doubles a row (odd: rows fall on different banks)
    static constexpr int LDX = D + 4;   // floats a row (16-byte aligned rows)
    static constexpr size_t sq = (size_t)kRowsPerBlock * LDD * 8;
    static constexpr size_t xs = (size_t)kRowsPerBlock * LDX * 4;
    static constexpr size_t bytes = sq > xs ? sq : xs;   // the squares, then the normed rows
};

template <int D, bool VEC>
__global__ void __launch_bounds__(kRowsPerBlock *(D / 8)) append_kernel(const AppendParams p)
{
    constexpr int G = D / 8;  // threads per row
    using S = AppendSmem<D>;
    __shared__ __align__(16) unsigned char sm[S::bytes];
    __shared__ float rscale[kRowsPerBlock];
    double *sq = reinterpret_cast<double *>(sm);
    float *xs = reinterpret_cast<float *>(sm);

    const int rloc = threadIdx.x / G;
    const int tig = threadIdx.x % G;
    const int64_t row0 = (int64_t)blockIdx.x * kRowsPerBlock;
    int t, kind, h;
    const bool active = row_of(p, row0 + rloc, t, kind, h);
    const bool rotates = active && kind < 2;
    // launched programmatically: the inputs and the cache rows only after the
    // previous kernel in the stream has completed
    pdl_wait();
    pdl_launch_dependents();

    float x[8];
#pragma unroll
    for (int e = 0; e < 8; e++) x[e] = 0.0f;
    if (active) {
        const float *src, *bias;
        if (kind == 0) {
            src = p.q + (int64_t)t * p.q_stride + (int64_t)(p.hq0 + h) * D;
            bias = p.q_bias ? p.q_bias + (int64_t)(p.hq0 + h) * D : nullptr;
        } else if (kind == 1) {
            src = p.k + (int64_t)t * p.k_stride + (int64_t)(p.hkv0 + h) * D;
            bias = p.k_bias ? p.k_bias + (int64_t)(p.hkv0 + h) * D : nullptr;
        } else {
            src = p.v + (int64_t)t * p.v_stride + (int64_t)(p.hkv0 + h) * D;
            bias = p.v_bias ? p.v_bias + (int64_t)(p.hkv0 + h) * D : nullptr;
        }
        load8(src + tig * 8, VEC, x);
        if (bias)   // ggml_add of the projection bias (model.cpp:1099-1102): one rounded add
#pragma unroll
            for (int e = 0; e < 8; e++) x[e] = __fadd_rn(x[e], __ldg(bias + tig * 8 + e));
    }

    // ---- QK-Norm: y = (x * (1/sqrt(mean(x*x) + eps))) * gamma --------------
    // ggml's mean: the float squares summed in double in element order, then
    // (float)(sum / D).  Fast path: the exact sum T from 64-bit integers (see
    // exact_mean); the sequential double sum s is within 2^-46 T of T,
    // so (float)s == (float)T whenever no float rounding midpoint lies within
    // 2^-44 T of T -- then the mean is (float)T / D.  Rows that fail the test
    // (about one in a million) or hold inf/nan or tiny sums run the sequential
    // double sum itself (warp 0, a row per lane).
    if (p.qk_norm) {
        float sqv[8];
#pragma unroll
        for (int e = 0; e < 8; e++) sqv[e] = __fmul_rn(x[e], x[e]);
        float fast_mean = 0.0f;
        const bool need_chain = (G & (G - 1)) != 0 || !exact_mean<G, D>(sqv, fast_mean);
        if (__syncthreads_or(rotates && need_chain)) {
            if (need_chain) {
#pragma unroll
                for (int e = 0; e < 8; e++) sq[rloc * S::LDD + tig * 8 + e] = (double)sqv[e];
            }
            __syncthreads();
            if (threadIdx.x < kRowsPerBlock) {
                int tr, kr, hr;
                if (row_of(p, row0 + threadIdx.x, tr, kr, hr) && kr < 2) {
                    const double *r = sq + threadIdx.x * S::LDD;
                    double sum = 0.0;
#pragma unroll 16
                    for (int i = 0; i < D; i++) sum = __dadd_rn(sum, r[i]);
                    rscale[threadIdx.x] = __double2float_rn(__ddiv_rn(sum, (double)D));
                }
            }
            __syncthreads();
            if (need_chain) fast_mean = rscale[rloc];
        }
        if (rotates) {
            const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(fast_mean, p.eps)));
            const float *w = (kind == 0 ? p.q_norm_w : p.k_norm_w) + tig * 8;
#pragma unroll
            for (int e = 0; e < 8; e++) x[e] = __fmul_rn(__fmul_rn(x[e], sc), __ldg(w + e));
        }
    }

    // ---- RoPE on the first n_rot dims (NEOX halves / NORMAL pairs) --------
    if (p.n_rot > 0) {
        const int half = p.n_rot >> 1;
        const int i0 = tig * 8;
        if (p.rope_mode == 2) {
            // NEOX: element i pairs with i +- half, held by another thread (the
            // squares' last reader, warp 0, has passed the norm's barrier)
            float *xr = xs + rloc * S::LDX;
            *reinterpret_cast<float4 *>(xr + i0) = make_float4(x[0], x[1], x[2], x[3]);
            *reinterpret_cast<float4 *>(xr + i0 + 4) = make_float4(x[4], x[5], x[6], x[7]);
            __syncthreads();
            if (rotates && i0 < p.n_rot) {
                const float2 *cs = p.rope + (p.n_past + t) * (int64_t)half;
                if ((half & 7) == 0 && i0 + 8 <= p.n_rot) {
                    // the thread's 8 elements sit in one half: vector loads
                    const bool lo = i0 < half;
                    const int j0 = lo ? i0 : i0 - half;          // table index of element 0
                    const int pj = lo ? i0 + half : i0 - half;   // partner of element 0
                    float y[8];
                    *reinterpret_cast<float4 *>(y) = *reinterpret_cast<const float4 *>(xr + pj);
                    *reinterpret_cast<float4 *>(y + 4) = *reinterpret_cast<const float4 *>(xr + pj + 4);
                    float2 c[8];
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        *reinterpret_cast<float4 *>(c + 2 * q) = __ldg(reinterpret_cast<const float4 *>(cs + j0) + q);
#pragma unroll
                    for (int e = 0; e < 8; e++)
                        x[e] = lo ? __fsub_rn(__fmul_rn(x[e], c[e].x), __fmul_rn(y[e], c[e].y))
                                  : __fadd_rn(__fmul_rn(y[e], c[e].y), __fmul_rn(x[e], c[e].x));
                } else {
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        const int i = i0 + e;
                        if (i >= p.n_rot) continue;
                        if (i < half) {
                            const float2 c = __ldg(cs + i);
                            x[e] = __fsub_rn(__fmul_rn(xr[i], c.x), __fmul_rn(xr[i + half], c.y));
                        } else {
                            const float2 c = __ldg(cs + (i - half));
                            x[e] = __fadd_rn(__fmul_rn(xr[i - half], c.y), __fmul_rn(xr[i], c.x));
                        }
                    }
                }
            }
        } else if (rotates) {
            // NORMAL: pairs (2k, 2k+1) inside the thread's 8 elements
            const float2 *cs = p.rope + (p.n_past + t) * (int64_t)half;
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                const int i = i0 + e;
                if (i >= p.n_rot) continue;
                const float2 c = __ldg(cs + (i >> 1));
                const float a = x[e], b = x[e + 1];
                x[e] = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y));
                x[e + 1] = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
            }
        }
    }

    if (!active) return;
    __half *dst;
    if (kind == 0) dst = p.qbuf + ((int64_t)t * p.hq_loc + h) * D;
    else if (kind == 1) dst = p.kc + (cache_row(p, t) * p.hkv_loc + h) * D;
    else dst = p.vc + (cache_row(p, t) * p.hkv_loc + h) * D;
    store8_f16(dst + tig * 8, x);
}

// The common shapes (head_dim 64 or 128, RoPE over the whole head or none): a
// row's D/8 threads are one aligned group of lanes, so the NEOX
// partners, the norm's sum and its rare sequential fallback move by shuffles
// -- no shared memory, no block barrier.  Same arithmetic as append_kernel.
// ggml's mean of a row's squares (A1) for the G threads holding it, 8 values
// each: exact_mean, else (one row in about a million) the sequential double sum
// with lane 0 of the row's group gathering the squares in element order.  Every
// lane of the warp calls it.
template <int G, int D>
__device__ __forceinline__ float row_mean(const float (&x)[8], bool rotates, int lane)
{
    float sqv[8];
#pragma unroll
    for (int e = 0; e < 8; e++) sqv[e] = __fmul_rn(x[e], x[e]);
    float mean = 0.0f;
    const bool need = !exact_mean<G, D>(sqv, mean);
    if (__any_sync(0xffffffffu, rotates && need)) {
        const int base = (lane / G) * G;
        double sum = 0.0;
#pragma unroll 1
        for (int s2 = 0; s2 < G; s2++)
#pragma unroll
            for (int e = 0; e < 8; e++) sum = __dadd_rn(sum, (double)__shfl_sync(0xffffffffu, sqv[e], base + s2));
        const float cm = __double2float_rn(__ddiv_rn(sum, (double)D));
        if (need) mean = cm;
    }
    return mean;
}

template <int D, bool VEC>
__global__ void __launch_bounds__(256) append_kernel_warp(const AppendParams p)
{
    constexpr int G = D / 8;               // threads per row (16 or 8)
    const int lane = threadIdx.x & 31;
    const int tig = lane % G;
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / G;
    int t, kind, h;
    const bool active = row_of(p, row, t, kind, h);
    const bool rotates = active && kind < 2;
    const int half = p.n_rot >> 1, i0 = tig * 8;
    const bool neox = p.rope_mode == 2;

    // RoPE entries first: they do not depend on the row's values
    float2 c[8];
    if (rotates && p.n_rot > 0) {
        const float2 *cs = p.rope + (p.n_past + t) * (int64_t)half;
        if (neox) {
            const int j0 = i0 < half ? i0 : i0 - half;
#pragma unroll
            for (int q = 0; q < 4; q++) *reinterpret_cast<float4 *>(c + 2 * q) = __ldg(reinterpret_cast<const float4 *>(cs + j0) + q);
        } else {
#pragma unroll
            for (int q = 0; q < 2; q++) *reinterpret_cast<float4 *>(c + 2 * q) = __ldg(reinterpret_cast<const float4 *>(cs + i0 / 2) + q);
        }
    }
    // launched programmatically: the RoPE entries above come from a table
    // written once at kv_alloc; the inputs and the cache rows only after the
    // previous kernel in the stream has completed
    pdl_wait();
    pdl_launch_dependents();
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; e++) x[e] = 0.0f;
    if (active) {
        const float *src, *bias;
        if (kind == 0) {
            src = p.q + (int64_t)t * p.q_stride + (int64_t)(p.hq0 + h) * D;
            bias = p.q_bias ? p.q_bias + (int64_t)(p.hq0 + h) * D : nullptr;
        } else if (kind == 1) {
            src = p.k + (int64_t)t * p.k_stride + (int64_t)(p.hkv0 + h) * D;
            bias = p.k_bias ? p.k_bias + (int64_t)(p.hkv0 + h) * D : nullptr;
        } else {
            src = p.v + (int64_t)t * p.v_stride + (int64_t)(p.hkv0 + h) * D;
            bias = p.v_bias ? p.v_bias + (int64_t)(p.hkv0 + h) * D : nullptr;
        }
        load8(src + i0, VEC, x);
        if (bias)   // ggml_add of the projection bias (model.cpp:1099-1102): one rounded add
#pragma unroll
            for (int e = 0; e < 8; e++) x[e] = __fadd_rn(x[e], __ldg(bias + i0 + e));
    }

    // ---- QK-Norm (see append_kernel); warps of V rows only skip it --------------
    if (p.qk_norm == 1 && __any_sync(0xffffffffu, rotates)) {
        const float mean = row_mean<G, D>(x, rotates, lane);
        if (rotates) {
            const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
            float wv[8];
            load8((kind == 0 ? p.q_norm_w : p.k_norm_w) + i0, VEC, wv);   // (VEC: gammas 16-byte aligned too)
#pragma unroll
            for (int e = 0; e < 8; e++) x[e] = __fmul_rn(__fmul_rn(x[e], sc), wv[e]);
        }
    }

    // ---- RoPE ---------------------------------------------------------------
    if (p.n_rot > 0) {
        if (neox) {
            // partner of element i is i +- D/2: the thread D/16 lanes away
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; e++) y[e] = __shfl_xor_sync(0xffffffffu, x[e], G / 2);
            if (rotates) {
                const bool lo = i0 < half;
#pragma unroll
                for (int e = 0; e < 8; e++)
                    x[e] = lo ? __fsub_rn(__fmul_rn(x[e], c[e].x), __fmul_rn(y[e], c[e].y))
                              : __fadd_rn(__fmul_rn(y[e], c[e].y), __fmul_rn(x[e], c[e].x));
            }
        } else if (rotates) {
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                const float2 cc = c[e / 2];
                const float a = x[e], b = x[e + 1];
                x[e] = __fsub_rn(__fmul_rn(a, cc.x), __fmul_rn(b, cc.y));
                x[e + 1] = __fadd_rn(__fmul_rn(a, cc.y), __fmul_rn(b, cc.x));
            }
        }
    }

    // ---- nGPT (dory, qk_norm 2; dory.c:577-580, 646-649): after RoPE,
    // rms_norm(x, 1e-6/D) (ggml's arithmetic, as QK-Norm) times 1/sqrt(D), then
    // Q times its per-head, per-channel scale (q_norm_w [n_head][D]); K unscaled
    if (p.qk_norm == 2 && __any_sync(0xffffffffu, rotates)) {
        const float mean = row_mean<G, D>(x, rotates, lane);
        if (rotates) {
            const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
#pragma unroll
            for (int e = 0; e < 8; e++) x[e] = __fmul_rn(__fmul_rn(x[e], sc), p.post);
            if (kind == 0) {
                float wv[8];
                load8(p.q_norm_w + (int64_t)(p.hq0 + h) * D + i0, VEC, wv);
#pragma unroll
                for (int e = 0; e < 8; e++) x[e] = __fmul_rn(x[e], wv[e]);
            }
        }
    }

    if (!active) return;
    __half *dst;
    if (kind == 0) dst = p.qbuf + ((int64_t)t * p.hq_loc + h) * D;
    else if (kind == 1) dst = p.kc + (cache_row(p, t) * p.hkv_loc + h) * D;
    else dst = p.vc + (cache_row(p, t) * p.hkv_loc + h) * D;
    store8_f16(dst + i0, x);
}

// a launch that may start while the previous kernel in the stream finishes
// (programmatic dependent launch; the kernels wait for it before they touch
// memory that kernel may write)
template <class K>
cudaError_t launch_early(K kernel, dim3 grid, dim3 block, cudaStream_t st, const AppendParams &p)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int D>
cudaError_t launch_append_d(bool vec, const AppendParams &p, cudaStream_t st)
{
    const int64_t rows = (int64_t)p.n_new * (p.hq_loc + 2 * p.hkv_loc);
    const int64_t blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
    if (blocks <= 0) return cudaSuccess;
    if constexpr (D == 64 || D == 128 || D == 256) {
        // shuffle-only kernel: RoPE over the whole head (or none); partial
        // rotary takes append_kernel (head_dim <= 128), as does a partial
        // rotation with the nGPT norm nowhere (dory rotates whole heads)
        if (p.n_rot == 0 || p.n_rot == D) {
            const int64_t wblocks = (rows * (D / 8) + 255) / 256;
            return vec ? launch_early(append_kernel_warp<D, true>, dim3((unsigned)wblocks), dim3(256), st, p)
                       : launch_early(append_kernel_warp<D, false>, dim3((unsigned)wblocks), dim3(256), st, p);
        }
    }
    if constexpr (D == 256) {
        return cudaErrorInvalidValue;   // partial rotation at head_dim 256: not built
    } else {
    if (p.qk_norm == 2) return cudaErrorInvalidValue;   // the nGPT norm needs whole-head rotation
    const dim3 grid((unsigned)blocks), block(kRowsPerBlock * (D / 8));
    return vec ? launch_early(append_kernel<D, true>, grid, block, st, p)
               : launch_early(append_kernel<D, false>, grid, block, st, p);
    }
}

// dory_fill_attn_mask (dory.c:553-575) over the n_used cells a ring attention
// reads: with head = pos0 + n_tokens - 1, cell c was last written at
// head - ((head - c) mod n_cells) = base + c (- n_cells when c > head mod
// n_cells), base = head - head mod n_cells; visible (0) to the query at pos0 + q
// when that write is a real position no later than it, else -inf.  F16 rows of
// `stride` elements.
__global__ void __launch_bounds__(256) ring_mask_kernel(__half *dst, int64_t stride, int64_t n_cells, int64_t pos0,
                                                        int n_tokens, int64_t n_used)
{
    const int q = blockIdx.y;
    const int64_t head = pos0 + n_tokens - 1, hm = head % n_cells, base = head - hm;
    const __half vis = __float2half_rn(0.0f), hid = __float2half_rn(-INFINITY);
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < n_used; c += (int64_t)gridDim.x * blockDim.x) {
        const int64_t lw = base + c - (c > hm ? n_cells : 0);
        dst[(int64_t)q * stride + c] = (lw >= 0 && lw <= pos0 + q) ? vis : hid;
    }
}

}  // namespace

cudaError_t launch_ring_mask(__half *dst, int64_t stride, int64_t n_cells, int64_t pos0, int n_tokens, int64_t n_used,
                             cudaStream_t st)
{
    if (n_tokens <= 0 || n_used <= 0) return cudaSuccess;
    const unsigned bx = (unsigned)std::min<int64_t>((n_used + 255) / 256, 64);
    ring_mask_kernel<<<dim3(bx, (unsigned)n_tokens), 256, 0, st>>>(dst, stride, n_cells, pos0, n_tokens, n_used);
    return cudaGetLastError();
}

cudaError_t launch_append(int D, bool vec_loads, const AppendParams &p, cudaStream_t st)
{
    switch (D) {
    case 64: return launch_append_d<64>(vec_loads, p, st);
    case 96: return launch_append_d<96>(vec_loads, p, st);
    case 128: return launch_append_d<128>(vec_loads, p, st);
    case 256: return launch_append_d<256>(vec_loads, p, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace kvb
