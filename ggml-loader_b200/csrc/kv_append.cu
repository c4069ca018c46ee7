// kv_append.cu -- fused QK-Norm + RoPE + F32->F16 (RNE) append of one layer.
//
// Replaces, for one layer, the reference's (src/model.cpp):
//   per-head RMSNorm * gamma on Q and K        model.cpp:1382-1387 (rms_norm_mul 1071-1074)
//   ggml_rope_ext on Q and K                   model.cpp:1389-1404
//   ggml_cpy(K/V -> cache rows [n_past, +n_new)) model.cpp:1406-1414
// and the F16 conversion of Q that ggml_mul_mat(K, Q) performs on its F32 src1.
//
// Bit-exactness: every product and sum is a separately rounded IEEE float op
// (__fmul_rn / __fadd_rn / __fsub_rn: nothing is contracted into an FMA); the
// RMSNorm sum of squares is sequential in double; sqrt and the reciprocal are
// correctly rounded; the (cos, sin) table is built on the host with the same
// libm calls as the CPU path.  So the cache bytes equal the CPU path's.
//
// Work decomposition: a "row" is one (token, head) vector of D floats of Q, K
// or V.  D/8 threads own a row, each thread 8 consecutive elements, so a
// thread stores its 8 halves with one 16-byte st.global and a row group writes
// a contiguous D*2-byte cache segment.  8 rows per block.
#include "kv_internal.h"

namespace kvb {
namespace {

constexpr int kRowsPerBlock = 8;

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

template <int D, bool VEC>
__global__ void __launch_bounds__(kRowsPerBlock *(D / 8)) append_kernel(const AppendParams p)
{
    constexpr int G = D / 8;  // threads per row
    __shared__ float xs[kRowsPerBlock][D];
    __shared__ float rscale[kRowsPerBlock];

    const int rloc = threadIdx.x / G;
    const int tig = threadIdx.x % G;
    const int rows_per_tok = p.hq_loc + 2 * p.hkv_loc;
    const int64_t row = (int64_t)blockIdx.x * kRowsPerBlock + rloc;
    const bool active = row < (int64_t)p.n_new * rows_per_tok;

    int t = 0, kind = 2, h = 0;
    if (active) {
        t = (int)(row / rows_per_tok);
        const int slot = (int)(row % rows_per_tok);
        if (slot < p.hq_loc) { kind = 0; h = slot; }
        else if (slot < p.hq_loc + p.hkv_loc) { kind = 1; h = slot - p.hq_loc; }
        else { kind = 2; h = slot - p.hq_loc - p.hkv_loc; }
    }
    const bool rotates = active && kind < 2;

    float x[8];
#pragma unroll
    for (int e = 0; e < 8; e++) x[e] = 0.0f;
    if (active) {
        const float *src;
        if (kind == 0) src = p.q + (int64_t)t * p.q_stride + (int64_t)(p.hq0 + h) * D;
        else if (kind == 1) src = p.k + (int64_t)t * p.k_stride + (int64_t)(p.hkv0 + h) * D;
        else src = p.v + (int64_t)t * p.v_stride + (int64_t)(p.hkv0 + h) * D;
        load8(src + tig * 8, VEC, x);
    }

    // ---- QK-Norm: y = (x * (1/sqrt(mean(x*x) + eps))) * gamma --------------
    if (p.qk_norm) {
#pragma unroll
        for (int e = 0; e < 8; e++) xs[rloc][tig * 8 + e] = __fmul_rn(x[e], x[e]);
        __syncthreads();
        if (rotates && tig == 0) {
            double sum = 0.0;
            for (int i = 0; i < D; i++) sum = __dadd_rn(sum, (double)xs[rloc][i]);
            const float mean = __double2float_rn(__ddiv_rn(sum, (double)D));
            rscale[rloc] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
        }
        __syncthreads();
        if (rotates) {
            const float sc = rscale[rloc];
            const float *w = (kind == 0 ? p.q_norm_w : p.k_norm_w) + tig * 8;
#pragma unroll
            for (int e = 0; e < 8; e++) x[e] = __fmul_rn(__fmul_rn(x[e], sc), __ldg(w + e));
        }
    }

    // ---- RoPE on the first n_rot dims (NEOX halves / NORMAL pairs) --------
    if (p.n_rot > 0) {
        __syncthreads();
#pragma unroll
        for (int e = 0; e < 8; e++) xs[rloc][tig * 8 + e] = x[e];
        __syncthreads();
        if (rotates) {
            const int half = p.n_rot >> 1;
            const float2 *cs = p.rope + (p.n_past + t) * (int64_t)half;
            const float *xr = xs[rloc];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const int i = tig * 8 + e;
                if (i >= p.n_rot) continue;
                if (p.rope_mode == 2) {
                    if (i < half) {
                        const float2 c = __ldg(cs + i);
                        x[e] = __fsub_rn(__fmul_rn(xr[i], c.x), __fmul_rn(xr[i + half], c.y));
                    } else {
                        const float2 c = __ldg(cs + (i - half));
                        x[e] = __fadd_rn(__fmul_rn(xr[i - half], c.y), __fmul_rn(xr[i], c.x));
                    }
                } else {
                    const float2 c = __ldg(cs + (i >> 1));
                    if ((i & 1) == 0) x[e] = __fsub_rn(__fmul_rn(xr[i], c.x), __fmul_rn(xr[i + 1], c.y));
                    else x[e] = __fadd_rn(__fmul_rn(xr[i - 1], c.y), __fmul_rn(xr[i], c.x));
                }
            }
        }
    }

    if (!active) return;
    __half *dst;
    if (kind == 0) dst = p.qbuf + ((int64_t)t * p.hq_loc + h) * D;
    else if (kind == 1) dst = p.kc + ((p.n_past + t) * (int64_t)p.hkv_loc + h) * D;
    else dst = p.vc + ((p.n_past + t) * (int64_t)p.hkv_loc + h) * D;
    store8_f16(dst + tig * 8, x);
}

template <int D>
cudaError_t launch_append_d(bool vec, const AppendParams &p, cudaStream_t st)
{
    const int64_t rows = (int64_t)p.n_new * (p.hq_loc + 2 * p.hkv_loc);
    const int64_t blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
    if (blocks <= 0) return cudaSuccess;
    const dim3 grid((unsigned)blocks), block(kRowsPerBlock * (D / 8));
    if (vec) append_kernel<D, true><<<grid, block, 0, st>>>(p);
    else append_kernel<D, false><<<grid, block, 0, st>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_append(int D, bool vec_loads, const AppendParams &p, cudaStream_t st)
{
    switch (D) {
    case 64: return launch_append_d<64>(vec_loads, p, st);
    case 96: return launch_append_d<96>(vec_loads, p, st);
    case 128: return launch_append_d<128>(vec_loads, p, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace kvb
