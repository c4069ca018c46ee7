// kv_internal.h -- shared declarations of the KV path library (host <-> kernels).
#pragma once

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
    int32_t n_new;
    int64_t n_past;
    int32_t hq_loc, hkv_loc;         // heads owned by this context
    int32_t hq0, hkv0;               // first owned global head
    int32_t n_rot, rope_mode, qk_norm;
    float eps;
    const float2 *rope;              // [n_ctx][n_rot/2] (cos, sin)
    __half *kc, *vc;                 // layer cache [n_ctx][hkv_loc][D]
    __half *qbuf;                    // [n_new][hq_loc][D]  rotated Q, F16
};

cudaError_t launch_append(int D, bool vec_loads, const AppendParams &p, cudaStream_t st);

// ---------------------------------------------------------------------------
// decode attention (CUDA cores, two passes): scores, then P.V + combine
// ---------------------------------------------------------------------------
// "Query rows" of a KV head: row i = t*r + j is token t, query head j of the
// GQA group.  One launch handles rows [row0, row0+nrows), nrows <= rmax(D).
struct ScoresParams {
    const __half *kc;                // layer K cache
    int32_t row_elems;               // hkv_loc * D
    const __half *qbuf;              // [n_new][hq_loc][D]
    int32_t hq_loc, r;
    int32_t row0, nrows;
    int64_t n_past, n_kv;
    int32_t split_len, n_splits;
    float scale;
    float *S;                        // [hkv_loc][RMAX][S_stride]
    int64_t S_stride;
    float *part_m;                   // [hkv_loc][n_splits][RMAX]
    double *part_z;
};

struct PVParams {
    const __half *vc;
    int32_t row_elems;
    const float *S;
    int64_t S_stride;
    const float *part_m;
    const double *part_z;
    float *part_o;                   // [hkv_loc][n_splits][RMAX][D]
    unsigned *counters;              // [hkv_loc], zero between calls
    int32_t r, row0, nrows;
    int64_t n_past, n_kv;
    int32_t split_len, n_splits;
    float *out;                      // row t at out + t*out_stride
    int64_t out_stride;
    int32_t out_head0;               // column head of local query head 0
};

int decode_rmax(int D);
size_t scores_smem(int D, int split_len);
size_t pv_smem(int D, int split_len);
int decode_split_max(int D);
cudaError_t decode_prepare(int D);   // raises dynamic smem limits once
cudaError_t launch_scores(int D, const ScoresParams &p, int hkv_loc, cudaStream_t st);
cudaError_t launch_pv(int D, const PVParams &p, int hkv_loc, cudaStream_t st);

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
