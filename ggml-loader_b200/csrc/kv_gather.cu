// kv_gather.cu -- layout of a sharded chunk's gathered outputs.
//
// A chunk (n_new > 1) on KV-head shards gathers every shard's [n_new][cols]
// block with one ncclAllGather into [G][n_new][cols]; the reference's output
// is token-major over all heads, [n_new][G*cols] (model.cpp:1444).  This
// kernel moves each element to that place.  (Single tokens need no move: the
// gathered [G][1][cols] already is the row.)
#include "kv_internal.h"

namespace kvb {
namespace {

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

}  // namespace

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
