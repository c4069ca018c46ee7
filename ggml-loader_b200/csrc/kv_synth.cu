// kv_synth.cu -- seeded synthetic cache rows and inputs for the benchmark and tests.
//
// Generator: splitmix64's output function applied to a per-(seed, stream)
// starting state advanced by the golden-ratio increment; a standard-normal-like
// value is the Irwin-Hall sum of twelve 16-bit uniforms (mean 0, variance 1,
// support [-6, 6]) shifted and scaled by powers of two, which is exact in F32,
// so every device and the host produce identical bits.
#include "kv_internal.h"

namespace kvb {
namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t x)
{
    x ^= x >> 30;
    x *= 0xBF58476D1CE4E5B9ull;
    x ^= x >> 27;
    x *= 0x94D049BB133111EBull;
    x ^= x >> 31;
    return x;
}

__device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint64_t stream)
{
    return mix64(seed ^ mix64(stream + 0x6B76B200ull));
}

__device__ __forceinline__ uint32_t sum4x16(uint64_t w)
{
    return (uint32_t)(w & 0xffffu) + (uint32_t)((w >> 16) & 0xffffu) + (uint32_t)((w >> 32) & 0xffffu) +
           (uint32_t)(w >> 48);
}

__device__ __forceinline__ float normal_at(uint64_t key, uint64_t idx)
{
    const uint64_t c = idx * 3u;
    const uint32_t s = sum4x16(mix64(key + c * 0x9E3779B97F4A7C15ull)) +
                       sum4x16(mix64(key + (c + 1u) * 0x9E3779B97F4A7C15ull)) +
                       sum4x16(mix64(key + (c + 2u) * 0x9E3779B97F4A7C15ull));
    return __fsub_rn(__fmul_rn((float)(s + 6u), 1.0f / 65536.0f), 6.0f);
}

// One thread writes 8 consecutive dims (16 bytes) of one (layer, K|V, row, head).
__global__ void fill_kernel(const FillParams p)
{
    const int chunks = p.D / 8;
    const int64_t per_row = (int64_t)p.hkv_loc * chunks;
    const int64_t total = (int64_t)p.n_layer * 2 * p.nrows * per_row;
    const int64_t layer_elems = p.n_ctx * (int64_t)p.hkv_loc * p.D;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(idx % chunks);
        int64_t rest = idx / chunks;
        const int hl = (int)(rest % p.hkv_loc);
        rest /= p.hkv_loc;
        const int64_t r = rest % p.nrows;
        rest /= p.nrows;
        const int which = (int)(rest % 2);
        const int layer = (int)(rest / 2);
        const int64_t row = p.row0 + r;
        const uint64_t key = stream_key(p.seed, p.stream_base + 2u * (uint64_t)layer + (uint64_t)which);
        const uint64_t i0 = (uint64_t)row * (uint64_t)p.hkv_total * (uint64_t)p.D +
                            (uint64_t)(p.hkv0 + hl) * (uint64_t)p.D + (uint64_t)c * 8u;
        __half2 hv[4];
#pragma unroll
        for (int e = 0; e < 4; e++)
            hv[e] = __halves2half2(__float2half_rn(normal_at(key, i0 + 2 * e)),
                                   __float2half_rn(normal_at(key, i0 + 2 * e + 1)));
        __half *dst = p.cache + ((int64_t)layer * 2 + which) * layer_elems +
                      (row * (int64_t)p.hkv_loc + hl) * p.D + c * 8;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(hv);
    }
}

__global__ void gen_normal_kernel(float *dst, uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n)
{
    const uint64_t key = stream_key(seed, stream);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = normal_at(key, idx0 + (uint64_t)i);
}

}  // namespace

cudaError_t launch_fill(const FillParams &p, cudaStream_t st)
{
    const int64_t total = (int64_t)p.n_layer * 2 * p.nrows * p.hkv_loc * (p.D / 8);
    if (total <= 0) return cudaSuccess;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    fill_kernel<<<(unsigned)blocks, 256, 0, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_gen_normal(float *dst, uint64_t seed, uint64_t stream, uint64_t idx0, int64_t n, cudaStream_t st)
{
    if (n <= 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    gen_normal_kernel<<<(unsigned)blocks, 256, 0, st>>>(dst, seed, stream, idx0, n);
    return cudaGetLastError();
}

}  // namespace kvb
