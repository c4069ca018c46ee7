// kv_noalloc.cu -- decode attention for callers that must not allocate device memory.
//
// kv_attend() works inside a kv_ctx whose scratch (rotated Q, scores, split
// partials, completion counters) kv_alloc() obtained with cudaMalloc.  Some
// callers cannot do that: a host framework that plans and owns every device
// buffer up front (ggml's graph allocator, a serving engine that reserves all
// of HBM for its own pool) and runs this op as a callback in the middle of its
// compute, where a cudaMalloc would either fail for lack of free memory or
// stall the device with the allocator's implicit synchronisation.  For them,
// kv_attend_decode_noalloc() runs the same two decode kernels (scores, then
// F16-rounded P.V with the deterministic combine) on one token, with the
// caller's cache, query and output buffers, and with all scratch taken from a
// fixed array compiled into this library.
//
// The array is a file-scope `static __device__` object of kScratchBytes: every
// GPU that loads the library holds it until the process exits.  Host code
// cannot use the array's name as a device address (on the host it names a
// stand-in object), so the first call on each device, with that device
// current, asks the runtime for its device address once (cudaGetSymbolAddress)
// and keeps it.  Because of that one-time set-up, the first call on a device
// should be made before any stream capture begins.
//
// All calls share the one array and it keeps whatever the last call left
// there; this file clears the part that must start at zero (the per-head
// completion counters) at the start of every call.  Two calls whose work
// overlaps on the GPU (different streams, or different host threads) race on
// the array: serialise them.
#include <cstdio>
#include <mutex>

#include "kv_api.h"
#include "kv_internal.h"

namespace {

constexpr size_t kScratchBytes = (size_t)8 << 20;   // 8 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
struct DeviceSlot {
    unsigned char *base = nullptr;  // device address of g_noalloc_scratch
    int sm_count = 0;
};
DeviceSlot g_slots[kMaxDevices];
std::mutex g_slot_mu;

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// F32 rotated query -> F16 (round to nearest even), the conversion ggml's
// mul_mat applies to its F32 operand (kv_append writes the same bits).
__global__ void q_to_f16_kernel(const float *q, __half *dst, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = __float2half_rn(q[i]);
}

int setup_device(int dev, DeviceSlot **out, const char **why)
{
    std::lock_guard<std::mutex> lk(g_slot_mu);
    DeviceSlot &s = g_slots[dev];
    if (!s.base) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) { *why = cudaGetErrorString(e); return KV_E_CUDA; }
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) { *why = cudaGetErrorString(e); return KV_E_CUDA; }
        s.base = static_cast<unsigned char *>(p);
        s.sm_count = sms;
    }
    *out = &s;
    return KV_OK;
}

}  // namespace

extern "C" int kv_attend_decode_noalloc(const uint16_t *k_cache, const uint16_t *v_cache,
                                        int32_t n_head, int32_t n_head_kv, int32_t head_dim, int64_t n_kv,
                                        const float *q, float *out, void *stream)
{
    if (!k_cache || !v_cache || !q || !out)
        return kvb::set_last_error(KV_E_ARG, "kv_attend_decode_noalloc: NULL buffer");
    if (head_dim != 64 && head_dim != 96 && head_dim != 128)
        return kvb::set_last_error(KV_E_ARG, "kv_attend_decode_noalloc: head_dim must be 64, 96 or 128");
    if (n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv != 0 || n_kv < 1)
        return kvb::set_last_error(KV_E_ARG, "kv_attend_decode_noalloc: bad head counts or n_kv < 1");
    if ((((uintptr_t)k_cache) | ((uintptr_t)v_cache)) & 15u)
        return kvb::set_last_error(KV_E_ARG, "kv_attend_decode_noalloc: cache pointers must be 16-byte aligned");
    // shapes whose Q copy or one row of scores alone exceed the static array:
    // refused before the sizing arithmetic below, which they could overflow
    if ((uint64_t)n_head * (uint64_t)head_dim * sizeof(__half) > kScratchBytes ||
        (uint64_t)n_kv > kScratchBytes / sizeof(float))
        return kvb::set_last_error(KV_E_RANGE, "kv_attend_decode_noalloc: the shape needs more scratch than the "
                                               "static array holds (fewer keys or heads per call)");

    const int D = head_dim, hkv = n_head_kv, r = n_head / n_head_kv;
    const int rmax = kvb::decode_rmax(D), split_max = kvb::decode_split_max(D);

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: no usable current device");
    DeviceSlot *slot = nullptr;
    const char *why = "";
    int rc = setup_device(dev, &slot, &why);
    if (rc != KV_OK) return kvb::set_last_error(rc, why);

    // the split choice of kv_attend: ~2 CTAs per SM, splits of 64..split_max keys
    const int target = (2 * slot->sm_count + hkv - 1) / hkv > 1 ? (2 * slot->sm_count + hkv - 1) / hkv : 1;
    int64_t split_len = (n_kv + target - 1) / target;
    split_len = ((split_len + 63) / 64) * 64;
    if (split_len < 64) split_len = 64;
    if (split_len > split_max) split_len = split_max;
    const int n_splits = (int)((n_kv + split_len - 1) / split_len);

    // carve the static array: Q (F16), scores, partial max / sum / output, counters
    const int64_t S_stride = ((n_kv + 3) / 4) * 4;
    const size_t n_part = (size_t)hkv * (size_t)n_splits * (size_t)rmax;
    const size_t off_q = 0;
    const size_t off_s = off_q + align256((size_t)n_head * D * sizeof(__half));
    const size_t off_m = off_s + align256((size_t)hkv * rmax * (size_t)S_stride * sizeof(float));
    const size_t off_z = off_m + align256(n_part * sizeof(float));
    const size_t off_o = off_z + align256(n_part * sizeof(double));
    const size_t off_c = off_o + align256(n_part * (size_t)D * sizeof(float));
    const size_t need = off_c + align256((size_t)hkv * sizeof(unsigned));
    if (need > kScratchBytes) {
        char msg[200];
        snprintf(msg, sizeof(msg), "kv_attend_decode_noalloc: needs %zu bytes of scratch, the static array holds %zu "
                 "(fewer keys or KV heads per call)", need, kScratchBytes);
        return kvb::set_last_error(KV_E_RANGE, msg);
    }

    unsigned char *base = slot->base;
    __half *qbuf = reinterpret_cast<__half *>(base + off_q);
    float *S = reinterpret_cast<float *>(base + off_s);
    float *part_m = reinterpret_cast<float *>(base + off_m);
    double *part_z = reinterpret_cast<double *>(base + off_z);
    float *part_o = reinterpret_cast<float *>(base + off_o);
    unsigned *counters = reinterpret_cast<unsigned *>(base + off_c);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

    if (kvb::decode_prepare(D) != cudaSuccess) return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: kernel attribute set-up failed");
    if (cudaMemsetAsync(counters, 0, (size_t)hkv * sizeof(unsigned), st) != cudaSuccess)
        return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: clearing the counters failed");
    const int nq = n_head * D;
    q_to_f16_kernel<<<(nq + 255) / 256, 256, 0, st>>>(q, qbuf, nq);
    if (cudaGetLastError() != cudaSuccess) return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: launch failed");

    for (int row0 = 0; row0 < r; row0 += rmax) {
        const int nrows = r - row0 < rmax ? r - row0 : rmax;
        kvb::ScoresParams sp;
        sp.kc = reinterpret_cast<const __half *>(k_cache);
        sp.row_elems = hkv * D;
        sp.qbuf = qbuf;
        sp.hq_loc = n_head;
        sp.r = r;
        sp.row0 = row0;
        sp.nrows = nrows;
        sp.n_past = n_kv - 1;
        sp.n_kv = n_kv;
        sp.split_len = (int)split_len;
        sp.n_splits = n_splits;
        sp.scale = 1.0f / sqrtf((float)D);
        sp.S = S;
        sp.S_stride = S_stride;
        sp.part_m = part_m;
        sp.part_z = part_z;
        if (kvb::launch_scores(D, sp, hkv, st) != cudaSuccess)
            return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: scores launch failed");
        kvb::PVParams pp;
        pp.vc = reinterpret_cast<const __half *>(v_cache);
        pp.row_elems = sp.row_elems;
        pp.S = S;
        pp.S_stride = S_stride;
        pp.part_m = part_m;
        pp.part_z = part_z;
        pp.part_o = part_o;
        pp.counters = counters;
        pp.r = r;
        pp.row0 = row0;
        pp.nrows = nrows;
        pp.n_past = n_kv - 1;
        pp.n_kv = n_kv;
        pp.split_len = (int)split_len;
        pp.n_splits = n_splits;
        pp.out = out;
        pp.out_stride = (int64_t)n_head * D;
        pp.out_head0 = 0;
        if (kvb::launch_pv(D, pp, hkv, st) != cudaSuccess)
            return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: P.V launch failed");
    }
    kvb::set_last_error(KV_OK, "");
    return KV_OK;
}
