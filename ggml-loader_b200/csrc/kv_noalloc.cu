// kv_noalloc.cu -- decode attention for callers that must not allocate device memory.
//
// kv_attend() works inside a kv_ctx whose scratch (scores, statistics slots,
// output accumulators, tickets) kv_alloc() obtained with cudaMalloc.  Some
// callers cannot do that: a host framework that plans and owns every device
// buffer up front (ggml's graph allocator, a serving engine that reserves all
// of HBM for its own pool) and runs this op as a callback in the middle of its
// compute, where a cudaMalloc would either fail for lack of free memory or
// stall the device with the allocator's implicit synchronisation.  For them,
// kv_attend_decode_noalloc() runs kv_attend's decode attention kernel on one
// token -- the default (not the flash-attn) branch, plain grid -- over the
// caller's cache, query and output buffers, with all scratch taken from a
// fixed array compiled into this library.
//
// The array is a file-scope `static __device__` object of kScratchBytes: every
// GPU that loads the library holds it until the process exits.  Host code
// cannot use the array's name as a device address (on the host it names a
// stand-in object), so the first call on each device, with that device
// current, asks the runtime for its device address once (cudaGetSymbolAddress)
// and keeps it, together with the kernel's shared-memory set-up.  Because of
// that one-time set-up, the first call on a device should be made before any
// stream capture begins; and because it is kept for the life of the process,
// a cudaDeviceReset() invalidates it (restart the process after one).
//
// All calls share the one array and it keeps whatever the last call left
// there; each call clears the part that must start at zero (the per-head
// output accumulators and tickets) before its kernels run.  Two calls whose
// work overlaps on the GPU (different streams, or different host threads)
// race on the array: serialise them.
//
// The kernel's CTAs wait on one another; this entry launches it cooperatively,
// so the driver starts it only with the whole grid resident, even when the
// caller's other work shares the GPU.
#include <cstdio>
#include <mutex>

#include "kv_api.h"
#include "kv_internal.h"

namespace {

constexpr size_t kScratchBytes = (size_t)16 << 20;   // 16 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
struct DeviceSlot {
    unsigned char *base = nullptr;  // device address of g_noalloc_scratch
    int sm_count = 0;
    unsigned prepared = 0;          // head dims whose kernel attributes are set (bit per 64/96/128)
    uint32_t epoch = 0;             // tag of the last launch's statistics slots
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

unsigned dim_bit(int D) { return D == 64 ? 1u : D == 96 ? 2u : 4u; }

// Per-device set-up, once: the array's device address and the kernel's
// shared-memory limit for this head_dim.  Returns the slot with the epochs of
// `launches` launches reserved (first one in *epoch0), under the lock.
int setup_device(int dev, int D, int launches, DeviceSlot *out, uint32_t *epoch0, bool *wrapped, const char **why)
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
    if (!(s.prepared & dim_bit(D))) {
        cudaError_t e = kvb::attn_prepare(D);
        if (e != cudaSuccess) { *why = cudaGetErrorString(e); return KV_E_CUDA; }
        s.prepared |= dim_bit(D);
    }
    // epochs tag the statistics slots; the array starts zeroed, so 0 is never
    // a launch's tag, and a wrap clears the slots (by the caller, on its stream)
    *wrapped = false;
    if (s.epoch > 0xffffffffu - (uint32_t)launches) {
        s.epoch = 0;
        *wrapped = true;
    }
    *epoch0 = s.epoch + 1;
    s.epoch += (uint32_t)launches;
    *out = s;
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
    // shapes whose query copy or scores alone exceed the static array:
    // refused before the sizing arithmetic below, which they could overflow
    const uint64_t tile_bytes = (uint64_t)kvb::attn_tile_scores() * sizeof(float);
    if ((uint64_t)n_head * (uint64_t)head_dim * sizeof(__half) > kScratchBytes ||
        (uint64_t)n_kv > (uint64_t)(kScratchBytes / tile_bytes) * kvb::attn_tile_keys() / (uint64_t)n_head_kv)
        return kvb::set_last_error(KV_E_RANGE, "kv_attend_decode_noalloc: the shape needs more scratch than the "
                                               "static array holds (fewer keys or KV heads per call)");
    if (n_head_kv > kvb::kMaxLocalHeads)
        return kvb::set_last_error(KV_E_RANGE, "kv_attend_decode_noalloc: more KV heads than a launch covers (64)");

    const int D = head_dim, hkv = n_head_kv, r = n_head / n_head_kv;
    const int rows_per = kvb::attn_rows();
    const int launches = (r + rows_per - 1) / rows_per;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: no usable current device");
    DeviceSlot slot;
    uint32_t epoch0 = 0;
    bool wrapped = false;
    const char *why = "";
    int rc = setup_device(dev, D, launches, &slot, &epoch0, &wrapped, &why);
    if (rc != KV_OK) return kvb::set_last_error(rc, why);

    // the plain split of kv_attend (one CTA per SM at most, >= 256 keys a CTA)
    kvb::AttnParams ap{};
    ap.n_cta = std::min(kvb::attn_plain_ctas(slot.sm_count, hkv, n_kv), kvb::attn_max_ctas());
    kvb::attn_split(ap, hkv, n_kv);

    // carve the static array: query (F16), scores, statistics slots, then the
    // zeroed block: output accumulators, tickets + non-finite flags, error word
    const size_t off_q = 0;
    const size_t off_s = off_q + align256((size_t)n_head * D * sizeof(__half));
    const size_t off_st = off_s + align256((size_t)ap.n_cta * ap.S_tiles * tile_bytes);
    const size_t off_acc = off_st + align256((size_t)ap.n_cta * 2u * 8u * 2u * sizeof(unsigned long long));
    const size_t off_ctl = off_acc + (size_t)hkv * 8u * (size_t)D * sizeof(long long);
    const size_t zero_bytes = (off_ctl - off_acc) + (2u * (size_t)hkv + 2u) * sizeof(unsigned);
    const size_t need = off_acc + zero_bytes;
    if (need > kScratchBytes) {
        char msg[200];
        snprintf(msg, sizeof(msg), "kv_attend_decode_noalloc: needs %zu bytes of scratch, the static array holds %zu "
                 "(fewer keys or KV heads per call)", need, kScratchBytes);
        return kvb::set_last_error(KV_E_RANGE, msg);
    }

    CUtensorMap km, vm;
    rc = kvb::encode_cache_map(&km, k_cache, n_kv, hkv, D);
    if (rc == KV_OK) rc = kvb::encode_cache_map(&vm, v_cache, n_kv, hkv, D);
    if (rc != KV_OK) return rc;

    unsigned char *base = slot.base;
    __half *qbuf = reinterpret_cast<__half *>(base + off_q);
    unsigned *ctl = reinterpret_cast<unsigned *>(base + off_ctl);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

    if (wrapped && cudaMemsetAsync(base + off_st, 0, off_acc - off_st, st) != cudaSuccess)
        return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: clearing the statistics slots failed");
    if (cudaMemsetAsync(base + off_acc, 0, zero_bytes, st) != cudaSuccess)
        return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: clearing the accumulators failed");
    const int nq = n_head * D;
    q_to_f16_kernel<<<(nq + 255) / 256, 256, 0, st>>>(q, qbuf, nq);
    if (cudaGetLastError() != cudaSuccess) return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: launch failed");

    ap.hkv = hkv;
    ap.r = r;
    ap.hq_loc = n_head;
    ap.n_kv = n_kv;
    ap.n_past = n_kv - 1;
    ap.scale = 1.0f / sqrtf((float)D);
    ap.qbuf = qbuf;
    ap.hz_row = -1;
    ap.S = reinterpret_cast<float *>(base + off_s);
    ap.stats = reinterpret_cast<unsigned long long *>(base + off_st);
    ap.acc = reinterpret_cast<long long *>(base + off_acc);
    ap.counters = ctl;
    ap.nonfin = ctl + hkv;
    ap.xticket = ctl + 2 * hkv;
    ap.err = ctl + 2 * hkv + 1;
    ap.limit_ns = 1000000000ull;
    ap.out = out;
    ap.out_stride = (int64_t)n_head * D;
    ap.cq = 1;
    ap.ncl = 1;
    for (int i = 0; i < launches; i++) {
        ap.row0 = i * rows_per;
        ap.nrows = std::min(rows_per, r - ap.row0);
        ap.epoch = epoch0 + (uint32_t)i;
        if (kvb::launch_attn(D, km, vm, ap, st, false, true) != cudaSuccess)
            return kvb::set_last_error(KV_E_CUDA, "kv_attend_decode_noalloc: attention launch failed");
    }
    kvb::set_last_error(KV_OK, "");
    return KV_OK;
}
