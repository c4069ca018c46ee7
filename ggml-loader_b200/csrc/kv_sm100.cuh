// kv_sm100.cuh -- thin inline-PTX helpers for sm_100a: mbarriers with bounded
// waits, TMA tensor loads, named barriers, the global nanosecond timer and the
// programmatic-dependent-launch controls.
//
// Every wait here is bounded: a wait that has not completed after
// `limit_ns` nanoseconds (%globaltimer) returns false so the caller can record
// an error word and leave the kernel instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace kvb {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete; false after limit_ns.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t n = 1;; n++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 15u) == 0 && globaltimer() - t0 > limit_ns) return false;
    }
}

// As mbar_wait, but also gives up (false) as soon as *abort is non-zero.
__device__ __forceinline__ bool mbar_wait_ab(uint64_t *bar, uint32_t parity, uint64_t limit_ns,
                                             const volatile int *abort)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t n = 1;; n++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 15u) == 0 && (*abort || globaltimer() - t0 > limit_ns)) return false;
    }
}

// ---- TMA ---------------------------------------------------------------------
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *m)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 3-D tiled load into shared memory, completion counted on `bar` (bytes).
// The innermost coordinate x must be a multiple of 16 bytes / element size.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *m, uint64_t *bar, int x, int y, int z)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// The CTA-pair form: the tile lands in this CTA's shared memory and its bytes
// complete on `bar_cluster`, an mbarrier of either CTA of the pair (a
// shared::cluster address from mapa).
__device__ __forceinline__ void tma_load_3d_pair(void *dst, const CUtensorMap *m, uint32_t bar_cluster, int x, int y,
                                                 int z)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
        "%5}], [%2];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// L2 policy for data read once (streamed K/V tiles): evicted before other lines
__device__ __forceinline__ uint64_t policy_evict_first()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ uint64_t policy_evict_last()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 16-byte store / L2-only load with an L2 eviction-priority policy
__device__ __forceinline__ void st_v4_hint(float *p, float4 v, uint64_t pol)
{
    asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w), "l"(pol)
                 : "memory");
}

__device__ __forceinline__ float4 ld_cg_v4_hint(const float *p, uint64_t pol)
{
    float4 v;
    asm volatile("ld.global.cg.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}

__device__ __forceinline__ void tma_load_3d_hint(void *dst, const CUtensorMap *m, uint64_t *bar, int x, int y, int z,
                                                 uint64_t pol)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
        "[%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z), "l"(pol)
        : "memory");
}

// 3-D tile of a tensor map into L2 only (no shared memory, no barrier); the
// innermost coordinate x follows tma_load_3d's alignment rule
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap *m, int x, int y, int z)
{
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(x), "r"(y), "r"(z)
                 : "memory");
}

// drop a dead 128-byte line from L2 without writing it back (scratch that is
// rewritten before it is read again)
__device__ __forceinline__ void l2_discard(const void *p)
{
    asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}

__device__ __forceinline__ void l2_prefetch(const void *p)
{
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *m, uint64_t *bar, int x, int y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

// ---- warp-level tensor-core fragments ------------------------------------------
// ldmatrix: four 8x8 b16 matrices; lane l supplies the row address of matrix
// l/8, row l%8.  .trans delivers each matrix transposed.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col): products of F16
// values are exact in F32 and accumulate in F32.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi)
{
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// ---- barriers / dependent launch ----------------------------------------------
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate over the participating threads:
// every thread gets the same answer, so a bounded wait that failed in one
// thread turns into a uniform decision to leave.
__device__ __forceinline__ bool named_sync_or(uint32_t id, uint32_t nthreads, bool pred)
{
    uint32_t res;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(res)
        : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
        : "memory");
    return res != 0;
}

// ---- per-thread asynchronous copies (L2 -> shared, 16 bytes) ---------------------
__device__ __forceinline__ void cp_async_16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit()
{
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- cross-CTA slots ------------------------------------------------------------
__device__ __forceinline__ unsigned ld_volatile_u32(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Ticket: an add with release (everything this CTA wrote before the barrier
// that precedes it) and acquire (what the CTAs counted in before wrote)
// semantics at GPU scope.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned *p, unsigned v)
{
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ void st_volatile_u32(unsigned *p, unsigned v)
{
    asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 16-byte stores / loads of two 64-bit words for cross-CTA slots; each word is
// single-copy atomic, the pair is not (readers check both words).
__device__ __forceinline__ void st_volatile_v2(unsigned long long *p, unsigned long long a, unsigned long long b)
{
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ void ld_volatile_v2(const unsigned long long *p, unsigned long long &a,
                                               unsigned long long &b)
{
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// ---- thread-block clusters: distributed shared memory ------------------------------
// A cluster's CTAs are resident together on one GPC; each can address the
// others' shared memory through the shared::cluster window (mapa).  Only this
// GPU's own shared memory is reached this way.
__device__ __forceinline__ uint32_t cluster_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// every thread of every CTA in the cluster: arrive (release) and wait (acquire)
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// the shared::cluster address of the same offset in CTA `rank`'s shared memory
__device__ __forceinline__ uint32_t mapa(uint32_t local_addr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void st_cluster_v2(uint32_t addr, float a, float b)
{
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float4 v)
{
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

// asynchronous stores into another CTA's shared memory (addresses from mapa):
// each completes `bytes` of the transaction count of the mbarrier `remote_bar`
// in that CTA, whose wait then sees the data
__device__ __forceinline__ void st_async_v2(uint32_t addr, float a, float b, uint32_t remote_bar)
{
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(addr),
                 "f"(a), "f"(b), "r"(remote_bar)
                 : "memory");
}

__device__ __forceinline__ void st_async_v4(uint32_t addr, float4 v, uint32_t remote_bar)
{
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     addr),
                 "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(remote_bar)
                 : "memory");
}

// the two halves of a cluster barrier phase: every thread of every CTA arrives
// once (release) and later waits once (acquire)
__device__ __forceinline__ void cluster_arrive()
{
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait()
{
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// arrive on an mbarrier in another CTA of the cluster (address from mapa),
// releasing at cluster scope what this thread -- and, through a preceding CTA
// barrier, its CTA -- wrote before
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote_bar)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}

// arrive on an mbarrier of either CTA of the cluster (address from mapa) with
// the default semantics (release at CTA scope, no cluster-wide fence): for
// hand-offs whose data the tensor cores read after tcgen05 fences (TMEM
// written with tcgen05.st, then tcgen05.wait::st and
// tcgen05.fence::before_thread_sync), as the CTA-pair pipelines do
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar)
{
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits (acquiring at cluster scope) for the phase with the given parity; false after limit_ns.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, uint64_t limit_ns)
{
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t n = 1;; n++) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((n & 15u) == 0 && globaltimer() - t0 > limit_ns) return false;
    }
}

// ---- 5th-generation tensor cores: TMEM and tcgen05.mma ----------------------------
// Tensor memory: 128 lanes x up to 512 columns of 32-bit cells per SM.  An
// address is (lane << 16) | column.  Allocation, relinquish and deallocation
// are warp-wide (.sync.aligned).
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// The CTA-pair forms (cta_group::2): one warp of each CTA of a 2-CTA cluster
// (the same warp in both) allocates, relinquishes and frees; the pair's
// columns have the same address in both CTAs.  A kernel uses one cta_group
// in all its tcgen05 instructions.
__device__ __forceinline__ void tmem_alloc2(uint32_t *dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish2()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Order tcgen05 operations against thread synchronisation (mbarrier, bar.sync).
__device__ __forceinline__ void tc_fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 bytes
// (64 halves) with the 16-byte chunks XOR-ed by (row & 7) -- the layout a TMA
// box of 64 halves with CU_TENSOR_MAP_SWIZZLE_128B writes -- 8-row groups 1024
// bytes apart.  The tile must start 1024-byte aligned; a step of 16 halves
// along K within a row advances the start address by 32 bytes.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// The same swizzled boxes read MN-major (the contiguous 64 halves of a row run
// along M or N): 64-element chunks of M/N `chunk_bytes` apart, 8-row groups
// along K 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t saddr, uint32_t chunk_bytes)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((chunk_bytes >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16 with F16 inputs and F32 accumulation.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N, bool b_mn_major)
{
    return (1u << 4) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem desc] * B[smem desc]; issued by one thread.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// The mbarrier gets one arrival once every tcgen05.mma this thread issued so far
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// The CTA pair's MMA, issued by one thread of the even CTA: M = 256 rows, the
// first 128 from the even CTA's A (shared memory or TMEM) into its TMEM, the
// others from the odd CTA's, at the same addresses; B's N columns are split,
// the first N/2 in the even CTA's shared memory, the rest in the odd one's.
__device__ __forceinline__ void umma_ss2(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_ts2(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// One arrival on `bar` in this CTA once the pair MMAs this thread issued have
// completed; the second form arrives on `bar` in every CTA of `cta_mask`
// (bar's offset in each).
__device__ __forceinline__ void umma_commit2(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void umma_commit2_mc(uint64_t *bar, uint16_t cta_mask)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                     "r"(smem_addr(bar)),
                 "h"(cta_mask)
                 : "memory");
}

// 32 consecutive 32-bit columns of this thread's lane (warp w reaches lanes
// 32*(w%4) .. +31); complete after tmem_wait_ld.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// 16 consecutive 32-bit columns of this thread's lane <- r; visible to
// tcgen05.mma after tmem_wait_st + tc_fence_before + a thread sync.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st()
{
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]: A is M rows (lanes) x 16-bit K values
// packed two per column (the lower half holds the even K index).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, bool accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// 16 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld()
{
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2^x, hardware approximation (flushes subnormal results to zero)
__device__ __forceinline__ float ex2_approx(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous kernel's results to be visible.
__device__ __forceinline__ void pdl_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

}  // namespace sm100
}  // namespace kvb
