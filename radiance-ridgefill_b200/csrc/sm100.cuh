/* sm100.cuh -- thin wrappers over the sm_100a PTX this library's tensor-core kernels issue: mbarriers,
 * TMA tile loads, tensor-memory allocation, tcgen05.mma and tcgen05.ld, and a bounded mbarrier wait.
 *
 * Every wait on an mbarrier is bounded: after kWaitTimeoutNs of global time without the phase
 * completing, the waiter records an error code in ridgefill_device_error, raises the CTA's abort flag
 * (so the other roles stop waiting too) and returns false; the kernel then drains what it issued and
 * frees its tensor memory. A GPU is never left spinning.
 */
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rf {

/* Set (first error wins) by a kernel that gave up waiting; read with ridgefill_device_error(). One copy
 * per translation unit that includes this header (no relocatable device code); the library's accessor
 * reads every copy. */
static __device__ int g_device_error = 0;

/* This translation unit's copy of g_device_error (host code; synchronises). `reset` clears it. */
static inline int read_device_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof v) != cudaSuccess) return -1;
    if (reset) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof zero) != cudaSuccess) return -1;
    }
    return v;
}

/* The DeltaNet fill's copy (gdn.cu). */
int gdn_device_error(int reset);
int peer_device_error(int reset);

enum DeviceError : int {
    kErrNone = 0,
    kErrGemmWaitProducer = 0x101,
    kErrGemmWaitMma = 0x102,
    kErrGemmWaitEpilogue = 0x103,
    kErrGemmDrain = 0x104,
    kErrGdnWait = 0x201,
};

constexpr uint64_t kWaitTimeoutNs = 2000000000ull;   /* 2 s */

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

/* Make the initialised barriers visible to the async proxy (TMA, tensor cores). */
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

/* Wait for the phase of `bar` with parity `parity`; false (and *abort raised, the error recorded)
 * after the timeout, or at once when another role already raised *abort. */
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*abort) return false;
            if (global_ns() - t0 > kWaitTimeoutNs) {
                *abort = 1;
                atomicCAS(&g_device_error, 0, err);
                return false;
            }
        }
    }
}

/* 2-D TMA tile load into shared memory, completing `bytes` on `bar`. (x, y): innermost coordinate
 * first, in elements. One destination CTA. */
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_addr(dst)), "l"((uint64_t)map), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

/* 3-D TMA tile load (coordinates innermost first, in elements), completing on `bar`. One destination CTA. */
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_addr(dst)), "l"((uint64_t)map), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

/* Bulk (non-tensor) copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global to
 * shared memory, completing on `bar`. One destination CTA. */
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

/* 2-D TMA tile store from shared memory (the tensor map's box and swizzle), in the current bulk group;
 * rows and columns outside the tensor are not written. The writers of the source make it visible first
 * (fence_proxy_async_smem). */
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"((uint64_t)map), "r"(smem_addr(src)), "r"(x), "r"(y)
                 : "memory");
}

/* Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from shared to global memory
 * in the current bulk group. The writers of the source make it visible first (fence_proxy_async_smem,
 * then a barrier); bulk_store_commit closes the group. */
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_addr(src)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
/* The committed bulk stores have read their sources (the shared memory may be written again). */
__device__ __forceinline__ void bulk_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
/* The committed bulk stores are complete. */
__device__ __forceinline__ void bulk_store_wait() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
/* Every committed bulk store group but the most recent one is complete. */
__device__ __forceinline__ void bulk_store_wait_prior() { asm volatile("cp.async.bulk.wait_group 1;" ::: "memory"); }
/* Generic-proxy writes to shared memory become visible to the async proxy (bulk copies, TMA). */
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

/* The driver's tensor-map encoder, resolved once through the runtime (no link against libcuda). */
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)f;
    }
    return fn;
}

/* ------------------------------------------------------------------ tensor memory */

template <uint32_t kCols>
__device__ __forceinline__ void tmem_alloc(uint32_t* slot) {   /* whole warp */
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

template <uint32_t kCols>
__device__ __forceinline__ void tmem_free(uint32_t base) {   /* whole warp */
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(kCols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

/* Shared-memory matrix descriptor of a K-major operand tile written by TMA with 128-byte swizzle:
 * rows of 128 bytes, 8-row groups 1024 bytes apart (SBO), LBO unused (1), descriptor version 1. */
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3ffffu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

/* Shared-memory matrix descriptor of an MN-major operand tile with 128-byte swizzle: 64 consecutive 16-bit
 * MN elements a 128-byte row, consecutive K in consecutive rows, 8-row groups 1024 bytes apart (SBO), the
 * next 64 MN elements `mn_block_bytes` further (LBO); descriptor version 1. */
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t saddr, uint32_t mn_block_bytes) {
    uint64_t d = (uint64_t)((saddr & 0x3ffffu) >> 4);
    d |= (uint64_t)((mn_block_bytes >> 4) & 0x3fffu) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

/* D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, one CTA. */
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* D[tmem] (+)= A[smem] * B[smem]^T, f16 x f16 -> f32 (kind::f16), one CTA. */
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* D[tmem] (+)= A[tmem] * B[smem]^T, f16 x f16 -> f32 (kind::f16), one CTA; A's row m in lane m, two
 * elements a 32-bit column along K. */
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* ------------------------------------------------------------------ CTA pairs (cta_group::2)
 * Two CTAs of a 2-CTA cluster share one tcgen05.mma: A's M = 256 rows are split 128 / 128 between the CTAs'
 * shared memory, B's N columns likewise split in halves, and each CTA's tensor memory holds the D rows of its
 * own A rows (all N columns). The even CTA (rank 0) issues the MMAs; every tcgen05 instruction of such a
 * kernel uses cta_group::2. */

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}

/* The shared::cluster address of the object at this CTA's shared address `saddr` in CTA `rank`. */
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

/* Every thread of every CTA of the cluster; orders the threads' prior memory operations (barrier
 * initialisation included) before any thread's later ones. */
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

/* Arrive (release, cluster scope) on an mbarrier given by its shared::cluster address, in any CTA of the cluster. */
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}

/* Packed f32x2 arithmetic (sm_100): two lanes of f32 per instruction, each rounded as its scalar form. */
__device__ __forceinline__ void fma2_rn(float& a0, float& a1, float x0, float x1, float y0, float y1) {   /* a = x * y + a */
    asm("{\n .reg .b64 a, x, y;\n mov.b64 a, {%0, %1};\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %5};\n"
        " fma.rn.f32x2 a, x, y, a;\n mov.b64 {%0, %1}, a;\n}"
        : "+f"(a0), "+f"(a1) : "f"(x0), "f"(x1), "f"(y0), "f"(y1));
}
/* Named barrier `id` over `threads` threads (a multiple of 32). */
__device__ __forceinline__ void bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

/* Named barrier `id` over `threads` threads that also ORs `pred` across them: every thread gets the same answer. */
__device__ __forceinline__ bool bar_any(int id, int threads, bool pred) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.or.pred q, %2, %3, p;\n\t"
                 "selp.u32 %0, 1, 0, q;\n\t}\n"
                 : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(threads) : "memory");
    return r != 0;
}

/* SiLU u / (1 + e^-u) as u times the approximate reciprocal (1 ulp) of the denominator, with the fast exp: well
 * inside bf16's rounding. The reciprocal is the non-flushing form, so a denominator above 2^126 (u below about
 * -87.3, where the value is about u e^u, under 1e-36 in magnitude) still gives the tiny value the f32 rule gives,
 * not 0; an infinite one (u below about -88.7) gives -0, as the division does. */
__device__ __forceinline__ float silu(float u) {
    float r;
    asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(1.0f + __expf(-u)));
    return u * r;
}

__device__ __forceinline__ void sub2_rn(float& d0, float& d1, float x0, float x1, float y0, float y1) {   /* d = x - y */
    asm("{\n .reg .b64 d, x, y;\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %5};\n sub.rn.f32x2 d, x, y;\n"
        " mov.b64 {%0, %1}, d;\n}"
        : "=f"(d0), "=f"(d1) : "f"(x0), "f"(x1), "f"(y0), "f"(y1));
}

__device__ __forceinline__ void mul2_rn(float& d0, float& d1, float x0, float x1, float y0, float y1) {
    asm("{\n .reg .b64 d, x, y;\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %5};\n mul.rn.f32x2 d, x, y;\n"
        " mov.b64 {%0, %1}, d;\n}"
        : "=f"(d0), "=f"(d1) : "f"(x0), "f"(x1), "f"(y0), "f"(y1));
}

/* A relaxed arrive (no release fence) on a barrier of this cluster: for hand-overs whose data needs no
 * ordering through memory -- a tensor-memory buffer whose reads the arriving thread has already waited for
 * (tcgen05.wait::ld), so the arrive only says that the columns may be overwritten. */
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t caddr) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}

/* Tensor memory of a CTA pair: the same warp of both CTAs allocates, each CTA receiving kCols columns at the
 * same address (written to its own `slot`). */
template <uint32_t kCols>
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot) {   /* whole warp, both CTAs */
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <uint32_t kCols>
__device__ __forceinline__ void tmem_free_pair(uint32_t base) {   /* whole warp, both CTAs */
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(kCols) : "memory");
}

/* 2-D TMA tile load into this CTA's shared memory whose bytes complete on the mbarrier at shared::cluster
 * address `bar_caddr`, which may be the pair's other CTA's. One destination CTA. */
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_caddr, int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_addr(dst)), "l"((uint64_t)map), "r"(bar_caddr), "r"(x), "r"(y)
        : "memory");
}

/* D[tmem] (+)= A[smem] * B[smem]^T over the CTA pair, int8 x int8 -> int32. Rank 0 issues. */
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* D[tmem] (+)= A[smem] * B[smem]^T over the CTA pair, f16 / bf16 -> f32 (kind::f16). Rank 0 issues. */
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* Arrive on the mbarrier at shared::cluster address `bar_caddr` (either CTA of the pair) once every pair MMA
 * this thread issued so far has completed. */
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_caddr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_caddr) : "memory");
}

/* Arrive on `bar` once every tcgen05.mma this thread issued so far has completed. */
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

/* 32 consecutive 32-bit columns of this thread's tensor-memory lane. */
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

/* 16 bytes global -> shared through L2 (cp.async.cg); `bytes` 16 copies, 0 writes zeros and reads nothing. */
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

/* 8 consecutive 32-bit columns of this thread's tensor-memory lane. */
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

/* 16 consecutive 32-bit columns of this thread's tensor-memory lane. */
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
                   "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

/* Store 32 consecutive 32-bit columns of this thread's tensor-memory lane. */
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
          "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
          "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
          "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

/* Store 16 consecutive 32-bit columns of this thread's tensor-memory lane. */
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
          "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

/* Store 8 consecutive 32-bit columns of this thread's tensor-memory lane. */
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace rf
