/* peer.cu -- the tensor-parallel team's NVLink kernels: one process per GPU, each rank's buffers mapped into its
 * peers' address spaces (CUDA IPC), and three kernels that move data and order the ranks without a library
 * collective:
 *
 *   ridgefill_gather_columns  a rank's column block [c0, c1) of a [rows, ld] bf16 matrix stored into the same place
 *                             of every peer's copy (plain 16-byte stores to peer memory over NVLink), then one
 *                             arrival a CTA added to each peer's counter `slot` (release, system scope);
 *   ridgefill_team_wait       one thread waits (acquire, system scope; bounded) until this rank's counter `slot`
 *                             holds `expected` arrivals, so the kernels after it on the stream read the gathered data;
 *   ridgefill_team_barrier    an arrival on every peer's counter `slot`, then the wait for all peers' arrivals: no
 *                             rank starts what follows before every rank has finished what precedes it on its stream.
 *
 * The reference has none of this: its engine replicates the projector on every rank and reduces with its own
 * all-reduce (notes/tp-map.md:28-29,48-49). Counters only grow (64-bit, one pass adds a known amount), so nothing is
 * reset between passes and a late arrival can never be mistaken for a fresh one. Every wait gives up after 2 s of
 * global time, records kErrTeamWait (ridgefill_device_error) and returns: a rank that died leaves the others with
 * an error, not a hang. No multicast of any kind: peer memory is reached by ordinary stores and atomics only.
 */
#include <cuda.h>

#include <cstring>

#include "common.cuh"
#include "ridgefill_team.h"
#include "sm100.cuh"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kGatherThreads = 512;
constexpr int kErrTeamWait = 0x301;

struct GatherCols {
    const uint16_t* src;              /* this rank's copy: its block is read from here */
    uint16_t* dst[kMaxRanks];         /* every rank's copy as mapped here (dst[rank] unused) */
    unsigned long long* flag[kMaxRanks];   /* every rank's counters as mapped here */
    int64_t rows, ld, c0, c1;         /* elements */
    int rank, world, slot;
};

__device__ __forceinline__ void red_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kGatherThreads) gather_cols_kernel(const GatherCols g) {
    const int64_t per_row = (g.c1 - g.c0) / 8;   /* 16-byte words of the block in a row */
    const int64_t words = g.rows * per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / per_row;
        const int64_t off = r * g.ld + g.c0 + (i - r * per_row) * 8;
        const uint4 v = *(const uint4*)(g.src + off);
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
            if (p < g.world && p != g.rank) *(uint4*)(g.dst[p] + off) = v;
    }
    __threadfence_system();   /* this thread's peer stores before the CTA's arrival */
    __syncthreads();
    if (threadIdx.x == 0)
        for (int p = 0; p < g.world; ++p)
            if (p != g.rank) red_release_sys(g.flag[p] + g.slot, 1ull);
}

/* Bounded wait of one thread for counter `slot` to reach `expected`; false (and kErrTeamWait) when it gave up. */
__device__ bool wait_count(const unsigned long long* flag, int slot, unsigned long long expected) {
    if (ld_acquire_sys(flag + slot) >= expected) return true;
    const uint64_t t0 = rf::global_ns();
    while (ld_acquire_sys(flag + slot) < expected) {
        if (rf::global_ns() - t0 > rf::kWaitTimeoutNs) {
            atomicCAS(&rf::g_device_error, 0, kErrTeamWait);
            return false;
        }
        __nanosleep(256);
    }
    return true;
}

__global__ void team_wait_kernel(const unsigned long long* flag, int slot, unsigned long long expected) {
    if (threadIdx.x == 0) wait_count(flag, slot, expected);
}

struct BarrierArgs {
    unsigned long long* flag[kMaxRanks];
};

__global__ void team_barrier_kernel(const BarrierArgs b, int rank, int world, int slot, unsigned long long expected) {
    if (threadIdx.x != 0) return;
    __threadfence_system();
    for (int p = 0; p < world; ++p)
        if (p != rank) red_release_sys(b.flag[p] + slot, 1ull);
    wait_count(b.flag[rank], slot, expected);
}

/* The base of the allocation holding `ptr` (cuMemGetAddressRange through the runtime's entry-point query). */
bool allocation_base(const void* ptr, void** base) {
    typedef CUresult (*GetRange)(CUdeviceptr*, size_t*, CUdeviceptr);
    static GetRange fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return false;
        fn = (GetRange)f;
    }
    CUdeviceptr b = 0;
    size_t n = 0;
    if (fn(&b, &n, (CUdeviceptr)ptr) != CUDA_SUCCESS) return false;
    *base = (void*)b;
    return true;
}

}  // namespace

/* This translation unit's copy of the device error word (sm100.cuh), for ridgefill_device_error. */
namespace rf {
int peer_device_error(int reset) { return read_device_error(reset); }
}

extern "C" int ridgefill_team_gather_ctas(void) { return 64; }

extern "C" int ridgefill_peer_export(const void* ptr, void* handle, int64_t* offset) {
    if (!ptr || !handle || !offset) return RAD_E_INVAL;
    void* base = nullptr;
    if (!allocation_base(ptr, &base)) return RAD_E_DEVICE;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, base) != cudaSuccess) return RAD_E_DEVICE;
    memcpy(handle, &h, sizeof h);
    *offset = (int64_t)((const char*)ptr - (const char*)base);
    return RAD_OK;
}

extern "C" int ridgefill_peer_import(const void* handle, int64_t offset, void** ptr) {
    if (!handle || !ptr || offset < 0) return RAD_E_INVAL;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void* base = nullptr;
    if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return RAD_E_DEVICE;
    *ptr = (char*)base + offset;
    return RAD_OK;
}

extern "C" int ridgefill_peer_release(void* ptr, int64_t offset) {
    if (!ptr || offset < 0) return RAD_E_INVAL;
    return cudaIpcCloseMemHandle((char*)ptr - offset) == cudaSuccess ? RAD_OK : RAD_E_DEVICE;
}

extern "C" int ridgefill_gather_columns(const uint16_t* src, uint16_t* const* dst, unsigned long long* const* flags, int rank,
                                        int world, int64_t rows, int64_t ld, int64_t c0, int64_t c1, int slot, RadStream s) {
    if (!src || !dst || !flags || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || slot < 0) return RAD_E_INVAL;
    if (rows < 0 || c0 < 0 || c1 < c0 || c1 > ld) return RAD_E_SHAPE;
    if (((uintptr_t)src | (uintptr_t)(ld * 2) | (uintptr_t)(c0 * 2) | (uintptr_t)(c1 * 2)) % 16) return RAD_E_STRIDE;
    GatherCols g{};
    g.src = src;
    for (int p = 0; p < world; ++p) {
        if (p != rank && (!dst[p] || !flags[p] || (uintptr_t)dst[p] % 16)) return RAD_E_INVAL;
        g.dst[p] = dst[p];
        g.flag[p] = flags[p];
    }
    g.rows = rows;
    g.ld = ld;
    g.c0 = c0;
    g.c1 = c1;
    g.rank = rank;
    g.world = world;
    g.slot = slot;
    if (world == 1) return RAD_OK;
    gather_cols_kernel<<<ridgefill_team_gather_ctas(), kGatherThreads, 0, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}

extern "C" int ridgefill_team_wait(const unsigned long long* own, int slot, unsigned long long expected, RadStream s) {
    if (!own || slot < 0) return RAD_E_INVAL;
    team_wait_kernel<<<1, 32, 0, rf::as_stream(s)>>>(own, slot, expected);
    return rf::launch_status();
}

extern "C" int ridgefill_team_barrier(unsigned long long* const* flags, int rank, int world, int slot,
                                      unsigned long long expected, RadStream s) {
    if (!flags || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || slot < 0) return RAD_E_INVAL;
    BarrierArgs b{};
    for (int p = 0; p < world; ++p) {
        if (!flags[p]) return RAD_E_INVAL;
        b.flag[p] = flags[p];
    }
    if (world == 1) return RAD_OK;
    team_barrier_kernel<<<1, 32, 0, rf::as_stream(s)>>>(b, rank, world, slot, expected);
    return rf::launch_status();
}
