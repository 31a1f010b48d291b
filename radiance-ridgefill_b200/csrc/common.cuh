/* common.cuh -- helpers shared by the B200 RidgeFill device rows. */
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "ridgefill.h"

namespace rf {

constexpr int kSMs = 148;   /* B200: 2 dies x 74 SMs; grids are sized in multiples of it */

/* RAD_OK when the launch just issued on this thread was accepted, RAD_E_DEVICE otherwise. */
inline int launch_status() { return cudaGetLastError() == cudaSuccess ? RAD_OK : RAD_E_DEVICE; }

inline cudaStream_t as_stream(RadStream s) { return (cudaStream_t)s; }

/* The number of SMs of the current device (148 on B200), queried once per process. */
inline int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0, v = 0;
        if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
            n = v;
        else
            n = kSMs;
    }
    return n;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

/* f32 -> bf16 bits, round to nearest even (NaN kept quiet), the same rule as the host rad_f32_to_bf16. */
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* Two f32 values as a pair of bf16 (lo in the low half), each rounded as f32_to_bf16_bits. */
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
}

/* Start of sequence i: cu[i] clamped to [0, T]. */
__device__ __forceinline__ int64_t seq_start(const int32_t* cu, int64_t T, int64_t i) {
    return min(max((int64_t)cu[i], (int64_t)0), T);
}

/* The sequence holding row r of a T-row batch split by cu_seqlens `cu` (n_seq + 1 entries): the last i whose clamped
 * start is <= r, if r lies before its clamped end (its start and end in *s0, *e0); -1 otherwise. Values outside
 * [0, T] are clamped, the fill's rule. */
__device__ inline int find_seq(const int32_t* cu, int64_t n_seq, int64_t T, int64_t r, int64_t* s0, int64_t* e0) {
    if (n_seq <= 0 || seq_start(cu, T, 0) > r) return -1;
    int64_t lo = 0, hi = n_seq - 1;
    while (lo < hi) {
        const int64_t mid = (lo + hi + 1) >> 1;
        if (seq_start(cu, T, mid) <= r) lo = mid;
        else hi = mid - 1;
    }
    const int64_t a = seq_start(cu, T, lo), b = min(max((int64_t)cu[lo + 1], a), T);
    if (r >= b) return -1;
    *s0 = a;
    *e0 = b;
    return (int)lo;
}

}  // namespace rf
