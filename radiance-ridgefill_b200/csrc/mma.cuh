/* mma.cuh -- warp-level tensor-core tiles (m16n8k16, f32 accumulate) and shared-memory matrix loads,
 * for the small, latency-bound matrices of the Gated DeltaNet fill.
 *
 * Fragment layouts (g = lane / 4, t = lane % 4):
 *   A 16x16:  a0 (g, 2t..2t+1)  a1 (g+8, 2t..)  a2 (g, 2t+8..)  a3 (g+8, 2t+8..)
 *   B 16x8:   b0 (k 2t..2t+1, n g)              b1 (k 2t+8.., n g)
 *   C 16x8:   c0,c1 (g, 2t..2t+1)               c2,c3 (g+8, 2t..2t+1)
 * so the C tiles of columns [16s, 16s+8) and [16s+8, 16s+16) pack into the A fragment of k-step s:
 * a result feeds the next product from registers (c_to_a).
 */
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace rf {

__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

/* A fragment of the 16x16 block at (row0, col0) of a row-major [m][k] b16 matrix, pitch in elements. */
__device__ __forceinline__ void load_a(uint32_t (&a)[4], const void* base, int pitch, int row0, int col0) {
    const int l = threadIdx.x & 31, mi = l >> 3, r = l & 7;
    const uint16_t* p = (const uint16_t*)base + (row0 + r + (mi & 1) * 8) * pitch + col0 + (mi >> 1) * 8;
    ldsm_x4(a, saddr(p));
}

/* B fragments of two n-tiles (n0..n0+7, n0+8..n0+15) x k16 at k0, from a row-major [n][k] matrix:
 * b[0], b[1] the first tile, b[2], b[3] the second. */
__device__ __forceinline__ void load_b_nk(uint32_t (&b)[4], const void* base, int pitch, int n0, int k0) {
    const int l = threadIdx.x & 31, mi = l >> 3, r = l & 7;
    const uint16_t* p = (const uint16_t*)base + (n0 + r + (mi >> 1) * 8) * pitch + k0 + (mi & 1) * 8;
    ldsm_x4(b, saddr(p));
}

/* The same fragments from a row-major [k][n] matrix (transposing load). */
__device__ __forceinline__ void load_b_kn(uint32_t (&b)[4], const void* base, int pitch, int k0, int n0) {
    const int l = threadIdx.x & 31, mi = l >> 3, r = l & 7;
    const uint16_t* p = (const uint16_t*)base + (k0 + r + (mi & 1) * 8) * pitch + n0 + (mi >> 1) * 8;
    ldsm_x4_t(b, saddr(p));
}

/* Byte offset of element (row, col) in a b16 tile of 64-column halves, each half [rows][64] with its rows
 * of 128 bytes and 128-byte swizzle (16-byte chunk j of row r at chunk j ^ (r & 7)), halves `half` bytes
 * apart: the layout TMA writes for a [64 rows][64] box with CU_TENSOR_MAP_SWIZZLE_128B, and the layout
 * this library keeps its own f16 tiles in. col & 7 selects the element inside the chunk. */
__device__ __forceinline__ uint32_t sw128_off(int row, int col, int half = 8192) {
    return (uint32_t)((col >> 6) * half + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}

/* Shared-memory byte address of element (row, col) of a [64][128] tile in that layout (two halves of
 * [64][64]); `tile` 1024-byte aligned when TMA wrote it. */
__device__ __forceinline__ uint32_t sw128_addr(uint32_t tile, int row, int col) { return tile + sw128_off(row, col); }

/* load_a / load_b_nk / load_b_kn on such a tile. */
__device__ __forceinline__ void load_a_sw(uint32_t (&a)[4], uint32_t tile, int row0, int col0) {
    const int l = threadIdx.x & 31, mi = l >> 3, r = l & 7;
    ldsm_x4(a, sw128_addr(tile, row0 + r + (mi & 1) * 8, col0 + (mi >> 1) * 8));
}
__device__ __forceinline__ void load_b_nk_sw(uint32_t (&b)[4], uint32_t tile, int n0, int k0) {
    const int l = threadIdx.x & 31, mi = l >> 3, r = l & 7;
    ldsm_x4(b, sw128_addr(tile, n0 + r + (mi >> 1) * 8, k0 + (mi & 1) * 8));
}
__device__ __forceinline__ void load_b_kn_sw(uint32_t (&b)[4], uint32_t tile, int k0, int n0) {
    const int l = threadIdx.x & 31, mi = l >> 3, r = l & 7;
    ldsm_x4_t(b, sw128_addr(tile, k0 + r + (mi & 1) * 8, n0 + (mi >> 1) * 8));
}
/* The A fragment of the 16x16 block (m0, k0) of A = X^T, X [k][m] stored in such a tile (transposing load). */
__device__ __forceinline__ void load_a_t_sw(uint32_t (&a)[4], uint32_t tile, int k0, int m0) {
    const int l = threadIdx.x & 31, mi = l >> 3, r = l & 7;
    ldsm_x4_t(a, sw128_addr(tile, k0 + r + (mi >> 1) * 8, m0 + (mi & 1) * 8));
}

__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *(const uint32_t*)&h;
}

/* The A fragment of k-step s from two f32 C tiles c[2s], c[2s+1] (each [4]), rounded to f16. */
__device__ __forceinline__ void c_to_a(uint32_t (&a)[4], const float (&lo)[4], const float (&hi)[4]) {
    a[0] = pack_f16(lo[0], lo[1]);
    a[1] = pack_f16(lo[2], lo[3]);
    a[2] = pack_f16(hi[0], hi[1]);
    a[3] = pack_f16(hi[2], hi[3]);
}

/* cp.async of 16 bytes; src_bytes 0 fills the destination with zeros and reads nothing. */
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr(dst)), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

}  // namespace rf
