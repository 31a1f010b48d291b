/* gdn.cu -- ridgefill_gdn_fill: the Gated DeltaNet chunk fill on B200.
 *
 * In the reference this is radiance libr4d's gdn_conv_prep -> gdn_kkt_solve -> gdn_chunk_scan, issued by
 * the adapter (arch/qwen4exp_fill.h:36-61; split scan arch/qwen4exp_blocks.h:110-157); no source of it
 * is available. The rule it computes, per v-head h (k-head h / (Hv/Hk)) and row t:
 *     S <- exp(g_t) S;   S <- S + beta_t (v_t - S k_t) k_t^T;   o_t = scale * S q_t
 * (Yang, Kautz & Hatamizadeh, "Gated Delta Networks", arXiv:2412.06464), state S [dv, dk] f32.
 *
 * Chunk form, chunks of C = 64 rows anchored at each sequence's first row. With G the in-chunk
 * cumulative log decay and gamma = exp(G), the chunk's corrected values u solve
 *     (I + A) u = diag(beta) v - diag(beta gamma) K S0^T,   A_ij = beta_i exp(G_i - G_j) k_i.k_j (j < i)
 * so with T = (I + A)^-1:  U = T (beta v) - T (beta gamma K) S0^T = U~ - W S0^T, and at the chunk end
 *     S_L = gamma_L S0 + U^T diag(exp(G_L - G)) K.
 *
 *   phase 1 (gdn_prep_kernel), every (chunk, head) in parallel, persistent CTAs, the next item's k rows
 *     arriving by TMA (two 128-byte-swizzled boxes) while the current one is computed: K K^T on tensor
 *     cores (bf16, exact inputs), A, T by blocked inversion (16x16 diagonal blocks by substitution in
 *     f32, off-diagonal blocks by f16 tensor-core products) and W = T (beta gamma K). T and W (f16) are
 *     written to the chunk's scratch slot already in phase 2's shared-memory layout, with G and beta.
 *   phase 2 (gdn_chain_kernel), one CTA per (32-row slice of dv, head, sequence), sequential over the
 *     sequence's chunks, warp-specialised:
 *       4 producer warps prepare chunk c+1 while the chain runs chunk c: each chunk's inputs arrive in
 *       five copies two chunks ahead (T, W, G|beta by bulk copy; k rows and the slice's v columns by TMA
 *       boxes); they form K~ = k * exp(G_L - G) (f16) and U~ = T (beta v) for the slice;
 *       4 chain warps (2 dv row halves x 2 dk halves) hold the state slice in registers and run
 *       V' = U~ - W S^T,  S <- gamma_L S + V'^T K~ on f16 mma.sync with f32 accumulation.
 *     The roles hand chunks over through mbarriers (bounded waits, taken by one thread a role and
 *     broadcast through the role's named barrier, so a role always leaves its loop as a whole).
 * f16 operands with f32 accumulation keep the state within 4e-4 relative L2 of the f64 sequential
 * rule in the configurations this library is tested on (bf16 operands would not: ~3e-3).
 */
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"
#include "mma.cuh"
#include "sm100.cuh"

namespace {

constexpr int C = 64;          /* rows a chunk */
constexpr int D = 128;         /* head dims (dk = dv) */
constexpr int KP = D + 8;      /* pitch of 128-wide b16 rows in shared memory (conflict-free ldmatrix) */
constexpr int TP = C + 8;      /* pitch of 64-wide b16 rows */
constexpr int VS = 32;         /* dv rows per phase-2 CTA */
constexpr int VP = VS + 8;     /* pitch of 32-wide b16 rows */
constexpr int AP = C + 4;      /* pitch of the f32 A matrix */
constexpr int UP = VS + 4;     /* pitch of the f32 U~ slice */
constexpr int PP = C + 4;      /* pitch of the f32 exchange tiles */

/* A chunk's scratch slot, per (chunk, v-head), in phase 2's shared-memory layout: T f16 [64][TP],
 * W f16 [64][KP], then G f32 [64] and beta f32 [64]. */
constexpr int kSlotT = 0, kSlotW = C * TP * 2, kSlotMeta = kSlotW + C * KP * 2;
constexpr int kSlotBytes = kSlotMeta + 2 * C * 4;
constexpr uint32_t kKBoxBytes = C * D * 2, kVBoxBytes = C * VS * 2;

enum { kBarProducers = 1, kBarChain = 2, kBarPair0 = 3 };   /* named barriers (0 is __syncthreads) */

struct GdnPlan {
    RidgeFillGdn g;
    uint8_t* scratch;
    int max_slots;
};

__device__ __forceinline__ uint8_t* slot_ptr(const GdnPlan& p, int64_t slot, int64_t h) {
    return p.scratch + (slot * p.g.n_head_v + h) * (int64_t)kSlotBytes;
}

__device__ __forceinline__ void bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

/* cp.async of 4 bytes (src_bytes 0: zero fill). */
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(rf::saddr(dst)), "l"(src), "r"(src_bytes) : "memory");
}

/* Sequence i's rows [*r0, *r1): cu_seqlens read on the device and clamped into [0, T] (a value the host
 * cannot check never sends a load outside the operands). */
__device__ __forceinline__ void seq_rows(const RidgeFillGdn& g, int64_t i, int64_t* r0, int64_t* r1) {
    const int64_t a = min(max((int64_t)g.cu[i], (int64_t)0), g.T);
    const int64_t b = min(max((int64_t)g.cu[i + 1], a), g.T);
    *r0 = a;
    *r1 = b;
}

/* The sequence holding chunk `slot` (chunks of each sequence numbered consecutively, sequence by
 * sequence), its chunk's first row and length; false past the last chunk. */
__device__ bool locate_chunk(const RidgeFillGdn& g, int64_t slot, int64_t* row0, int* len) {
    int64_t base = 0;
    for (int64_t i = 0; i < g.n_seq; ++i) {
        int64_t r0, r1;
        seq_rows(g, i, &r0, &r1);
        const int64_t chunks = (r1 - r0 + C - 1) / C;
        if (slot < base + chunks) {
            const int64_t c = slot - base;
            *row0 = r0 + c * C;
            *len = (int)min((int64_t)C, r1 - r0 - c * C);
            return true;
        }
        base += chunks;
    }
    return false;
}

__device__ int64_t total_chunks(const GdnPlan& p) {
    int64_t n = 0, r0, r1;
    for (int64_t i = 0; i < p.g.n_seq; ++i) {
        seq_rows(p.g, i, &r0, &r1);
        n += (r1 - r0 + C - 1) / C;
    }
    return min(n, (int64_t)p.max_slots);
}

/* ------------------------------------------------------------------ phase 1 */

constexpr int kPrepThreads = 256;

struct PrepSmem {
    uint16_t kraw[2][2][C][C];   /* k rows of the current and the next item: two 128-byte-swizzled halves */
    float graw[2][C], braw[2][C];
    float a32[C][AP];            /* A, f32 */
    uint16_t l16[C][TP];         /* A, f16 (the off-diagonal blocks of I + A) */
    uint16_t t16[C][TP];         /* T = (I + A)^-1, f16 */
    uint16_t x1[C][KP];          /* beta gamma k, f16 */
    uint16_t w16[C][KP];         /* W = T x1, f16 */
    uint16_t tmp[3][16][24];     /* per-warp 16x16 staging */
    float G[C], beta[C];
    uint64_t landed[2];          /* the k rows of buffer b have landed */
    int abort, ok;
};

/* T[bi][bj] = -T[bi][bi] * sum_{k=bj}^{bi-1} L[bi][k] T[k][bj] for one 16x16 block, one warp. */
__device__ void tri_offdiag_block(PrepSmem& s, int bi, int bj, int w) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    float acc[2][4] = {};
    for (int k = bj; k < bi; ++k) {
        uint32_t a[4], b[4];
        rf::load_a(a, &s.l16[0][0], TP, 16 * bi, 16 * k);
        rf::load_b_kn(b, &s.t16[0][0], TP, 16 * k, 16 * bj);
        rf::mma_f16(acc[0], a, b[0], b[1]);
        rf::mma_f16(acc[1], a, b[2], b[3]);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
        *(uint32_t*)&s.tmp[w][g][8 * nt + 2 * t] = rf::pack_f16(acc[nt][0], acc[nt][1]);
        *(uint32_t*)&s.tmp[w][g + 8][8 * nt + 2 * t] = rf::pack_f16(acc[nt][2], acc[nt][3]);
    }
    __syncwarp();
    float out[2][4] = {};
    uint32_t a[4], b[4];
    rf::load_a(a, &s.t16[0][0], TP, 16 * bi, 16 * bi);
    rf::load_b_kn(b, &s.tmp[w][0][0], 24, 0, 0);
    rf::mma_f16(out[0], a, b[0], b[1]);
    rf::mma_f16(out[1], a, b[2], b[3]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
        *(uint32_t*)&s.t16[16 * bi + g][16 * bj + 8 * nt + 2 * t] = rf::pack_f16(-out[nt][0], -out[nt][1]);
        *(uint32_t*)&s.t16[16 * bi + g + 8][16 * bj + 8 * nt + 2 * t] = rf::pack_f16(-out[nt][2], -out[nt][3]);
    }
}

/* Item i = (chunk slot i / Hv, v-head i % Hv): start its k rows (two TMA boxes of [64 rows][64], rows
 * past the end of k read as zero) completing on landed[buf], and g, beta (cp.async; zero past the chunk). */
__device__ void prep_issue(const GdnPlan& p, const CUtensorMap* kmap, PrepSmem& s, int64_t item, int buf) {
    const RidgeFillGdn& g = p.g;
    const int64_t slot = item / g.n_head_v, h = item % g.n_head_v, hk = h / (g.n_head_v / g.n_head_k);
    int64_t row0 = 0;
    int len = 0;
    locate_chunk(g, slot, &row0, &len);
    if (threadIdx.x == 0) {
        rf::mbar_arrive_expect_tx(&s.landed[buf], kKBoxBytes);
        rf::tma_load_3d(&s.kraw[buf][0][0][0], kmap, &s.landed[buf], 0, (int)hk, (int)row0);
        rf::tma_load_3d(&s.kraw[buf][1][0][0], kmap, &s.landed[buf], C, (int)hk, (int)row0);
    }
    if (threadIdx.x < C) {
        const int r = threadIdx.x;
        const int64_t row = row0 + (r < len ? r : 0);
        cp_async4(&s.graw[buf][r], g.g + row * g.g_row + h, r < len ? 4 : 0);
        cp_async4(&s.braw[buf][r], g.beta + row * g.b_row + h, r < len ? 4 : 0);
    }
}

__global__ void __launch_bounds__(kPrepThreads, 2) gdn_prep_kernel(const __grid_constant__ CUtensorMap kmap, const GdnPlan p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    PrepSmem& s = *(PrepSmem*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const RidgeFillGdn& g = p.g;
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31, gq = l >> 2, tq = l & 3;
    const int64_t items = total_chunks(p) * g.n_head_v;
    if (tid == 0) {
        rf::mbar_init(&s.landed[0], 1);
        rf::mbar_init(&s.landed[1], 1);
        s.abort = 0;
        rf::mbar_init_fence();
        rf::tma_prefetch_map(&kmap);
    }
    __syncthreads();

    if ((int64_t)blockIdx.x < items) prep_issue(p, &kmap, s, blockIdx.x, 0);
    rf::cp_async_commit();
    int buf = 0;
    int64_t waited = 0, issued = (int64_t)blockIdx.x < items ? 1 : 0;
    for (int64_t item = blockIdx.x; item < items; item += gridDim.x, buf ^= 1) {
        if (item + gridDim.x < items) {
            prep_issue(p, &kmap, s, item + gridDim.x, buf ^ 1);
            ++issued;
        }
        rf::cp_async_commit();
        rf::cp_async_wait<1>();
        if (tid == 0) s.ok = rf::mbar_wait(&s.landed[buf], (uint32_t)((waited >> 1) & 1), &s.abort, rf::kErrGdnWait);
        __syncthreads();
        if (!s.ok) break;
        ++waited;
        const int64_t slot = item / g.n_head_v, h = item % g.n_head_v;
        int64_t row0 = 0;
        int len = 0;
        locate_chunk(g, slot, &row0, &len);
        const uint32_t ktile = rf::saddr(&s.kraw[buf][0][0][0]);

        /* G (inclusive cumulative log decay; zero past the chunk) and beta. */
        if (tid < C) {
            float x = s.graw[buf][tid];
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, x, o);
                if (l >= o) x += y;
            }
            s.G[tid] = x;
            s.beta[tid] = s.braw[buf][tid];
        }
        __syncthreads();
        if (tid >= 32 && tid < C) s.G[tid] += s.G[31];
        __syncthreads();

        /* x1 = beta gamma k in f16 (rows past the chunk: beta 0); K K^T (warp w: rows 16 (w & 3),
         * columns 32 (w >> 2)..+32) and A. */
        for (int i = tid; i < C * (D / 8); i += kPrepThreads) {
            const int r = i >> 4, seg = i & 15;
            uint4 raw;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(raw.x), "=r"(raw.y), "=r"(raw.z), "=r"(raw.w)
                         : "r"(rf::sw128_addr(ktile, r, seg * 8)));
            const uint32_t rw[4] = { raw.x, raw.y, raw.z, raw.w };
            const float f = r < len ? s.beta[r] * __expf(s.G[r]) : 0.0f;
            uint32_t xx[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                xx[e] = r < len ? rf::pack_f16(f * __uint_as_float(rw[e] << 16), f * __uint_as_float(rw[e] & 0xffff0000u)) : 0u;
            *(uint4*)&s.x1[r][seg * 8] = make_uint4(xx[0], xx[1], xx[2], xx[3]);
        }
        {
            const int rb = 16 * (w & 3), cb = 32 * (w >> 2);
            float acc[4][4] = {};
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
                uint32_t a[4];
                rf::load_a_sw(a, ktile, rb, 16 * ks);
#pragma unroll
                for (int pr = 0; pr < 2; ++pr) {
                    uint32_t b[4];
                    rf::load_b_nk_sw(b, ktile, cb + 16 * pr, 16 * ks);
                    rf::mma_bf16(acc[2 * pr], a, b[0], b[1]);
                    rf::mma_bf16(acc[2 * pr + 1], a, b[2], b[3]);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int i = rb + gq + (e >> 1) * 8, j = cb + 8 * nt + 2 * tq + (e & 1);
                    const float v = (j < i && i < len) ? s.beta[i] * __expf(s.G[i] - s.G[j]) * acc[nt][e] : 0.0f;
                    s.a32[i][j] = v;
                    s.l16[i][j] = __half_as_ushort(__float2half_rn(v));
                }
        }
        __syncthreads();

        /* Diagonal blocks: column c of block b by forward substitution in f32; upper blocks zero. */
        if (tid < C) {
            const int b = tid >> 4, c = tid & 15;
            float col[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                float x = r == c ? 1.0f : 0.0f;
#pragma unroll
                for (int j = 0; j < r; ++j) x -= s.a32[16 * b + r][16 * b + j] * col[j];
                col[r] = x;
                s.t16[16 * b + r][16 * b + c] = __half_as_ushort(__float2half_rn(x));
            }
        } else {
            for (int i = tid - C; i < C * C; i += kPrepThreads - C) {
                const int r = i >> 6, c = i & 63;
                if ((c >> 4) > (r >> 4)) s.t16[r][c] = 0;
            }
        }
        __syncthreads();
        if (w < 3) tri_offdiag_block(s, w + 1, w, w);            /* T10, T21, T32 */
        __syncthreads();
        if (w < 2) tri_offdiag_block(s, w + 2, w, w);            /* T20, T31 */
        __syncthreads();
        if (w == 0) tri_offdiag_block(s, 3, 0, 0);               /* T30 */
        __syncthreads();

        /* W = T x1 (warp w: rows 16 (w & 3), columns 64 (w >> 2)..+64). */
        {
            const int rb = 16 * (w & 3), cb = 64 * (w >> 2);
            uint32_t ta[4][4];
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) rf::load_a(ta[ks], &s.t16[0][0], TP, rb, 16 * ks);
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                float acc[2][4] = {};
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    uint32_t b[4];
                    rf::load_b_kn(b, &s.x1[0][0], KP, 16 * ks, cb + 16 * pr);
                    rf::mma_f16(acc[0], ta[ks], b[0], b[1]);
                    rf::mma_f16(acc[1], ta[ks], b[2], b[3]);
                }
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    *(uint32_t*)&s.w16[rb + gq][cb + 16 * pr + 8 * nt + 2 * tq] = rf::pack_f16(acc[nt][0], acc[nt][1]);
                    *(uint32_t*)&s.w16[rb + gq + 8][cb + 16 * pr + 8 * nt + 2 * tq] = rf::pack_f16(acc[nt][2], acc[nt][3]);
                }
            }
        }
        __syncthreads();

        /* The slot, in phase 2's layout: T and W byte for byte as they sit here, then G and beta. */
        uint8_t* out = slot_ptr(p, slot, h);
        for (int i = tid; i < (int)(sizeof(s.t16) / 16); i += kPrepThreads)
            *(uint4*)(out + kSlotT + i * 16) = *((const uint4*)&s.t16[0][0] + i);
        for (int i = tid; i < (int)(sizeof(s.w16) / 16); i += kPrepThreads)
            *(uint4*)(out + kSlotW + i * 16) = *((const uint4*)&s.w16[0][0] + i);
        float* meta = (float*)(out + kSlotMeta);
        if (tid < C) meta[tid] = s.G[tid];
        else if (tid < 2 * C) meta[tid] = s.beta[tid - C];
        __syncthreads();   /* this item's buffers are read before the next item's loads land in them */
    }
    rf::cp_async_wait<0>();
    /* After a timed-out wait: let the copies already issued land before the CTA's shared memory is
     * released (bounded too). */
    if (tid == 0)
        for (int64_t i = waited; i < issued; ++i) {
            const uint64_t t0 = rf::global_ns();
            while (!rf::mbar_try_wait(&s.landed[i & 1], (uint32_t)((i >> 1) & 1)) && rf::global_ns() - t0 < rf::kWaitTimeoutNs) {
            }
        }
}

/* ------------------------------------------------------------------ phase 2 */

constexpr int kChainThreads = 256;   /* warps 0-3: the chain; warps 4-7: producers */

struct RawStage {
    uint16_t t16[C][TP];      /* T, f16 (bulk copy of the slot) */
    float meta[2 * C];        /* G, beta */
    uint16_t kraw[C][D];      /* k rows, bf16 (TMA box; rows past the chunk are the next rows or zero) */
    uint16_t vraw[C][VS];     /* this CTA's 32 columns of v, bf16 (TMA box) */
};

struct ChainSmem {
    RawStage raw[2];             /* producers' inputs, two chunks in flight */
    uint16_t w16[3][C][KP];      /* W of chunks c, c+1, c+2 (the chain reads W of c) */
    uint16_t kt16[2][C][KP];     /* K~ = k * exp(G_L - G), f16, per chunk */
    float u32[2][C][UP];         /* U~ = T (beta v) for the slice, f32, per chunk */
    uint16_t x2[C][VP];          /* beta v, f16 (producers only) */
    float part[2][4][16][PP];    /* the chain warps' partial V'^T, double-buffered */
    float gl[2];                 /* gamma_L per chunk */
    uint64_t landed[2];          /* raw stage b (and its W stage) has landed */
    uint64_t ready[2], consumed[2];
    int abort, ok_producers, ok_chain;
};

/* Start chunk `slot`'s inputs into raw stage `rbuf` and W stage `wbuf`: T, W and G|beta by one bulk copy
 * each from its scratch slot, the k rows and this CTA's v columns by one TMA box each; all complete on
 * landed[rbuf]. One producer thread. */
__device__ void chain_issue(const GdnPlan& p, const CUtensorMap* kmap, const CUtensorMap* vmap, ChainSmem& s, int64_t slot,
                            int64_t row0, int64_t h, int64_t hk, int v0, int rbuf, int wbuf) {
    const uint8_t* src = slot_ptr(p, slot, h);
    RawStage& st = s.raw[rbuf];
    uint64_t* bar = &s.landed[rbuf];
    rf::mbar_arrive_expect_tx(bar, (uint32_t)(sizeof(st.t16) + sizeof(s.w16[0]) + sizeof(st.meta)) + kKBoxBytes + kVBoxBytes);
    rf::bulk_load(&st.t16[0][0], src + kSlotT, sizeof(st.t16), bar);
    rf::bulk_load(&s.w16[wbuf][0][0], src + kSlotW, sizeof(s.w16[0]), bar);
    rf::bulk_load(&st.meta[0], src + kSlotMeta, sizeof(st.meta), bar);
    rf::tma_load_3d(&st.kraw[0][0], kmap, bar, 0, (int)hk, (int)row0);
    rf::tma_load_3d(&st.vraw[0][0], vmap, bar, v0, (int)h, (int)row0);
}

__global__ void __launch_bounds__(kChainThreads, 1)
gdn_chain_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const GdnPlan p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    ChainSmem& s = *(ChainSmem*)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
    const RidgeFillGdn& g = p.g;
    const int vsl = blockIdx.x;
    const int64_t h = blockIdx.y, seq = blockIdx.z, hk = h / (g.n_head_v / g.n_head_k);
    const int64_t state_slot = g.state_idx[seq * g.idx_pitch];
    if (state_slot < 0 || state_slot >= g.n_states) return;
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31, gq = l >> 2, tq = l & 3;
    const int v0 = vsl * VS;

    /* This sequence's rows and first chunk slot. */
    int64_t base = 0, r0 = 0, r1 = 0;
    for (int64_t i = 0; i < seq; ++i) {
        seq_rows(g, i, &r0, &r1);
        base += (r1 - r0 + C - 1) / C;
    }
    seq_rows(g, seq, &r0, &r1);
    /* Overlapping sequences (cu not increasing) could number more chunks than phase 1 had slots for:
     * those chunks are not read. */
    const int64_t chunks = max((int64_t)0, min((r1 - r0 + C - 1) / C, (int64_t)p.max_slots - base));
    auto chunk_len = [&](int64_t c) { return (int)min((int64_t)C, r1 - r0 - c * C); };

    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            rf::mbar_init(&s.landed[b], 1);
            rf::mbar_init(&s.ready[b], 128);
            rf::mbar_init(&s.consumed[b], 128);
        }
        s.abort = 0;
        rf::mbar_init_fence();
        rf::tma_prefetch_map(&kmap);
        rf::tma_prefetch_map(&vmap);
    }
    __syncthreads();

    if (w >= 4) {
        /* ---------------------------------------------------------- producers */
        const int pt = tid - 128, pw = w - 4;
        int64_t issued = 0, landed = 0;
        if (pt == 0)
            for (; issued < 2 && issued < chunks; ++issued)
                chain_issue(p, &kmap, &vmap, s, base + issued, r0 + issued * C, h, hk, v0, (int)issued, (int)issued);
        for (int64_t c = 0; c < chunks; ++c) {
            const int b = (int)(c & 1);
            const int len = chunk_len(c);
            if (pt == 0) {   /* chunk c's inputs have landed, and chunk c-2 is consumed (its K~, U~ buffers are free) */
                s.ok_producers = rf::mbar_wait(&s.landed[b], (uint32_t)((c >> 1) & 1), &s.abort, rf::kErrGdnWait) &&
                                 (c < 2 || rf::mbar_wait(&s.consumed[b], (uint32_t)(((c - 2) >> 1) & 1), &s.abort, rf::kErrGdnWait));
                s.gl[b] = __expf(s.raw[b].meta[len - 1]);
            }
            bar_sync(kBarProducers, 128);
            if (!s.ok_producers) break;
            landed = c + 1;
            RawStage& st = s.raw[b];
            const float* G = st.meta;
            const float* beta = st.meta + C;
            const float gl = G[len - 1];
            for (int i = pt; i < C * (D / 8); i += 128) {   /* K~ = k * exp(G_L - G); rows past the chunk 0 */
                const int r = i >> 4, seg = i & 15;
                const uint4 raw = *(const uint4*)&st.kraw[r][seg * 8];
                const uint32_t rw[4] = { raw.x, raw.y, raw.z, raw.w };
                const float f = r < len ? __expf(gl - G[r]) : 0.0f;
                uint32_t kk[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    kk[e] = r < len ? rf::pack_f16(f * __uint_as_float(rw[e] << 16), f * __uint_as_float(rw[e] & 0xffff0000u)) : 0u;
                *(uint4*)&s.kt16[b][r][seg * 8] = make_uint4(kk[0], kk[1], kk[2], kk[3]);
            }
            for (int i = pt; i < C * (VS / 8); i += 128) {  /* x2 = beta v; rows past the chunk 0 */
                const int r = i >> 2, seg = i & 3;
                const uint4 raw = *(const uint4*)&st.vraw[r][seg * 8];
                const uint32_t rw[4] = { raw.x, raw.y, raw.z, raw.w };
                uint32_t xx[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    xx[e] = r < len ? rf::pack_f16(beta[r] * __uint_as_float(rw[e] << 16), beta[r] * __uint_as_float(rw[e] & 0xffff0000u)) : 0u;
                *(uint4*)&s.x2[r][seg * 8] = make_uint4(xx[0], xx[1], xx[2], xx[3]);
            }
            bar_sync(kBarProducers, 128);
            {   /* U~ = T x2: producer warp pw, rows 16 pw..+16, the slice's 32 columns */
                uint32_t ta[4][4];
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) rf::load_a(ta[ks], &st.t16[0][0], TP, 16 * pw, 16 * ks);
#pragma unroll
                for (int pr = 0; pr < 2; ++pr) {
                    float acc[2][4] = {};
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        uint32_t bb[4];
                        rf::load_b_kn(bb, &s.x2[0][0], VP, 16 * ks, 16 * pr);
                        rf::mma_f16(acc[0], ta[ks], bb[0], bb[1]);
                        rf::mma_f16(acc[1], ta[ks], bb[2], bb[3]);
                    }
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        *(float2*)&s.u32[b][16 * pw + gq][16 * pr + 8 * nt + 2 * tq] = make_float2(acc[nt][0], acc[nt][1]);
                        *(float2*)&s.u32[b][16 * pw + gq + 8][16 * pr + 8 * nt + 2 * tq] = make_float2(acc[nt][2], acc[nt][3]);
                    }
                }
            }
            rf::mbar_arrive(&s.ready[b]);   /* chunk c's K~, U~, gamma_L and W (landed above) are the chain's */
            if (pt == 0)   /* chunk c-1 is consumed: W stage (c+2) % 3 is free */
                s.ok_producers = c < 1 || rf::mbar_wait(&s.consumed[b ^ 1], (uint32_t)(((c - 1) >> 1) & 1), &s.abort, rf::kErrGdnWait);
            bar_sync(kBarProducers, 128);   /* also: every producer is done with raw stage b and x2 */
            if (!s.ok_producers) break;
            if (pt == 0 && c + 2 < chunks) {
                chain_issue(p, &kmap, &vmap, s, base + c + 2, r0 + (c + 2) * C, h, hk, v0, b, (int)((c + 2) % 3));
                ++issued;
            }
        }
        /* After a timed-out hand-over: let the copies already issued land before the CTA's shared memory
         * is released (bounded too). */
        if (pt == 0)
            for (int64_t i = landed; i < issued; ++i) {
                const uint64_t t0 = rf::global_ns();
                while (!rf::mbar_try_wait(&s.landed[i & 1], (uint32_t)((i >> 1) & 1)) && rf::global_ns() - t0 < rf::kWaitTimeoutNs) {
                }
            }
        return;
    }

    /* -------------------------------------------------------------- the chain */
    const int vh = w & 1, kh = w >> 1;
    /* The state slice: S[v0 + 16 vh + m][64 kh + n] as C tiles over dk (8 tiles of 8 columns). */
    float S[8][4];
    float* st = g.state + state_slot * g.st_slot + h * g.st_head;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int v = v0 + 16 * vh + gq + 8 * hr, k = 64 * kh + 8 * j + 2 * tq;
            const float2 x = *(const float2*)(st + (int64_t)v * D + k);
            S[j][2 * hr] = x.x;
            S[j][2 * hr + 1] = x.y;
        }
    bool ok = true;
    for (int64_t c = 0; c < chunks; ++c) {
        const int b = (int)(c & 1);
        if (tid == 0) s.ok_chain = rf::mbar_wait(&s.ready[b], (uint32_t)((c >> 1) & 1), &s.abort, rf::kErrGdnWait);
        bar_sync(kBarChain, 128);
        if (!(ok = s.ok_chain)) break;
        const uint16_t* W = &s.w16[c % 3][0][0];

        /* V'^T partial over this warp's dk half: [16 dv rows] x [64 chunk rows]. */
        float pv[8][4] = {};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            uint32_t a[4];
            rf::c_to_a(a, S[2 * ks], S[2 * ks + 1]);
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                uint32_t bb[4];
                rf::load_b_nk(bb, W, KP, 16 * pr, 64 * kh + 16 * ks);
                rf::mma_f16(pv[2 * pr], a, bb[0], bb[1]);
                rf::mma_f16(pv[2 * pr + 1], a, bb[2], bb[3]);
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            *(float2*)&s.part[b][w][gq][8 * j + 2 * tq] = make_float2(pv[j][0], pv[j][1]);
            *(float2*)&s.part[b][w][gq + 8][8 * j + 2 * tq] = make_float2(pv[j][2], pv[j][3]);
        }
        bar_sync(kBarPair0 + vh, 64);
        const float gamma_l = s.gl[b];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int m = gq + (e >> 1) * 8, n = 8 * j + 2 * tq + (e & 1);
                pv[j][e] = s.u32[b][n][16 * vh + m] - (pv[j][e] + s.part[b][w ^ 2][m][n]);
            }

        /* S <- gamma_L S + V'^T K~ over this warp's dk half. */
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) S[j][e] *= gamma_l;
        const uint16_t* Kt = &s.kt16[b][0][0];
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            uint32_t a[4];
            rf::c_to_a(a, pv[2 * ks], pv[2 * ks + 1]);
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                uint32_t bb[4];
                rf::load_b_kn(bb, Kt, KP, 16 * ks, 64 * kh + 16 * pr);
                rf::mma_f16(S[2 * pr], a, bb[0], bb[1]);
                rf::mma_f16(S[2 * pr + 1], a, bb[2], bb[3]);
            }
        }
        rf::mbar_arrive(&s.consumed[b]);
    }
    if (!ok) return;   /* a hand-over timed out (recorded in ridgefill_device_error): leave the state as it was */
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int v = v0 + 16 * vh + gq + 8 * hr, k = 64 * kh + 8 * j + 2 * tq;
            *(float2*)(st + (int64_t)v * D + k) = make_float2(S[j][2 * hr], S[j][2 * hr + 1]);
        }
}

int64_t max_slots_of(const RidgeFillGdn& g) { return (g.T + C - 1) / C + g.n_seq; }

/* A [T, heads, 128] bf16 operand (element strides row, head; 1 within a head) as a 3-D tensor map read in
 * boxes of [64 rows][1 head][box_cols], swizzled or dense; rows past T read as zero. */
bool head_rows_map(CUtensorMap* map, const void* base, int64_t T, int64_t heads, int64_t row_stride, int64_t head_stride,
                   uint32_t box_cols, bool swizzle) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = rf::tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[3] = { (cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)T };
    const cuuint64_t strides[2] = { (cuuint64_t)head_stride * 2, (cuuint64_t)row_stride * 2 };
    const cuuint32_t box[3] = { box_cols, 1, (cuuint32_t)C };
    const cuuint32_t estr[3] = { 1, 1, 1 };
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int64_t ridgefill_gdn_fill_scratch(const RadArgs* a) {
    RidgeFillGdn g;
    if (ridgefill_gdn_parse(a, &g) != RAD_OK) return 0;
    return max_slots_of(g) * g.n_head_v * (int64_t)kSlotBytes;
}

extern "C" int ridgefill_gdn_fill_device(const RadArgs* a, RadStream s) {
    RidgeFillGdn g;
    const int rc = ridgefill_gdn_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.o) return RAD_E_UNSUPPORTED;   /* the output form (o) is not served by this row yet */
    if (g.n_seq == 0 || g.T == 0) return RAD_OK;
    if (g.n_seq > 65535 || g.n_head_v > 65535 || g.T > 0x7fffffffLL) return RAD_E_SHAPE;
    const int64_t slots = max_slots_of(g);
    const int64_t need = slots * g.n_head_v * (int64_t)kSlotBytes;
    if (!a->scratch || a->scratch_bytes < need || (uintptr_t)a->scratch % 16) return RAD_E_INVAL;
    if (slots > 0x7fffffffLL) return RAD_E_SHAPE;
    /* k and v are read through TMA tensor maps: positive strides below 2^39 elements. */
    const int64_t lim = 1LL << 39;
    if (g.k_row <= 0 || g.k_head <= 0 || g.v_row <= 0 || g.v_head <= 0 || g.k_row >= lim || g.k_head >= lim ||
        g.v_row >= lim || g.v_head >= lim)
        return RAD_E_STRIDE;
    CUtensorMap kmap_sw, kmap, vmap;
    if (!head_rows_map(&kmap_sw, g.k, g.T, g.n_head_k, g.k_row, g.k_head, C, true) ||
        !head_rows_map(&kmap, g.k, g.T, g.n_head_k, g.k_row, g.k_head, D, false) ||
        !head_rows_map(&vmap, g.v, g.T, g.n_head_v, g.v_row, g.v_head, VS, false))
        return RAD_E_DEVICE;
    GdnPlan p;
    p.g = g;
    p.scratch = (uint8_t*)a->scratch;
    p.max_slots = (int)slots;
    cudaStream_t stream = rf::as_stream(s);
    const int smem1 = (int)sizeof(PrepSmem) + 1024, smem2 = (int)sizeof(ChainSmem) + 128;
    if (cudaFuncSetAttribute(gdn_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1) != cudaSuccess ||
        cudaFuncSetAttribute(gdn_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2) != cudaSuccess)
        return RAD_E_DEVICE;
    const int64_t items = slots * g.n_head_v;
    const int64_t grid1 = items < 2LL * rf::sm_count() ? items : 2LL * rf::sm_count();
    gdn_prep_kernel<<<(unsigned)grid1, kPrepThreads, smem1, stream>>>(kmap_sw, p);
    if (cudaGetLastError() != cudaSuccess) return RAD_E_DEVICE;
    gdn_chain_kernel<<<dim3(D / VS, (unsigned)g.n_head_v, (unsigned)g.n_seq), kChainThreads, smem2, stream>>>(kmap, vmap, p);
    return rf::launch_status();
}

/* This translation unit's copy of the device error word (sm100.cuh), for ridgefill_device_error. */
namespace rf {
int gdn_device_error(int reset) { return read_device_error(reset); }
}

/* ================================================================== the allocation-free entry point
 *
 * ridgefill_gdn_fill_noalloc: the DeltaNet fill for callers that cannot hand it a workspace. Some callers
 * of this library have no way to allocate device memory at the point they launch the fill: a host that
 * binds the C ABI through an FFI (ctypes, cgo, JNI) and receives its device buffers from elsewhere but
 * has no device allocator of its own, and an engine step whose device memory is fixed before the pass
 * starts, where a cudaMalloc inside the pass is not allowed (it can synchronise the device and stall
 * every stream of the step). This entry point takes the same operands as the ridgefill_gdn_fill row,
 * ignores RadArgs::scratch, and uses instead a workspace compiled into the library: a file-scope device
 * array of kNoAllocScratchBytes (48 MiB), which every GPU that loads the library holds until the
 * process exits. 48 MiB holds the fill's workspace (26.5 KiB per 64-row chunk and value head, one chunk
 * more per sequence) for a one-sequence 2,048-row call -- the engine's default chunk -- at up to 56 value
 * heads, or a 4,096-row call at up to 28; a call that needs more returns RAD_E_SHAPE and launches nothing.
 *
 * The first call on each device resolves the array's device address there (cudaGetSymbolAddress, once
 * per device, with that device current); make that first call before any stream capture. No call
 * allocates or frees device memory. Every call shares the one array and the array keeps the last call's
 * contents: nothing in it needs to start at zero (each call writes every byte of the workspace it reads
 * before reading it, in stream order), but two calls that overlap on the GPU -- on different streams,
 * or from different threads, without an ordering between them -- race on it.
 */
namespace {
constexpr int64_t kNoAllocScratchBytes = 48ll << 20;
constexpr int kNoAllocMaxDevices = 64;
}   // namespace

static __device__ __align__(256) uint8_t g_gdn_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mutex;
void* g_noalloc_address[kNoAllocMaxDevices];

/* The array's device address on the current device; resolved on the first call there. */
int noalloc_workspace(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return RAD_E_DEVICE;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_address[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_gdn_noalloc_scratch) != cudaSuccess || !ptr) return RAD_E_DEVICE;
        g_noalloc_address[dev] = ptr;
    }
    *out = g_noalloc_address[dev];
    return RAD_OK;
}
}   // namespace

extern "C" int ridgefill_gdn_fill_noalloc(const RadArgs* a, RadStream s) {
    RidgeFillGdn g;
    const int rc = ridgefill_gdn_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (ridgefill_gdn_fill_scratch(a) > kNoAllocScratchBytes) return RAD_E_SHAPE;   /* past the built-in workspace */
    void* workspace = nullptr;
    const int ws = noalloc_workspace(&workspace);
    if (ws != RAD_OK) return ws;
    RadArgs with = *a;
    with.scratch = workspace;
    with.scratch_bytes = kNoAllocScratchBytes;
    return ridgefill_gdn_fill_device(&with, s);
}
