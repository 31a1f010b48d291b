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
 *   phase 1 (gdn_tri_kernel), every (chunk, head) in parallel: K K^T on tensor cores (bf16, exact
 *     inputs), A, and T by blocked inversion: 16x16 diagonal blocks by substitution in f32, the
 *     off-diagonal blocks by f16 tensor-core products. T (f16) and G, beta go to the row's scratch.
 *   phase 2 (gdn_chain_kernel), one CTA per (32-row slice of dv, head, sequence), sequential over the
 *     sequence's chunks: W = T (beta gamma K), U~ = T (beta v) and the carry
 *     V' = U~ - W S^T,  S <- gamma_L S + (V' * decay)^T K  on f16 tensor cores with f32 accumulation;
 *     the state slice stays in registers across chunks (4 warps: 2 row halves x 2 dk halves), the
 *     next chunk's inputs stream in with cp.async while the current one runs.
 * f16 operands with f32 accumulation keep the state within 4e-4 relative L2 of the f64 sequential
 * rule in the configurations this library is tested on (bf16 operands would not: ~3e-3).
 */
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"
#include "mma.cuh"

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
constexpr int kSlotBytes = C * C * 2 + 2 * C * 4;   /* T f16 [64][64], then G and beta f32 [64] each */

struct GdnPlan {
    RidgeFillGdn g;
    uint8_t* scratch;
    int max_slots;
};

__device__ __forceinline__ uint8_t* slot_ptr(const GdnPlan& p, int64_t slot, int64_t h) {
    return p.scratch + (slot * p.g.n_head_v + h) * (int64_t)kSlotBytes;
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

/* ------------------------------------------------------------------ phase 1 */

struct TriSmem {
    uint16_t ks[C][KP];       /* k rows, bf16 */
    float a32[C][AP];         /* A, f32 */
    uint16_t l16[C][TP];      /* A, f16 (the off-diagonal blocks of I + A) */
    uint16_t t16[C][TP];      /* T = (I + A)^-1, f16 */
    uint16_t tmp[3][16][24];  /* per-warp 16x16 staging */
    float G[C], beta[C];
};

/* T[bi][bj] = -T[bi][bi] * sum_{k=bj}^{bi-1} L[bi][k] T[k][bj] for one 16x16 block, one warp. */
__device__ void tri_offdiag_block(TriSmem& s, int bi, int bj, int w) {
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

__global__ void __launch_bounds__(128) gdn_tri_kernel(const GdnPlan p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    TriSmem& s = *(TriSmem*)smem_raw;
    const RidgeFillGdn& g = p.g;
    const int64_t slot = blockIdx.x, h = blockIdx.y, hk = h / (g.n_head_v / g.n_head_k);
    int64_t row0 = 0;
    int len = 0;
    if (!locate_chunk(g, slot, &row0, &len)) return;
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31, gq = l >> 2, tq = l & 3;

    /* k rows (zero past the chunk), g and beta. */
    for (int i = tid; i < C * (D / 8); i += 128) {
        const int r = i >> 4, seg = i & 15;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < len) v = *(const uint4*)(g.k + (row0 + r) * g.k_row + hk * g.k_head + seg * 8);
        *(uint4*)&s.ks[r][seg * 8] = v;
    }
    if (tid < 64) {
        const float gv = tid < len ? g.g[(row0 + tid) * g.g_row + h] : 0.0f;
        s.beta[tid] = tid < len ? g.beta[(row0 + tid) * g.b_row + h] : 0.0f;
        float x = gv;   /* inclusive scan of the two 32-row halves */
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, x, o);
            if (l >= o) x += y;
        }
        s.G[tid] = x;
    }
    __syncthreads();
    if (tid >= 32 && tid < 64) s.G[tid] += s.G[31];
    __syncthreads();

    /* K K^T (bf16 inputs exact, f32 accumulate), then A. Warp w: rows 16w..16w+15. */
    {
        float acc[8][4] = {};
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
            uint32_t a[4];
            rf::load_a(a, &s.ks[0][0], KP, 16 * w, 16 * ks);
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                uint32_t b[4];
                rf::load_b_nk(b, &s.ks[0][0], KP, 16 * pr, 16 * ks);
                rf::mma_bf16(acc[2 * pr], a, b[0], b[1]);
                rf::mma_bf16(acc[2 * pr + 1], a, b[2], b[3]);
            }
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = 16 * w + gq + (e >> 1) * 8, j = 8 * nt + 2 * tq + (e & 1);
                const float v = (j < i && i < len) ? s.beta[i] * expf(s.G[i] - s.G[j]) * acc[nt][e] : 0.0f;
                s.a32[i][j] = v;
                s.l16[i][j] = __half_as_ushort(__float2half_rn(v));
            }
    }
    __syncthreads();

    /* Diagonal blocks: column c of block b by forward substitution in f32; upper blocks zero. */
    if (tid < 64) {
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
        for (int i = tid - 64; i < C * C; i += 64) {
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

    uint8_t* out = slot_ptr(p, slot, h);
    for (int i = tid; i < C * (C / 8); i += 128) {
        const int r = i >> 3, seg = i & 7;
        *(uint4*)(out + (r * C + seg * 8) * 2) = *(const uint4*)&s.t16[r][seg * 8];
    }
    float* meta = (float*)(out + C * C * 2);
    if (tid < 64) meta[tid] = s.G[tid];
    else meta[tid] = s.beta[tid - 64];
}

/* ------------------------------------------------------------------ phase 2 */

struct Stage {
    uint16_t t16[C][TP];      /* T, f16 */
    float meta[2 * C];        /* G, beta */
    uint16_t kraw[C][KP];     /* k rows, bf16 */
    uint16_t vraw[C][VP];     /* this CTA's 32 columns of v, bf16 */
};

struct ChainSmem {
    Stage st[2];
    uint16_t x1[C][KP];       /* beta gamma k, f16 */
    uint16_t k16[C][KP];      /* k, f16 */
    uint16_t w16[C][KP];      /* W = T x1, f16 */
    uint16_t x2[C][VP];       /* beta v, f16 */
    float u32[C][UP];         /* U~ = T x2, f32 */
    float part[4][16][PP];    /* per-warp partial V'^T */
    float gam[C], dec[C];
};

__device__ void issue_chunk_loads(const GdnPlan& p, ChainSmem& s, int buf, int64_t slot, int64_t row0, int len,
                                  int64_t h, int64_t hk, int v0) {
    const RidgeFillGdn& g = p.g;
    const uint8_t* src = slot_ptr(p, slot, h);
    Stage& st = s.st[buf];
    const int tid = threadIdx.x;
    for (int i = tid; i < C * (C / 8); i += 128) {   /* T: 64 rows x 8 segments */
        const int r = i >> 3, seg = i & 7;
        rf::cp_async16(&st.t16[r][seg * 8], src + (r * C + seg * 8) * 2, 16);
    }
    if (tid < 2 * C / 4) rf::cp_async16(&st.meta[tid * 4], src + C * C * 2 + tid * 16, 16);
    for (int i = tid; i < C * (D / 8); i += 128) {   /* k: 64 rows x 16 segments */
        const int r = i >> 4, seg = i & 15;
        const int64_t row = row0 + (r < len ? r : 0);
        rf::cp_async16(&st.kraw[r][seg * 8], g.k + row * g.k_row + hk * g.k_head + seg * 8, r < len ? 16 : 0);
    }
    for (int i = tid; i < C * (VS / 8); i += 128) {  /* v slice: 64 rows x 4 segments */
        const int r = i >> 2, seg = i & 3;
        const int64_t row = row0 + (r < len ? r : 0);
        rf::cp_async16(&st.vraw[r][seg * 8], g.v + row * g.v_row + h * g.v_head + v0 + seg * 8, r < len ? 16 : 0);
    }
}

__global__ void __launch_bounds__(128, 1) gdn_chain_kernel(const GdnPlan p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    ChainSmem& s = *(ChainSmem*)smem_raw;
    const RidgeFillGdn& g = p.g;
    const int vsl = blockIdx.x;
    const int64_t h = blockIdx.y, seq = blockIdx.z, hk = h / (g.n_head_v / g.n_head_k);
    const int64_t state_slot = g.state_idx[seq * g.idx_pitch];
    if (state_slot < 0 || state_slot >= g.n_states) return;
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31, gq = l >> 2, tq = l & 3;
    const int vh = w & 1, kh = w >> 1;
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

    if (chunks > 0) issue_chunk_loads(p, s, 0, base, r0, (int)min((int64_t)C, r1 - r0), h, hk, v0);
    rf::cp_async_commit();
    for (int64_t c = 0; c < chunks; ++c) {
        const int buf = (int)(c & 1);
        const int64_t row0 = r0 + c * C;
        const int len = (int)min((int64_t)C, r1 - row0);
        if (c + 1 < chunks)
            issue_chunk_loads(p, s, buf ^ 1, base + c + 1, row0 + C, (int)min((int64_t)C, r1 - row0 - C), h, hk, v0);
        rf::cp_async_commit();
        rf::cp_async_wait<1>();
        __syncthreads();
        Stage& sg = s.st[buf];
        const float* G = sg.meta;
        const float* beta = sg.meta + C;

        /* Operands of this chunk. */
        if (tid < C) {
            const float gl = G[len - 1];
            s.gam[tid] = expf(G[tid]);
            s.dec[tid] = tid < len ? expf(gl - G[tid]) : 0.0f;
        }
        __syncthreads();
        for (int i = tid; i < C * (D / 8); i += 128) {
            const int r = i >> 4, seg = i & 15;
            const uint4 raw = *(const uint4*)&sg.kraw[r][seg * 8];
            const uint16_t* kb = (const uint16_t*)&raw;
            const float f = beta[r] * s.gam[r];
            uint32_t kk[4], xx[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float k0 = rf::bf16_bits_to_f32(kb[2 * e]), k1 = rf::bf16_bits_to_f32(kb[2 * e + 1]);
                kk[e] = rf::pack_f16(k0, k1);
                xx[e] = rf::pack_f16(f * k0, f * k1);
            }
            *(uint4*)&s.k16[r][seg * 8] = make_uint4(kk[0], kk[1], kk[2], kk[3]);
            *(uint4*)&s.x1[r][seg * 8] = make_uint4(xx[0], xx[1], xx[2], xx[3]);
        }
        for (int i = tid; i < C * (VS / 8); i += 128) {
            const int r = i >> 2, seg = i & 3;
            const uint4 raw = *(const uint4*)&sg.vraw[r][seg * 8];
            const uint16_t* vb = (const uint16_t*)&raw;
            uint32_t xx[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                xx[e] = rf::pack_f16(beta[r] * rf::bf16_bits_to_f32(vb[2 * e]), beta[r] * rf::bf16_bits_to_f32(vb[2 * e + 1]));
            *(uint4*)&s.x2[r][seg * 8] = make_uint4(xx[0], xx[1], xx[2], xx[3]);
        }
        __syncthreads();

        /* W = T x1 (rows 16w..16w+15, all 128 columns) and U~ = T x2 (the 32-column slice). */
        {
            uint32_t ta[4][4];
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) rf::load_a(ta[ks], &sg.t16[0][0], TP, 16 * w, 16 * ks);
#pragma unroll
            for (int pr = 0; pr < 8; ++pr) {
                float acc[2][4] = {};
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    uint32_t b[4];
                    rf::load_b_kn(b, &s.x1[0][0], KP, 16 * ks, 16 * pr);
                    rf::mma_f16(acc[0], ta[ks], b[0], b[1]);
                    rf::mma_f16(acc[1], ta[ks], b[2], b[3]);
                }
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    *(uint32_t*)&s.w16[16 * w + gq][16 * pr + 8 * nt + 2 * tq] = rf::pack_f16(acc[nt][0], acc[nt][1]);
                    *(uint32_t*)&s.w16[16 * w + gq + 8][16 * pr + 8 * nt + 2 * tq] = rf::pack_f16(acc[nt][2], acc[nt][3]);
                }
            }
#pragma unroll
            for (int pr = 0; pr < 2; ++pr) {
                float acc[2][4] = {};
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    uint32_t b[4];
                    rf::load_b_kn(b, &s.x2[0][0], VP, 16 * ks, 16 * pr);
                    rf::mma_f16(acc[0], ta[ks], b[0], b[1]);
                    rf::mma_f16(acc[1], ta[ks], b[2], b[3]);
                }
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    *(float2*)&s.u32[16 * w + gq][16 * pr + 8 * nt + 2 * tq] = make_float2(acc[nt][0], acc[nt][1]);
                    *(float2*)&s.u32[16 * w + gq + 8][16 * pr + 8 * nt + 2 * tq] = make_float2(acc[nt][2], acc[nt][3]);
                }
            }
        }
        __syncthreads();

        /* V'^T partial over this warp's dk half: [16 dv rows] x [64 chunk rows]. */
        float pv[8][4] = {};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            uint32_t a[4];
            rf::c_to_a(a, S[2 * ks], S[2 * ks + 1]);
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                uint32_t b[4];
                rf::load_b_nk(b, &s.w16[0][0], KP, 16 * pr, 64 * kh + 16 * ks);
                rf::mma_f16(pv[2 * pr], a, b[0], b[1]);
                rf::mma_f16(pv[2 * pr + 1], a, b[2], b[3]);
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            *(float2*)&s.part[w][gq][8 * j + 2 * tq] = make_float2(pv[j][0], pv[j][1]);
            *(float2*)&s.part[w][gq + 8][8 * j + 2 * tq] = make_float2(pv[j][2], pv[j][3]);
        }
        __syncthreads();
        const int other = w ^ 2;
        const float gamma_l = s.gam[len - 1];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int m = gq + (e >> 1) * 8, n = 8 * j + 2 * tq + (e & 1);
                const float vn = s.u32[n][16 * vh + m] - (pv[j][e] + s.part[other][m][n]);
                pv[j][e] = vn * s.dec[n];   /* decayed corrected value, tokens past len decay to 0 */
            }

        /* S <- gamma_L S + (V' decay)^T K over this warp's dk half. */
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) S[j][e] *= gamma_l;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            uint32_t a[4];
            rf::c_to_a(a, pv[2 * ks], pv[2 * ks + 1]);
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                uint32_t b[4];
                rf::load_b_kn(b, &s.k16[0][0], KP, 16 * ks, 64 * kh + 16 * pr);
                rf::mma_f16(S[2 * pr], a, b[0], b[1]);
                rf::mma_f16(S[2 * pr + 1], a, b[2], b[3]);
            }
        }
        __syncthreads();   /* every buffer of this chunk is read before the next chunk overwrites it */
    }
    rf::cp_async_wait<0>();

#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int v = v0 + 16 * vh + gq + 8 * hr, k = 64 * kh + 8 * j + 2 * tq;
            *(float2*)(st + (int64_t)v * D + k) = make_float2(S[j][2 * hr], S[j][2 * hr + 1]);
        }
}

int64_t max_slots_of(const RidgeFillGdn& g) { return (g.T + C - 1) / C + g.n_seq; }

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
    if (g.n_seq == 0) return RAD_OK;
    if (g.n_seq > 65535 || g.n_head_v > 65535) return RAD_E_SHAPE;
    const int64_t slots = max_slots_of(g);
    const int64_t need = slots * g.n_head_v * (int64_t)kSlotBytes;
    if (!a->scratch || a->scratch_bytes < need || (uintptr_t)a->scratch % 16) return RAD_E_INVAL;
    if (slots > 0x7fffffffLL) return RAD_E_SHAPE;
    GdnPlan p;
    p.g = g;
    p.scratch = (uint8_t*)a->scratch;
    p.max_slots = (int)slots;
    cudaStream_t stream = rf::as_stream(s);
    if (cudaFuncSetAttribute(gdn_tri_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(TriSmem)) != cudaSuccess ||
        cudaFuncSetAttribute(gdn_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(ChainSmem)) != cudaSuccess)
        return RAD_E_DEVICE;
    gdn_tri_kernel<<<dim3((unsigned)slots, (unsigned)g.n_head_v), 128, sizeof(TriSmem), stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return RAD_E_DEVICE;
    gdn_chain_kernel<<<dim3(D / VS, (unsigned)g.n_head_v, (unsigned)g.n_seq), 128, sizeof(ChainSmem), stream>>>(p);
    return rf::launch_status();
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
 * array of kNoAllocScratchBytes (32 MiB), which every GPU that loads the library holds until the
 * process exits. 32 MiB holds the fill's workspace for a 4,096-row call at 48 value heads (8.5 KiB per
 * 64-row chunk and head); a call that needs more returns RAD_E_SHAPE and launches nothing.
 *
 * The first call on each device resolves the array's device address there (cudaGetSymbolAddress, once
 * per device, with that device current); make that first call before any stream capture. No call
 * allocates or frees device memory. Every call shares the one array and the array keeps the last call's
 * contents: nothing in it needs to start at zero (each call writes every byte of the workspace it reads
 * before reading it, in stream order), but two calls that overlap on the GPU -- on different streams,
 * or from different threads, without an ordering between them -- race on it.
 */
namespace {
constexpr int64_t kNoAllocScratchBytes = 32ll << 20;
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
