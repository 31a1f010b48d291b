/* conv_prep.cu -- ridgefill_gdn_conv_prep: the Gated DeltaNet block's input preparation on B200, the step
 * between the block's input projections and the chunk fill (issue site arch/qwen4exp_fill.h:41-50,
 * arch/qwen4exp_blocks.h:118-134). The reference issues radiance's in-tree gdn_conv_prep, whose source is not
 * part of the checkout; the arithmetic here is the Gated DeltaNet block's published input path (causal
 * depthwise convolution of width 4, SiLU, per-head L2 normalisation of q and k) and the reference's own gate
 * g = -exp(A_log) softplus(a + dt_bias) (kernels/ridgefill.h:93-97), written per row for ridgefill_gdn_fill.
 *
 * HBM-bound: x is read once and q, k, v written once (2 x 2 C bytes a row). Without a q operand (the state-only
 * fill reads no q) the q columns are neither read nor computed; the conv state still takes every channel of each
 * sequence's last three rows, so x's q columns need be valid only there. A warp takes 16 rows of a pair of
 * 128-channel head columns, lane l channels 8 (l % 16)..+8 of column l / 16 (16-byte loads and stores, a
 * warp's row 512 contiguous bytes); the convolution's three earlier rows ride in registers; when the 16 rows
 * lie in one sequence, all their loads are in flight at once as asynchronous copies into the lane's own
 * shared-memory slots (64 KiB a CTA). A second kernel then writes each sequence's last three input rows into its
 * conv-state slot (it reads the old state first, thread by thread, so the update is in place).
 */
#include <cuda_bf16.h>

#include "common.cuh"
#include "sm100.cuh"

namespace {

constexpr int kRows = 16;        /* rows a warp task */
constexpr int kThreads = 256;
constexpr int kStageBytes = (kThreads / 32) * kRows * 512;   /* a warp's 16 rows of 512 bytes, for every warp */

/* 16-byte asynchronous copy global -> shared (through L2 only), in the current cp.async group. */
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
    const uint32_t w[4] = { v.x, v.y, v.z, v.w };
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        f[2 * e] = __uint_as_float(w[e] << 16);
        f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
    }
}

/* Two f32 as a bf16 pair, rounded to nearest even by the hardware conversion (one instruction for both). */
__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *(const uint32_t*)&p;
}

__device__ __forceinline__ int64_t seq_start(const RidgeFillConvPrep& g, int64_t i) {
    return min(max((int64_t)g.cu[i], (int64_t)0), g.T);
}

/* The sequence holding row r: the last i whose clamped start is <= r, if r lies before its clamped end;
 * -1 otherwise. cu is read where it lies; values outside [0, T] are clamped (the fill's rule). */
__device__ int find_seq(const RidgeFillConvPrep& g, int64_t r, int64_t* s0, int64_t* e0) {
    if (g.n_seq <= 0 || seq_start(g, 0) > r) return -1;
    int64_t lo = 0, hi = g.n_seq - 1;
    while (lo < hi) {
        const int64_t mid = (lo + hi + 1) >> 1;
        if (seq_start(g, mid) <= r) lo = mid;
        else hi = mid - 1;
    }
    const int64_t a = seq_start(g, lo), b = min(max((int64_t)g.cu[lo + 1], a), g.T);
    if (r >= b) return -1;
    *s0 = a;
    *e0 = b;
    return (int)lo;
}

/* Whether sequence `seq` continues a context held in its conv-state slot; the slot (or -1). */
__device__ __forceinline__ int64_t history_slot(const RidgeFillConvPrep& g, int64_t seq) {
    const int64_t slot = g.idx[seq * g.idx_pitch];
    const bool has = g.ctx != nullptr && g.ctx[seq] > 0 && slot >= 0 && slot < g.n_states;
    return has ? slot : -1;
}

/* Channels c..c+7 of input row `row` of the sequence starting at s0 (row >= s0 - 3): x, or the state's
 * history row (s0 - row rows back), or zero. */
__device__ __forceinline__ uint4 window_row(const RidgeFillConvPrep& g, int64_t slot, int64_t s0, int64_t row, int64_t c,
                                            int64_t C) {
    if (row >= s0) return *(const uint4*)(g.x + row * g.x_row + c);
    if (slot < 0) return make_uint4(0u, 0u, 0u, 0u);
    return *(const uint4*)(g.state + slot * g.st_slot + (3 - (s0 - row)) * C + c);
}

/* SiLU u / (1 + e^-u) with the fast exp and divide (well inside bf16's rounding), except where the fast divide
 * returns 0: a denominator above 2^126 (u below about -87.3, where the value is about u e^u, under 1e-36 in
 * magnitude) takes the exact division, so those rows keep their tiny values as the f32 rule gives them. */
__device__ __forceinline__ float silu(float u) {
    const float den = 1.0f + __expf(-u);
    return den < 0x1p126f ? __fdividef(u, den) : u / den;
}

/* A warp takes kRows rows of a pair of 128-channel head columns (2 j, 2 j + 1; the pair is q / k or v alike,
 * as 2 Hk is even): half-warp hw owns column 2 j + hw, lane l of the half channels 8 l..8 l + 7. */
__global__ void __launch_bounds__(kThreads) conv_prep_kernel(RidgeFillConvPrep g) {
    extern __shared__ uint4 rows_smem[];   /* [warp][kRows][lane] */
    const int lane = threadIdx.x & 31, hw = lane >> 4, hl = lane & 15;
    uint4* stage = rows_smem + (threadIdx.x >> 5) * kRows * 32 + lane;
    const int64_t hk = g.n_head_k, hv = g.n_head_v;
    const int64_t C = 2 * hk * 128 + hv * 128, n_hc = C / 128, n_pairs = (n_hc + 1) / 2;
    /* without a q output the q columns are not computed: the pairs start at the first that holds a k column */
    const int64_t first = g.q ? 0 : hk / 2, pairs = n_pairs - first;
    const int64_t tasks = (g.T + kRows - 1) / kRows * pairs;
    const int64_t stride = (int64_t)gridDim.x * (kThreads / 32);
    for (int64_t task = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); task < tasks; task += stride) {
        const int64_t pair = first + task % pairs, r0 = task / pairs * kRows, r1 = min(r0 + kRows, g.T);
        const int64_t hc = 2 * pair + hw;
        /* an odd column count leaves the last pair's second half idle; an odd hk without q, the first pair's first */
        const bool live = hc < n_hc && (g.q != nullptr || hc >= hk);
        const int64_t c = (live ? hc : 2 * pair) * 128 + 8 * hl;
        const bool norm = 2 * pair < 2 * hk;         /* q and k columns are L2-normalised; the pair is alike */
        float wt[8][4], bs[8];
        {
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {         /* channels c + 2 q4, c + 2 q4 + 1: 16 bytes of taps */
                const uint4 wv = *(const uint4*)(g.w + (c + 2 * q4) * 4);
                const uint32_t ww[4] = { wv.x, wv.y, wv.z, wv.w };
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t word = ww[2 * h + (j >> 1)];
                        wt[2 * q4 + h][j] = __uint_as_float((j & 1) ? (word & 0xffff0000u) : (word << 16));
                    }
            }
            if (g.bias) unpack8(*(const uint4*)(g.bias + c), bs);
            else {
#pragma unroll
                for (int e = 0; e < 8; ++e) bs[e] = 0.0f;
            }
        }
        const int kind = hc < hk ? 0 : (hc < 2 * hk ? 1 : 2);   /* q, k, v */
        const int64_t head = kind == 0 ? hc : (kind == 1 ? hc - hk : hc - 2 * hk);
        uint16_t* out = kind == 0 ? g.q + head * g.q_head : (kind == 1 ? g.k + head * g.k_head : g.v + head * g.v_head);
        const int64_t out_row = kind == 0 ? g.q_row : (kind == 1 ? g.k_row : g.v_row);
        const bool gate = live && kind == 2 && hl == 0;   /* the row-by-row path's gate lane */
        const float neg_a = live && kind == 2 ? -expf(g.a_log[head]) : 0.0f, dtb = live && kind == 2 ? g.dt_bias[head] : 0.0f;

        float w0[8], w1[8], w2[8];   /* rows r-3, r-2, r-1 */
        /* one row: the convolution over (w0, w1, w2, cur), SiLU, the head's L2 norm for q and k, bf16 out; the gate */
        auto gate_row = [&](int64_t r) {   /* g and beta of row r for this half's v-head */
            const float av = rf::bf16_bits_to_f32(g.a[r * g.a_row + head]);
            const float bv = rf::bf16_bits_to_f32(g.b[r * g.b_row + head]);
            g.g[r * g.g_row + head] = neg_a * ridgefill_softplus(av + dtb);
            g.beta[r * g.beta_row + head] = 1.0f / (1.0f + expf(-bv));
        };
        auto emit = [&](int64_t r, const float (&cur)[8], bool with_gate) {
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {   /* the taps two channels an instruction (packed f32x2, same roundings) */
                float u0 = bs[e], u1 = bs[e + 1];
                rf::fma2_rn(u0, u1, wt[e][0], wt[e + 1][0], w0[e], w0[e + 1]);
                rf::fma2_rn(u0, u1, wt[e][1], wt[e + 1][1], w1[e], w1[e + 1]);
                rf::fma2_rn(u0, u1, wt[e][2], wt[e + 1][2], w2[e], w2[e + 1]);
                rf::fma2_rn(u0, u1, wt[e][3], wt[e + 1][3], cur[e], cur[e + 1]);
                y[e] = silu(u0);
                y[e + 1] = silu(u1);
            }
            if (norm) {
                float ss = 0.0f;
#pragma unroll
                for (int e = 0; e < 8; ++e) ss = fmaf(y[e], y[e], ss);
                for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);   /* within the half */
                const float inv = rsqrtf(ss + 1e-6f);   /* within 2 ulp: well inside bf16's rounding */
#pragma unroll
                for (int e = 0; e < 8; e += 2) rf::mul2_rn(y[e], y[e + 1], y[e], y[e + 1], inv, inv);
            }
            if (live)
                *(uint4*)(out + r * out_row + 8 * hl) = make_uint4(bf16x2(y[0], y[1]), bf16x2(y[2], y[3]), bf16x2(y[4], y[5]),
                                                                   bf16x2(y[6], y[7]));
            if (with_gate && gate) gate_row(r);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                w0[e] = w1[e];
                w1[e] = w2[e];
                w2[e] = cur[e];
            }
        };
        auto prime = [&](int64_t seq, int64_t s0, int64_t r) {
            const int64_t slot = history_slot(g, seq);
            unpack8(window_row(g, slot, s0, r - 3, c, C), w0);
            unpack8(window_row(g, slot, s0, r - 2, c, C), w1);
            unpack8(window_row(g, slot, s0, r - 1, c, C), w2);
        };

        int64_t s0 = 0, e0 = 0;
        const int seq0 = find_seq(g, r0, &s0, &e0);
        if (seq0 >= 0 && e0 >= r1) {
            /* the task's rows lie in one sequence: all their loads in flight at once, as asynchronous copies into
             * this lane's own shared-memory slots (no register holds them meanwhile) */
            const int n = (int)(r1 - r0);
            const uint16_t* src = g.x + r0 * g.x_row + c;
            for (int i = 0; i < n; ++i) cp_async16(stage + i * 32, src + i * g.x_row);
            asm volatile("cp.async.commit_group;" ::: "memory");
            prime(seq0, s0, r0);
            if (live && kind == 2 && hl < n) gate_row(r0 + hl);   /* the task's gates, a row a lane, up front */
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            if (n == kRows) {   /* fully unrolled: the window's shifts become register renames */
#pragma unroll
                for (int i = 0; i < kRows; ++i) {
                    float cur[8];
                    unpack8(stage[i * 32], cur);
                    emit(r0 + i, cur, false);
                }
            } else {
                for (int i = 0; i < n; ++i) {
                    float cur[8];
                    unpack8(stage[i * 32], cur);
                    emit(r0 + i, cur, false);
                }
            }
        } else {
            /* sequence boundaries (or rows outside every sequence) inside the task: row by row */
            int seq = seq0;
            bool primed = false;
            for (int64_t r = r0; r < r1; ++r) {
                if (seq < 0 || r >= e0) {
                    seq = find_seq(g, r, &s0, &e0);
                    primed = false;
                    if (seq < 0) continue;
                }
                if (!primed) {
                    prime(seq, s0, r);
                    primed = true;
                }
                float cur[8];
                unpack8(*(const uint4*)(g.x + r * g.x_row + c), cur);
                emit(r, cur, true);
            }
        }
    }
}

/* Each sequence's conv-state slot becomes the last three input rows of (its history, its rows): thread t
 * takes (sequence, 4 channels), reads the old rows, then writes the new ones. */
__global__ void __launch_bounds__(kThreads) conv_state_kernel(RidgeFillConvPrep g) {
    const int64_t C = 2 * g.n_head_k * 128 + g.n_head_v * 128, quads = C / 4;
    const int64_t total = g.n_seq * quads;
    for (int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x; t < total; t += (int64_t)gridDim.x * kThreads) {
        const int64_t seq = t / quads, c = (t - seq * quads) * 4;
        const int64_t slot = g.idx[seq * g.idx_pitch];
        if (slot < 0 || slot >= g.n_states) continue;
        const int64_t a = seq_start(g, seq), b = min(max((int64_t)g.cu[seq + 1], a), g.T), L = b - a;
        const bool has = g.ctx != nullptr && g.ctx[seq] > 0;
        uint16_t* st = g.state + slot * g.st_slot + c;
        uint2 old[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) old[j] = has ? *(const uint2*)(st + j * C) : make_uint2(0u, 0u);
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const uint2 nv = L + j < 3 ? old[L + j] : *(const uint2*)(g.x + (b - 3 + j) * g.x_row + c);
            *(uint2*)(st + j * C) = nv;
        }
    }
}

}  // namespace

extern "C" int ridgefill_gdn_conv_prep_device(const RadArgs* a, RadStream s) {
    RidgeFillConvPrep g;
    const int rc = ridgefill_conv_prep_parse(a, &g);
    if (rc != RAD_OK) return rc;
    cudaStream_t stream = rf::as_stream(s);
    const int64_t C = 2 * g.n_head_k * 128 + g.n_head_v * 128;
    const int64_t tasks = (g.T + kRows - 1) / kRows * ((C / 128 + 1) / 2 - (g.q ? 0 : g.n_head_k / 2));
    if (tasks > 0) {
        static int per_sm = 0;   /* resident CTAs a SM (registers and the 64 KiB stage bound it) */
        if (!per_sm) {
            if (cudaFuncSetAttribute(conv_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kStageBytes) != cudaSuccess ||
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, conv_prep_kernel, kThreads, kStageBytes) != cudaSuccess ||
                per_sm <= 0)
                return RAD_E_DEVICE;
        }
        const int64_t blocks = (tasks + kThreads / 32 - 1) / (kThreads / 32), cap = (int64_t)rf::sm_count() * per_sm;
        conv_prep_kernel<<<(unsigned)(blocks < cap ? blocks : cap), kThreads, kStageBytes, stream>>>(g);
    }
    const int64_t quads = g.n_seq * (C / 4);
    if (quads > 0) {
        const int64_t blocks = (quads + kThreads - 1) / kThreads, cap = (int64_t)rf::sm_count() * 4;
        conv_state_kernel<<<(unsigned)(blocks < cap ? blocks : cap), kThreads, 0, stream>>>(g);
    }
    return rf::launch_status();
}
