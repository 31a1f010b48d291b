/* conv_prep.cu -- ridgefill_gdn_conv_prep: the Gated DeltaNet block's input preparation on B200, the step
 * between the block's input projections and the chunk fill (issue site arch/qwen4exp_fill.h:41-50,
 * arch/qwen4exp_blocks.h:118-134). The reference issues radiance's in-tree gdn_conv_prep, whose source is not
 * part of the checkout; the arithmetic here is the Gated DeltaNet block's published input path (causal
 * depthwise convolution of width 4, SiLU, per-head L2 normalisation of q and k) and the reference's own gate
 * g = -exp(A_log) softplus(a + dt_bias) (kernels/ridgefill.h:93-97), written per row for ridgefill_gdn_fill.
 *
 * HBM-bound: x is read once and q, k, v written once (2 x 2 C bytes a row). Without a q operand (the state-only
 * fill reads no q) the q columns are neither read nor computed; the conv state still takes every channel of each
 * sequence's last three rows, so x's q columns need be valid only there. A warp takes 16 rows of one 128-channel
 * head column, lane l channels 4 l..4 l + 3 (8-byte loads and stores, a warp's row 256 contiguous bytes); the
 * convolution's three earlier rows ride in registers; when the 16 rows lie in one sequence, all their loads are in
 * flight at once as asynchronous copies into the lane's own shared-memory slots (32 KiB a CTA, three CTAs a SM). The
 * gates of a row block are one more warp task, a lane per v-head. A second kernel then writes each sequence's last
 * three input rows into its conv-state slot (it reads the old state first, thread by thread, so the update is in
 * place). With columns == 0 (ridgefill_gdn_in_proj has produced k and v) only the gates and the conv state are
 * written.
 */
#include <cuda_bf16.h>

#include "common.cuh"
#include "sm100.cuh"

namespace {

constexpr int kRows = 16;        /* rows a warp task */
constexpr int kThreads = 256;
constexpr int kStageBytes = (kThreads / 32) * kRows * 256;   /* a warp's 16 rows of 256 bytes, for every warp */

/* 8-byte asynchronous copy global -> shared, in the current cp.async group. */
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void unpack4(uint2 v, float (&f)[4]) {
    f[0] = __uint_as_float(v.x << 16);
    f[1] = __uint_as_float(v.x & 0xffff0000u);
    f[2] = __uint_as_float(v.y << 16);
    f[3] = __uint_as_float(v.y & 0xffff0000u);
}

/* Two f32 as a bf16 pair, rounded to nearest even by the hardware conversion (one instruction for both). */
__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *(const uint32_t*)&p;
}

__device__ __forceinline__ int64_t seq_start(const RidgeFillConvPrep& g, int64_t i) { return rf::seq_start(g.cu, g.T, i); }

__device__ __forceinline__ int find_seq(const RidgeFillConvPrep& g, int64_t r, int64_t* s0, int64_t* e0) {
    return rf::find_seq(g.cu, g.n_seq, g.T, r, s0, e0);
}

/* Whether sequence `seq` continues a context held in its conv-state slot; the slot (or -1). */
__device__ __forceinline__ int64_t history_slot(const RidgeFillConvPrep& g, int64_t seq) {
    const int64_t slot = g.idx[seq * g.idx_pitch];
    const bool has = g.ctx != nullptr && g.ctx[seq] > 0 && slot >= 0 && slot < g.n_states;
    return has ? slot : -1;
}

/* Channels c..c+3 of input row `row` of the sequence starting at s0 (row >= s0 - 3): x, or the state's
 * history row (s0 - row rows back), or zero. */
__device__ __forceinline__ uint2 window_row(const RidgeFillConvPrep& g, int64_t slot, int64_t s0, int64_t row, int64_t c,
                                            int64_t C) {
    if (row >= s0) return *(const uint2*)(g.x + row * g.x_row + c);
    if (slot < 0) return make_uint2(0u, 0u);
    return *(const uint2*)(g.state + slot * g.st_slot + (3 - (s0 - row)) * C + c);
}

/* The gates of rows [r0, r1) for every v-head, lane = head (coalesced over the heads): rows outside every sequence
 * are left untouched. */
__device__ void gate_rows(const RidgeFillConvPrep& g, int64_t r0, int64_t r1, int lane) {
    int64_t s0 = 0, e0 = 0;
    const int seq0 = find_seq(g, r0, &s0, &e0);
    const bool all_in = seq0 >= 0 && e0 >= r1;
    for (int64_t h = lane; h < g.n_head_v; h += 32) {
        const float neg_a = -expf(g.a_log[h]), dtb = g.dt_bias[h];
        int64_t s = s0, e = e0;
        int seq = seq0;
        for (int64_t r = r0; r < r1; ++r) {
            if (!all_in && (seq < 0 || r >= e)) {
                seq = find_seq(g, r, &s, &e);
                if (seq < 0) continue;
            }
            const float av = rf::bf16_bits_to_f32(g.a[r * g.a_row + h]);
            const float bv = rf::bf16_bits_to_f32(g.b[r * g.b_row + h]);
            g.g[r * g.g_row + h] = neg_a * ridgefill_softplus(av + dtb);
            g.beta[r * g.beta_row + h] = 1.0f / (1.0f + expf(-bv));
        }
    }
}

/* The gates alone (columns == 0: ridgefill_gdn_in_proj has written k and v): a warp per 16-row block, a lane per
 * v-head; when the block lies in one sequence, eight rows' a and b are in flight before their arithmetic. The same
 * per-element arithmetic as gate_rows. */
__global__ void __launch_bounds__(kThreads, 4) gate_kernel(RidgeFillConvPrep g) {
    const int lane = threadIdx.x & 31;
    const int64_t blocks = (g.T + kRows - 1) / kRows, stride = (int64_t)gridDim.x * (kThreads / 32);
    for (int64_t blk = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); blk < blocks; blk += stride) {
        const int64_t r0 = blk * kRows, r1 = min(r0 + kRows, g.T);
        int64_t s0 = 0, e0 = 0;
        const int seq0 = find_seq(g, r0, &s0, &e0);
        if (seq0 < 0 || e0 < r1) {   /* sequence boundaries or rows outside every sequence inside the block */
            gate_rows(g, r0, r1, lane);
            continue;
        }
        for (int64_t h = lane; h < g.n_head_v; h += 32) {
            const float neg_a = -expf(g.a_log[h]), dtb = g.dt_bias[h];
            for (int64_t q0 = r0; q0 < r1; q0 += 8) {
                const int n = (int)min((int64_t)8, r1 - q0);
                uint16_t ab[8], bb[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if (i < n) {
                        ab[i] = __ldg(g.a + (q0 + i) * g.a_row + h);
                        bb[i] = __ldg(g.b + (q0 + i) * g.b_row + h);
                    }
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if (i < n) {
                        const int64_t r = q0 + i;
                        g.g[r * g.g_row + h] = neg_a * ridgefill_softplus(rf::bf16_bits_to_f32(ab[i]) + dtb);
                        g.beta[r * g.beta_row + h] = 1.0f / (1.0f + expf(-rf::bf16_bits_to_f32(bb[i])));
                    }
            }
        }
    }
}

/* Tasks of kRows rows: per row block, one task per computed 128-channel head column (a warp; lane l channels
 * 4 l..4 l + 3) and one gate task (gate_rows). The block's tasks are consecutive, so the warps of a wave share
 * rows. In a head task the convolution's three earlier rows ride in registers; when the rows lie in one sequence
 * all their loads are in flight at once as asynchronous copies into the lane's own shared-memory slots (4 KiB a
 * warp), so 78 registers and 32 KiB a CTA leave room for three CTAs (24 warps) a SM. */
__global__ void __launch_bounds__(kThreads, 3) conv_prep_kernel(RidgeFillConvPrep g) {
    extern __shared__ uint2 rows_smem[];   /* [warp][kRows][lane] */
    const int lane = threadIdx.x & 31;
    uint2* stage = rows_smem + (threadIdx.x >> 5) * kRows * 32 + lane;
    const int64_t hk = g.n_head_k;
    const int64_t C = 2 * hk * 128 + g.n_head_v * 128, n_hc = C / 128;
    /* without a q output the q columns are not computed; with columns == 0 none is (only the gates) */
    const int64_t first = g.q ? 0 : hk, live = g.columns ? n_hc - first : 0, per_block = live + 1;
    const int64_t tasks = (g.T + kRows - 1) / kRows * per_block;
    const int64_t stride = (int64_t)gridDim.x * (kThreads / 32);
    for (int64_t task = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); task < tasks; task += stride) {
        const int64_t blk = task / per_block, j = task - blk * per_block;
        const int64_t r0 = blk * kRows, r1 = min(r0 + kRows, g.T);
        if (j == live) {
            gate_rows(g, r0, r1, lane);
            continue;
        }
        const int64_t hc = first + j, c = hc * 128 + 4 * lane;
        const bool norm = hc < 2 * hk;   /* q and k columns are L2-normalised */
        float wt[4][4], bs[4];
        {
            const uint4 w01 = *(const uint4*)(g.w + c * 4), w23 = *(const uint4*)(g.w + c * 4 + 8);
            const uint32_t ww[8] = { w01.x, w01.y, w01.z, w01.w, w23.x, w23.y, w23.z, w23.w };
#pragma unroll
            for (int e = 0; e < 4; ++e)
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint32_t word = ww[2 * e + (t >> 1)];
                    wt[e][t] = __uint_as_float((t & 1) ? (word & 0xffff0000u) : (word << 16));
                }
            if (g.bias) unpack4(*(const uint2*)(g.bias + c), bs);
            else {
#pragma unroll
                for (int e = 0; e < 4; ++e) bs[e] = 0.0f;
            }
        }
        const int kind = hc < hk ? 0 : (hc < 2 * hk ? 1 : 2);   /* q, k, v */
        const int64_t head = kind == 0 ? hc : (kind == 1 ? hc - hk : hc - 2 * hk);
        uint16_t* out = (kind == 0 ? g.q + head * g.q_head : (kind == 1 ? g.k + head * g.k_head : g.v + head * g.v_head)) + 4 * lane;
        const int64_t out_row = kind == 0 ? g.q_row : (kind == 1 ? g.k_row : g.v_row);

        float w0[4], w1[4], w2[4];   /* rows r-3, r-2, r-1 */
        /* one row: the convolution over (w0, w1, w2, cur), SiLU, the head's L2 norm for q and k, bf16 out */
        auto emit = [&](uint16_t* dst, const float (&cur)[4]) {
            float y[4];
#pragma unroll
            for (int e = 0; e < 4; e += 2) {   /* the taps two channels an instruction (packed f32x2, same roundings) */
                float u0 = bs[e], u1 = bs[e + 1];
                rf::fma2_rn(u0, u1, wt[e][0], wt[e + 1][0], w0[e], w0[e + 1]);
                rf::fma2_rn(u0, u1, wt[e][1], wt[e + 1][1], w1[e], w1[e + 1]);
                rf::fma2_rn(u0, u1, wt[e][2], wt[e + 1][2], w2[e], w2[e + 1]);
                rf::fma2_rn(u0, u1, wt[e][3], wt[e + 1][3], cur[e], cur[e + 1]);
                y[e] = rf::silu(u0);
                y[e + 1] = rf::silu(u1);
            }
            if (norm) {
                float ss = 0.0f;
#pragma unroll
                for (int e = 0; e < 4; ++e) ss = fmaf(y[e], y[e], ss);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                const float inv = rsqrtf(ss + 1e-6f);   /* within 2 ulp: well inside bf16's rounding */
                rf::mul2_rn(y[0], y[1], y[0], y[1], inv, inv);
                rf::mul2_rn(y[2], y[3], y[2], y[3], inv, inv);
            }
            *(uint2*)dst = make_uint2(bf16x2(y[0], y[1]), bf16x2(y[2], y[3]));
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                w0[e] = w1[e];
                w1[e] = w2[e];
                w2[e] = cur[e];
            }
        };
        auto prime = [&](int64_t seq, int64_t s0, int64_t r) {
            const int64_t slot = history_slot(g, seq);
            unpack4(window_row(g, slot, s0, r - 3, c, C), w0);
            unpack4(window_row(g, slot, s0, r - 2, c, C), w1);
            unpack4(window_row(g, slot, s0, r - 1, c, C), w2);
        };

        int64_t s0 = 0, e0 = 0;
        const int seq0 = find_seq(g, r0, &s0, &e0);
        if (seq0 >= 0 && e0 >= r1) {
            /* the task's rows lie in one sequence: all their loads in flight at once (no register holds them) */
            const int n = (int)(r1 - r0);
            {
                const uint16_t* src = g.x + r0 * g.x_row + c;
                for (int i = 0; i < n; ++i, src += g.x_row) cp_async8(stage + i * 32, src);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            prime(seq0, s0, r0);
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            uint16_t* dst = out + r0 * out_row;
#pragma unroll 2
            for (int i = 0; i < n; ++i, dst += out_row) {
                float cur[4];
                unpack4(stage[i * 32], cur);
                emit(dst, cur);
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
                float cur[4];
                unpack4(*(const uint2*)(g.x + r * g.x_row + c), cur);
                emit(out + r * out_row, cur);
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
    const int64_t tasks = (g.T + kRows - 1) / kRows * ((g.columns ? C / 128 - (g.q ? 0 : g.n_head_k) : 0) + 1);
    if (!g.columns && tasks > 0) {
        const int64_t blocks = (tasks + kThreads / 32 - 1) / (kThreads / 32), cap = (int64_t)rf::sm_count() * 8;
        gate_kernel<<<(unsigned)(blocks < cap ? blocks : cap), kThreads, 0, stream>>>(g);
    } else if (tasks > 0) {
        static int per_sm = 0;   /* resident CTAs a SM (registers and the 32 KiB stage bound it) */
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
