/* small_ops.cu -- device rows of the reference's row ops: ridgefill_select, ridgefill_drop_rows,
 * ridgefill_state_correct, ridgefill_state_read, ridgefill_hazard and ridgefill_rho_update.
 *
 * Semantics are the reference's host rows (kernels/host_ref.cpp:334-472); each kernel is written for
 * the B200 memory system instead of the reference's one-workgroup-per-row layout
 * (kernels/select.hip, kernels/state_correct.hip, kernels/rho.hip):
 *  - select / drop: one warp per row over a persistent grid, 16-byte words where the pair allows;
 *    an exact row costs one broadcast read of its mask word.
 *  - state_correct / state_read: one CTA per (head, sequence), float4 traffic when the plane is
 *    packed; `x + s*c` rounds twice (__fmul_rn then __fadd_rn / __fsub_rn), as the host row compiled
 *    -ffp-contract=off does, so the two agree to the bit.
 *  - rho_update: the per-head recurrence D = e*D + 1, N = e*N + m is an affine map per row, so the
 *    rows are split into 256 runs (8 CTAs of a cluster x 32 runs), each run composes its maps
 *    sequentially, and the runs are combined in order (shared memory, then the cluster's
 *    distributed shared memory). Runs are anchored at the first row, so a call with bounds {s, ..}
 *    and a call on the slice [s, n) are the same arithmetic, bit for bit.
 */
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace {

/* ------------------------------------------------------------------ select / drop */

constexpr int kRowWarps = 8;   /* warps per CTA of the row kernels */

/* A row's words, lane l taking words l, l + 32, ...; eight of a lane's loads are issued before their stores. */
template <typename Word>
__device__ __forceinline__ void copy_row(const RidgeFillCopy& p, int64_t row, int lane) {
    const Word* src = (const Word*)(p.src + row * p.src_pitch);
    Word* dst = (Word*)(p.dst + row * p.dst_pitch);
    const int64_t words = p.row_bytes / (int64_t)sizeof(Word);
    int64_t w = lane;
    for (; w + 32 * 7 < words; w += 32 * 8) {
        Word v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = src[w + 32 * u];
#pragma unroll
        for (int u = 0; u < 8; ++u) dst[w + 32 * u] = v[u];
    }
    for (; w < words; w += 32) dst[w] = src[w];
}

__global__ void __launch_bounds__(32 * kRowWarps) select_kernel(RidgeFillSelect g) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * kRowWarps;
    for (int64_t row = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5); row < g.n; row += warps) {
        if (g.mask[row] != 1) continue;
#pragma unroll
        for (int k = 0; k < RIDGEFILL_SELECT_PAIRS; ++k) {
            const RidgeFillCopy& p = g.pair[k];
            if (p.word == 16) copy_row<uint4>(p, row, lane);
            else if (p.word == 4) copy_row<uint32_t>(p, row, lane);
            else if (p.word == 1) copy_row<uint8_t>(p, row, lane);
        }
    }
}

__global__ void __launch_bounds__(32 * kRowWarps) drop_kernel(RidgeFillDrop g) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * kRowWarps;
    for (int64_t row = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5); row < g.n; row += warps) {
        if (g.mask[row] != 1) continue;
        int32_t* ids = g.ids + row * g.pitch;
        for (int64_t j = lane; j < g.top_k; j += 32) ids[j] = -1;
    }
}

unsigned row_grid(int64_t rows) {
    const int64_t want = (rows + kRowWarps - 1) / kRowWarps;
    const int64_t cap = (int64_t)rf::sm_count() * 8;   /* 8 CTAs of 256 threads resident per SM */
    return (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
}

/* ------------------------------------------------------------------ state_correct / state_read */

constexpr int kPlaneThreads = 256;

constexpr int kCorrThreads = 1024, kCorrLoads = 4;   /* a plane's CTA: four float4 of x and of C in flight a thread */

__global__ void __launch_bounds__(kCorrThreads) correct_kernel(RidgeFillCorrect g) {
    const int64_t h = blockIdx.x, s = blockIdx.y;
    if (!ridgefill_correct_has_bulk(&g)) return;   /* bounds are device memory: read here */
    int64_t st = 0, ap = 0, nd = 0;
    if (!ridgefill_correct_slots(&g, s, &st, &ap, &nd)) return;
    float* applied = g.applied + ap * g.ap_slot + h * g.ap_head;
    __shared__ float s_scale;
    if (threadIdx.x == 0) {
        float scale = *applied;
        if (g.apply) {
            const float* p = g.nd ? g.nd + nd * g.nd_slot + h * g.nd_head : nullptr;
            scale = __fmul_rn(g.alpha, p ? ridgefill_rho(p[0], p[g.nd_inner]) : 1.0f);
        }
        s_scale = scale;
    }
    __syncthreads();
    const float scale = s_scale;
    if (scale != 0.0f) {
        float* x = g.state + st * g.st_slot + h * g.st_head;
        const float* c = g.c + h * g.c_head;
        const int64_t cells = g.sd0 * g.sd1;
        const bool vec = g.st_col == 1 && g.sd1 % 4 == 0 && g.st_row % 4 == 0 && ((uintptr_t)x & 15) == 0 &&
                         ((uintptr_t)c & 15) == 0;
        if (vec) {
            /* kCorrLoads float4 of x and of C loaded before any is updated (x and C may not alias) */
            for (int64_t e0 = (int64_t)threadIdx.x * 4; e0 < cells; e0 += (int64_t)kCorrThreads * 4 * kCorrLoads) {
                float4 xv[kCorrLoads], cv[kCorrLoads];
                float4* px[kCorrLoads];
#pragma unroll
                for (int u = 0; u < kCorrLoads; ++u) {
                    const int64_t e = e0 + (int64_t)u * kCorrThreads * 4;
                    const int64_t i = e / g.sd1, j = e - i * g.sd1;
                    px[u] = (float4*)(x + i * g.st_row + j);
                    if (e < cells) {
                        cv[u] = *(const float4*)(c + e);
                        xv[u] = *px[u];
                    }
                }
#pragma unroll
                for (int u = 0; u < kCorrLoads; ++u) {
                    if (e0 + (int64_t)u * kCorrThreads * 4 >= cells) break;
                    float4 v = xv[u];
                    const float d0 = __fmul_rn(scale, cv[u].x), d1 = __fmul_rn(scale, cv[u].y);
                    const float d2 = __fmul_rn(scale, cv[u].z), d3 = __fmul_rn(scale, cv[u].w);
                    if (g.apply) {
                        v.x = __fadd_rn(v.x, d0); v.y = __fadd_rn(v.y, d1); v.z = __fadd_rn(v.z, d2); v.w = __fadd_rn(v.w, d3);
                    } else {
                        v.x = __fsub_rn(v.x, d0); v.y = __fsub_rn(v.y, d1); v.z = __fsub_rn(v.z, d2); v.w = __fsub_rn(v.w, d3);
                    }
                    *px[u] = v;
                }
            }
        } else {
            for (int64_t e = threadIdx.x; e < cells; e += kCorrThreads) {
                const int64_t i = e / g.sd1, j = e - i * g.sd1;
                float* px = x + i * g.st_row + j * g.st_col;
                const float d = __fmul_rn(scale, c[i * g.c_row + j]);
                *px = g.apply ? __fadd_rn(*px, d) : __fsub_rn(*px, d);
            }
        }
    }
    if (threadIdx.x == 0) *applied = g.apply ? scale : 0.0f;
}

__global__ void __launch_bounds__(kPlaneThreads) state_read_kernel(RidgeFillStateRead g) {
    const int64_t h = blockIdx.x, s = blockIdx.y;
    const int32_t slot = g.idx[s * g.idx_pitch];
    const bool inside = slot >= 0 && slot < g.n_states;
    const float* x = inside ? g.state + slot * g.st_slot + h * g.st_head : g.state;
    float* out = g.out + (s * g.n_head + h) * g.sd0 * g.sd1;
    const int64_t cells = g.sd0 * g.sd1;
    const bool vec = g.st_col == 1 && g.sd1 % 4 == 0 && g.st_row % 4 == 0 && ((uintptr_t)x & 15) == 0 &&
                     ((uintptr_t)out & 15) == 0;
    if (vec) {
        for (int64_t e = (int64_t)threadIdx.x * 4; e < cells; e += kPlaneThreads * 4) {
            const int64_t i = e / g.sd1, j = e - i * g.sd1;
            *(float4*)(out + e) = inside ? *(const float4*)(x + i * g.st_row + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    } else {
        for (int64_t e = threadIdx.x; e < cells; e += kPlaneThreads) {
            const int64_t i = e / g.sd1, j = e - i * g.sd1;
            out[e] = inside ? x[i * g.st_row + j * g.st_col] : 0.0f;
        }
    }
}

/* ------------------------------------------------------------------ hazard */

__global__ void hazard_kernel(RidgeFillHazard g) {
    if (g.cu_last[0] < 0 || g.cu_last[0] > g.cu_last[1]) return;   /* fail-safe: count nothing */
    ridgefill_hazard_step(&g);
}

/* ------------------------------------------------------------------ rho_update */

constexpr int kRhoHeads = 4;    /* heads per CTA (threadIdx.x) */
constexpr int kRhoRuns = 256;   /* runs per CTA (threadIdx.y) */
constexpr int kRhoCluster = 8;  /* CTAs per cluster, each a segment of the rows */
constexpr int kRhoBatch = 8;    /* rows whose loads a thread issues together */

struct Affine { float a, bn, bd; };   /* x -> a*x + b, for N and D */

/* `first` then `second`: second(first(x)). */
__device__ __forceinline__ Affine compose(const Affine& first, const Affine& second) {
    return Affine{ second.a * first.a, second.a * first.bn + second.bn, second.a * first.bd + second.bd };
}

__global__ void __cluster_dims__(1, kRhoCluster, 1) __launch_bounds__(kRhoHeads * kRhoRuns)
rho_kernel(RidgeFillRho g) {
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ Affine part[kRhoRuns][kRhoHeads];
    const int hx = threadIdx.x, run = threadIdx.y;
    const int64_t h = (int64_t)blockIdx.x * kRhoHeads + hx;
    const int seg = (int)cluster.block_rank();
    const int32_t slot = g.state_idx[0];
    const bool live = slot >= 0 && slot < g.n_states;
    const int64_t first = ridgefill_rho_first_row(&g);
    const int64_t total = g.n - first;
    const int64_t runs = (int64_t)kRhoCluster * kRhoRuns;
    const int64_t len = (total + runs - 1) / runs;
    const int64_t r = (int64_t)seg * kRhoRuns + run;
    Affine m{ 1.0f, 0.0f, 0.0f };
    if (live && h < g.n_head && len > 0) {
        const float rate = expf(g.a_log[h]), bias = g.dt_bias[h];
        const int64_t t0 = first + r * len;
        const int64_t t1 = min(g.n, t0 + len);
        /* Rows in batches of kRhoBatch: the batch's loads are issued together, then the recurrence runs
         * over them in row order. */
        for (int64_t tb = t0; tb < t1; tb += kRhoBatch) {
            float x[kRhoBatch];
            int32_t mk[kRhoBatch];
#pragma unroll
            for (int u = 0; u < kRhoBatch; ++u) {
                const int64_t t = tb + u < t1 ? tb + u : t1 - 1;
                const int64_t at = t * g.a_pitch + h * g.a_col;
                x[u] = g.a_bf16 ? rf::bf16_bits_to_f32(((const uint16_t*)g.a)[at]) : ((const float*)g.a)[at];
                mk[u] = g.mask[t];
            }
#pragma unroll
            for (int u = 0; u < kRhoBatch; ++u) {
                if (tb + u >= t1) break;
                const float e = expf(-rate * ridgefill_softplus(x[u] + bias));
                m.a = e * m.a;
                m.bn = e * m.bn + (float)mk[u];
                m.bd = e * m.bd + 1.0f;
            }
        }
    }
    part[run][hx] = m;
    __syncthreads();
    /* In-order tree over this CTA's runs: after it, part[0][hx] is the segment's map. */
    for (int step = 1; step < kRhoRuns; step <<= 1) {
        if (run % (2 * step) == 0 && run + step < kRhoRuns) part[run][hx] = compose(part[run][hx], part[run + step][hx]);
        __syncthreads();
    }
    cluster.sync();   /* every segment's map is in its CTA's shared memory */
    if (seg == 0 && run == 0 && live && h < g.n_head) {
        Affine total_map = part[0][hx];
        for (int other = 1; other < kRhoCluster; ++other) {
            const Affine* remote = cluster.map_shared_rank(&part[0][hx], other);
            total_map = compose(total_map, *remote);
        }
        float* nd = g.nd + slot * g.nd_slot + h * g.nd_head;
        const float n0 = nd[0], d0 = nd[g.nd_inner];
        nd[0] = total_map.a * n0 + total_map.bn;
        nd[g.nd_inner] = total_map.a * d0 + total_map.bd;
    }
    cluster.sync();   /* no CTA leaves while its shared memory may still be read */
}

}  // namespace

extern "C" int ridgefill_select_device(const RadArgs* a, RadStream s) {
    RidgeFillSelect g;
    const int rc = ridgefill_select_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.n == 0) return RAD_OK;
    select_kernel<<<row_grid(g.n), 32 * kRowWarps, 0, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}

extern "C" int ridgefill_drop_device(const RadArgs* a, RadStream s) {
    RidgeFillDrop g;
    const int rc = ridgefill_drop_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.n == 0 || g.top_k == 0) return RAD_OK;
    drop_kernel<<<row_grid(g.n), 32 * kRowWarps, 0, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}

extern "C" int ridgefill_correct_device(const RadArgs* a, RadStream s) {
    RidgeFillCorrect g;
    const int rc = ridgefill_correct_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.n_seq == 0 || g.n_head == 0) return RAD_OK;
    if (g.n_head > 0x7fffffff || g.n_seq > 65535) return RAD_E_SHAPE;
    correct_kernel<<<dim3((unsigned)g.n_head, (unsigned)g.n_seq), kCorrThreads, 0, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}

extern "C" int ridgefill_state_read_device(const RadArgs* a, RadStream s) {
    RidgeFillStateRead g;
    const int rc = ridgefill_state_read_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.n_seq == 0 || g.n_head == 0) return RAD_OK;
    if (g.n_head > 0x7fffffff || g.n_seq > 65535) return RAD_E_SHAPE;
    state_read_kernel<<<dim3((unsigned)g.n_head, (unsigned)g.n_seq), kPlaneThreads, 0, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}

extern "C" int ridgefill_hazard_device(const RadArgs* a, RadStream s) {
    RidgeFillHazard g;
    const int rc = ridgefill_hazard_parse(a, &g);
    if (rc != RAD_OK) return rc;
    hazard_kernel<<<1, 1, 0, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}

extern "C" int ridgefill_rho_device(const RadArgs* a, RadStream s) {
    RidgeFillRho g;
    const int rc = ridgefill_rho_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.n == 0 || g.n_head == 0) return RAD_OK;
    const dim3 grid((unsigned)((g.n_head + kRhoHeads - 1) / kRhoHeads), kRhoCluster);
    rho_kernel<<<grid, dim3(kRhoHeads, kRhoRuns), 0, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}
