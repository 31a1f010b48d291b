/* mask.cu -- ridgefill_mask's device row: the exact rows of the step's last sequence.
 *
 * Semantics: kernels/host_ref.cpp:284-330 (rank counting) and the window rule of
 * kernels/ridgefill.h:130-139, read here from cu_last in device memory. The reference's device row
 * counts every row's rank against every other row (O(w^2), one workgroup, kernels/mask.hip:39-76) and
 * stops at 8,192 rows. This one selects instead:
 *
 *   key  class: the score mapped to an unsigned integer whose ascending order is the score's
 *        DESCENDING order (+0 and -0 one key, as the float compare sees them); a row that does not
 *        match gets 0xffffffff, which no finite score maps to. random: the row hash, ascending.
 *   k    = rint(share * matches), half to even, in double as the host computes it.
 *   T    = the k-th smallest key, found by an 8-bit radix select (four histogram passes over the
 *        keys in shared memory). Rows with key < T are kept; of the rows with key == T the first
 *        (k - #{key < T}) in row order are kept: the tie rule "ties by lower row".
 *
 * Every key, the tie order and k are the host row's, so the mask is identical to the host's bit for
 * bit. An 8-CTA cluster of 1024 threads each holds up to RIDGEFILL_MASK_MAX_ROWS keys, an eighth a CTA.
 */
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kCtas = 8;   /* the cluster: each CTA an eighth of the window */

/* Float order to unsigned order, then inverted: larger scores get smaller keys. */
__device__ __forceinline__ uint32_t class_key(float s) {
    if (!(s > -INFINITY)) return 0xffffffffu;   /* no match (the score is -inf after ridgefill_mask_score) */
    if (s == 0.0f) s = 0.0f;                    /* -0 ranks as +0 */
    const uint32_t u = __float_as_uint(s);
    const uint32_t ascending = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ~ascending;
}

/* Block-wide sum of one int per thread (all threads get it). */
__device__ int block_sum(int v, int* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    int t = lane < kWarps ? scratch[lane] : 0;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    __syncthreads();   /* scratch is read before its next use */
    return t;
}

constexpr int kKeyBatch = 8;     /* rows whose loads a thread issues together */
constexpr int kHists = 16;       /* private histograms, one per two warps */

/* An 8-CTA cluster; CTA r takes the window's rows [r P, r P + P), P = ceil(w / 8): its keys in its shared
 * memory, its part of the histograms, its rows' decisions. The cluster's sums (matches, each pass's
 * histogram, the equal keys of lower-ranked parts) are read through distributed shared memory; every CTA
 * then takes the same selection steps, so the threshold and the ranks are the one-CTA ones. */
__global__ void __cluster_dims__(kCtas, 1, 1) __launch_bounds__(kThreads, 1) mask_kernel(RidgeFillMask g) {
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ uint32_t keys[];
    __shared__ int hist_w[kHists][256];
    __shared__ int hist[256];          /* this CTA's histogram of the pass (read by the peers) */
    __shared__ int gsum[256];          /* the cluster's */
    __shared__ int scratch[kWarps];
    __shared__ int s_count;            /* this CTA's matches (read by the peers) */
    __shared__ int s_equal;            /* this CTA's rows with key == threshold (read by the peers) */
    __shared__ int s_total;
    __shared__ uint32_t s_prefix;
    __shared__ int s_remaining;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, rank = (int)cluster.block_rank();
    const int gtid = rank * kThreads + threadIdx.x;

    int64_t win[3];
    ridgefill_mask_window(g.cu_last[0], g.cu_last[1], g.b, g.n, win);   /* invalid: empty window */
    const int64_t from = ridgefill_mask_from(g.mode, win), end = win[1];
    if (gtid == 0) {
        g.bounds[0] = (int32_t)win[0];
        g.bounds[1] = (int32_t)end;
        g.bounds[2] = (int32_t)end;
        g.bounds[3] = (int32_t)win[2];
    }
    for (int64_t i = gtid; i < g.n; i += kCtas * kThreads)
        if (i < from || i >= end) g.mask[i] = 0;
    for (int64_t i = gtid; i < g.n_zeros; i += kCtas * kThreads) g.zeros[i] = 0;

    const int w = (int)(end - from);
    if (w <= 0) return;   /* every CTA of the cluster leaves here alike */
    const int per = (w + kCtas - 1) / kCtas, p0 = min(w, rank * per), p1 = min(w, p0 + per), pl = p1 - p0;
    const bool ranked = g.mode == RIDGEFILL_MODE_CLASS || g.mode == RIDGEFILL_MODE_RANDOM;
    if (!ranked) {
        const int32_t v = g.mode == RIDGEFILL_MODE_ALL ? 0 : 1;   /* none and step approximate the window */
        for (int j = p0 + threadIdx.x; j < p1; j += kThreads) g.mask[from + j] = v;
        return;
    }

    /* This part's keys and match count (rows whose token has a finite score, in both modes), kKeyBatch rows'
     * loads issued together. */
    int matches = 0;
    const bool cls = g.mode == RIDGEFILL_MODE_CLASS;
    for (int j0 = threadIdx.x; j0 < pl; j0 += kThreads * kKeyBatch) {
        int32_t id[kKeyBatch], pos[kKeyBatch];
#pragma unroll
        for (int u = 0; u < kKeyBatch; ++u) {
            const int j = j0 + u * kThreads;
            id[u] = j < pl ? g.tokens[from + p0 + j] : -1;
            pos[u] = j < pl && !cls ? g.positions[(from + p0 + j) * g.pos_stride] : 0;
        }
        float sc[kKeyBatch];
#pragma unroll
        for (int u = 0; u < kKeyBatch; ++u) sc[u] = id[u] >= 0 && id[u] < g.vocab ? g.score[id[u]] : -INFINITY;
#pragma unroll
        for (int u = 0; u < kKeyBatch; ++u) {
            const int j = j0 + u * kThreads;
            if (j >= pl) break;
            const float s = sc[u] > -INFINITY && sc[u] < INFINITY ? sc[u] : -INFINITY;   /* ridgefill_mask_score */
            matches += s > -INFINITY ? 1 : 0;
            keys[j] = cls ? class_key(s) : ridgefill_row_hash(g.seed, (uint32_t)pos[u]);
        }
    }
    const int part_matches = block_sum(matches, scratch);
    if (threadIdx.x == 0) s_count = part_matches;
    cluster.sync();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int r = 0; r < kCtas; ++r) t += *cluster.map_shared_rank(&s_count, r);
        s_total = t;
        s_prefix = 0;
    }
    __syncthreads();
    const long long k = (long long)rint(g.share * (double)s_total);
    if (threadIdx.x == 0) s_remaining = (int)k;
    const bool selecting = k > 0 && k <= w;

    /* Radix select of the k-th smallest key (1-based): four 8-bit passes, each the cluster's histogram of
     * the keys that match the threshold's known bits. */
    uint32_t known = 0;
    if (selecting) {
        int* myhist = hist_w[warp % kHists];
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = threadIdx.x; i < kHists * 256; i += kThreads) (&hist_w[0][0])[i] = 0;
            __syncthreads();
            const uint32_t prefix = s_prefix;
            const int want = s_remaining;
            for (int j0 = warp * 32; j0 < pl; j0 += kThreads) {   /* whole warps: match_any needs every lane */
                const int j = j0 + lane;
                const uint32_t key = j < pl ? keys[j] : 0u;
                const int bin = j < pl && (key & known) == prefix ? (int)((key >> shift) & 0xff) : 256;
                const unsigned any = __ballot_sync(0xffffffffu, bin < 256);
                if (!any) continue;
                const unsigned same = __match_any_sync(0xffffffffu, bin);
                if (bin < 256 && lane == __ffs(same) - 1) atomicAdd(&myhist[bin], __popc(same));
            }
            __syncthreads();
            if (threadIdx.x < 256) {
                int t = 0;
#pragma unroll
                for (int q = 0; q < kHists; ++q) t += hist_w[q][threadIdx.x];
                hist[threadIdx.x] = t;
            }
            cluster.sync();   /* every part's histogram is ready */
            if (threadIdx.x < 256) {
                int t = 0;
                for (int r = 0; r < kCtas; ++r) t += cluster.map_shared_rank(hist, r)[threadIdx.x];
                gsum[threadIdx.x] = t;
            }
            __syncthreads();
            if (threadIdx.x < 32) {
                /* Warp 0 finds the bin holding the remaining-th key: 8 bins a lane, then a scan. */
                int local[8], sum = 0;
                for (int b = 0; b < 8; ++b) { local[b] = gsum[lane * 8 + b]; sum += local[b]; }
                int incl = sum;
                for (int o = 1; o < 32; o <<= 1) {
                    const int v = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += v;
                }
                const int excl = incl - sum;
                if (want > excl && want <= incl) {
                    int acc = excl, bin = 0;
                    for (int b = 0; b < 8; ++b) {
                        if (want <= acc + local[b]) { bin = lane * 8 + b; break; }
                        acc += local[b];
                    }
                    s_prefix = prefix | ((uint32_t)bin << shift);
                    s_remaining = want - acc;
                }
            }
            known |= 0xffu << shift;
            cluster.sync();   /* the peers have read this CTA's histogram before the next pass rewrites it */
        }
    }
    const uint32_t threshold = s_prefix;
    const int need_equal = s_remaining;   /* rows with key == threshold to keep, in row order */

    /* Decide each row of the part in row order. Warp v owns the block of rows [v B, v B + B), walked 32 rows
     * at a time; a row's equal-key rank = the equal keys of the lower-ranked parts + of the blocks before
     * its warp's + before it in its block (ballots). */
    const int B = ((pl + kThreads - 1) / kThreads) * 32;
    const int b0 = min(pl, warp * B), b1 = min(pl, b0 + B);
    int equal_here = 0;
    if (selecting)
        for (int j = b0 + lane; j - lane < b1; j += 32)
            equal_here += __popc(__ballot_sync(0xffffffffu, j < b1 && keys[j] == threshold));
    if (lane == 0) scratch[warp] = equal_here;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int q = 0; q < kWarps; ++q) t += scratch[q];
        s_equal = t;
    }
    cluster.sync();
    int rank_base = 0;
    for (int r = 0; r < rank; ++r) rank_base += *cluster.map_shared_rank(&s_equal, r);
    for (int q = 0; q < warp; ++q) rank_base += scratch[q];
    int eq_rank = rank_base;
    for (int j = b0 + lane; j - lane < b1; j += 32) {
        const bool inside = j < b1;
        const uint32_t key = inside ? keys[j] : 0xffffffffu;
        const bool equal = selecting && inside && key == threshold;
        const unsigned eq = __ballot_sync(0xffffffffu, equal);
        const int my_rank = eq_rank + __popc(eq & ((1u << lane) - 1u));
        eq_rank += __popc(eq);
        if (!inside) continue;
        bool kept;
        if (k <= 0) kept = false;
        else if (k > w) kept = g.mode == RIDGEFILL_MODE_RANDOM || key != 0xffffffffu;   /* every candidate */
        else kept = equal ? my_rank < need_equal : key < threshold;
        if (g.mode == RIDGEFILL_MODE_CLASS && key == 0xffffffffu) kept = false;
        g.mask[from + p0 + j] = kept ? 0 : 1;
    }
    cluster.sync();   /* no CTA leaves while a peer may still read its shared memory */
}

}  // namespace

extern "C" int ridgefill_mask_device(const RadArgs* a, RadStream s) {
    RidgeFillMask g;
    const int rc = ridgefill_mask_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.b > RIDGEFILL_MASK_MAX_ROWS) return RAD_E_SHAPE;   /* the window (<= b rows) must fit shared memory */
    const size_t smem = (size_t)((g.b > 0 ? g.b : 1) + kCtas - 1) / kCtas * sizeof(uint32_t);   /* a CTA's part */
    if (cudaFuncSetAttribute(mask_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return RAD_E_DEVICE;
    mask_kernel<<<kCtas, kThreads, smem, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}
