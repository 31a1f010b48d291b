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
 * bit. One CTA of 1024 threads holds up to RIDGEFILL_MASK_MAX_ROWS keys (192 KiB of shared memory).
 */
#include "common.cuh"

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

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
    return t;
}

/* Exclusive prefix (in thread order) of one 0/1 flag per thread, and the block total. */
__device__ int block_exclusive_flag(bool flag, int* scratch, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned ballot = __ballot_sync(0xffffffffu, flag);
    const int before_in_warp = __popc(ballot & ((1u << lane) - 1u));
    __syncthreads();
    if (lane == 0) scratch[warp] = __popc(ballot);
    __syncthreads();
    int warp_base = 0, sum = 0;
    for (int w = 0; w < kWarps; ++w) {
        const int c = scratch[w];
        warp_base += w < warp ? c : 0;
        sum += c;
    }
    *total = sum;
    return warp_base + before_in_warp;
}

__global__ void __launch_bounds__(kThreads, 1) mask_kernel(RidgeFillMask g) {
    extern __shared__ uint32_t keys[];
    __shared__ int hist[256];
    __shared__ int scratch[kWarps];
    __shared__ uint32_t s_prefix;
    __shared__ int s_remaining;

    int64_t win[3];
    ridgefill_mask_window(g.cu_last[0], g.cu_last[1], g.b, g.n, win);   /* invalid: empty window */
    const int64_t from = ridgefill_mask_from(g.mode, win), end = win[1];
    if (threadIdx.x == 0) {
        g.bounds[0] = (int32_t)win[0];
        g.bounds[1] = (int32_t)end;
        g.bounds[2] = (int32_t)end;
        g.bounds[3] = (int32_t)win[2];
    }
    for (int64_t i = threadIdx.x; i < g.n; i += kThreads)
        if (i < from || i >= end) g.mask[i] = 0;
    for (int64_t i = threadIdx.x; i < g.n_zeros; i += kThreads) g.zeros[i] = 0;

    const int w = (int)(end - from);
    if (w <= 0) return;
    const bool ranked = g.mode == RIDGEFILL_MODE_CLASS || g.mode == RIDGEFILL_MODE_RANDOM;
    if (!ranked) {
        const int32_t v = g.mode == RIDGEFILL_MODE_ALL ? 0 : 1;   /* none and step approximate the window */
        for (int j = threadIdx.x; j < w; j += kThreads) g.mask[from + j] = v;
        return;
    }

    /* Keys and the match count. */
    int matches = 0;
    for (int j = threadIdx.x; j < w; j += kThreads) {
        const float sc = ridgefill_mask_score(&g, from + j);
        matches += sc > -INFINITY ? 1 : 0;
        keys[j] = g.mode == RIDGEFILL_MODE_CLASS ? class_key(sc)
                                                  : ridgefill_row_hash(g.seed, (uint32_t)g.positions[(from + j) * g.pos_stride]);
    }
    const int total_matches = block_sum(matches, scratch);
    const long long k = (long long)rint(g.share * (double)total_matches);

    /* Radix select of the k-th smallest key (1-based). */
    if (threadIdx.x == 0) {
        s_prefix = 0;
        s_remaining = (int)k;
    }
    uint32_t known = 0;   /* bits of the threshold fixed so far */
    if (k > 0 && k <= w) {
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
            __syncthreads();
            const uint32_t prefix = s_prefix;
            const int want = s_remaining;
            for (int j = threadIdx.x; j < w; j += kThreads) {
                const uint32_t key = keys[j];
                if ((key & known) == prefix) atomicAdd(&hist[(key >> shift) & 0xff], 1);
            }
            __syncthreads();
            if (threadIdx.x < 32) {
                /* Warp 0 finds the bin holding the remaining-th key: 8 bins a lane, then a scan. */
                const int lane = threadIdx.x;
                int local[8], sum = 0;
                for (int b = 0; b < 8; ++b) { local[b] = hist[lane * 8 + b]; sum += local[b]; }
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
            __syncthreads();
        }
    }
    __syncthreads();
    const uint32_t threshold = s_prefix;
    const int need_equal = s_remaining;   /* rows with key == threshold to keep, in row order */

    /* Decide each row in row order, 1024 rows at a time: the equal-key rank is a block prefix. */
    int equal_before = 0;
    for (int base = 0; base < w; base += kThreads) {
        const int j = base + threadIdx.x;
        const bool inside = j < w;
        const uint32_t key = inside ? keys[j] : 0xffffffffu;
        const bool equal = inside && k > 0 && k <= w && key == threshold;
        int chunk_equal = 0;
        const int rank = block_exclusive_flag(equal, scratch, &chunk_equal);
        if (inside) {
            bool kept;
            if (k <= 0) kept = false;
            else if (k > w) kept = g.mode == RIDGEFILL_MODE_RANDOM || key != 0xffffffffu;   /* every candidate */
            else kept = key < threshold || (equal && equal_before + rank < need_equal);
            if (g.mode == RIDGEFILL_MODE_CLASS && key == 0xffffffffu) kept = false;
            g.mask[from + j] = kept ? 0 : 1;
        }
        equal_before += chunk_equal;
    }
}

}  // namespace

extern "C" int ridgefill_mask_device(const RadArgs* a, RadStream s) {
    RidgeFillMask g;
    const int rc = ridgefill_mask_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.b > RIDGEFILL_MASK_MAX_ROWS) return RAD_E_SHAPE;   /* the window (<= b rows) must fit shared memory */
    const size_t smem = (size_t)(g.b > 0 ? g.b : 1) * sizeof(uint32_t);
    if (cudaFuncSetAttribute(mask_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return RAD_E_DEVICE;
    mask_kernel<<<1, kThreads, smem, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}
