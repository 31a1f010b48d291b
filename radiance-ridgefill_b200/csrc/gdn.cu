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
 *     S_L = gamma_L S0 + U^T K~,   K~ = diag(exp(G_L - G)) K.
 *
 *   plan (gdn_plan_kernel), one CTA: each sequence's clamped rows and the number of chunks before it,
 *     into the head of the scratch, so neither phase walks cu_seqlens.
 *   phase 1 (gdn_prep_kernel), every (chunk, v-head) in parallel, persistent CTAs, the next item's k and
 *     v rows arriving by TMA (128-byte-swizzled boxes) while the current one is computed: K K^T on tensor
 *     cores (bf16, exact inputs), A, T by blocked inversion (16x16 diagonal blocks by column-parallel
 *     substitution in f32, off-diagonal blocks by f16 tensor-core products), then W = T (beta gamma K),
 *     U~ = T (beta V) and K~, all f16. The chunk's scratch slot receives W, K~, U~^T (128-byte-swizzled
 *     f16 tiles), G, beta and gamma_L: W and U~^T staged over the consumed input tiles and bulk-stored,
 *     K~ straight from registers.
 *   phase 2 (gdn_chain_kernel), one CTA per (32-row slice of dv, head, sequence), sequential over the
 *     sequence's chunks: one loader lane keeps four chunks in flight (W|K~, the slice of U~^T and gamma_L,
 *     three bulk copies a chunk); 4 chain warps (2 dv row halves x 2 dk halves) hold the state slice in
 *     registers and run V' = U~ - W S^T,  S <- gamma_L S + V'^T K~ on f16 mma.sync with f32
 *     accumulation. Loader and chain hand stages over through mbarriers (bounded waits; the chain's wait
 *     is taken by one thread and broadcast through a named barrier, so the chain leaves its loop as a
 *     whole).
 * f16 operands with f32 accumulation keep the state within 4e-4 relative L2 of the f64 sequential
 * rule in the configurations this library is tested on (bf16 operands would not: ~3e-3).
 */
#include <cuda_fp16.h>

#include <cstddef>
#include <mutex>

#include "common.cuh"
#include "mma.cuh"
#include "sm100.cuh"

namespace {

constexpr int C = 64;          /* rows a chunk */
constexpr int D = 128;         /* head dims (dk = dv) */
constexpr int TP = C + 8;      /* pitch of 64-wide b16 rows in shared memory (conflict-free ldmatrix) */
constexpr int VS = 32;         /* dv rows per phase-2 CTA */
constexpr int PP = C + 8;      /* pitch of the f32 exchange tiles (float2 stores and loads without conflicts) */
constexpr int kStages = 4;     /* phase 2: chunks in flight */

/* A chunk's scratch slot, per (chunk, v-head), f16 tiles in the 128-byte-swizzled layout of sw128_off:
 * W [64 rows][128 dk] (two 64-column halves), K~ [64 rows][128 dk] (two halves, the k tile's own layout) and
 * U~^T [128 dv][64 rows] (dv slice s of phase 2 at 4096 s), then G f32 [64], beta f32 [64] and gamma_L
 * (16 bytes). W and U~^T are K-major operands of the chain's products, K~ an MN-major one. */
constexpr int kSlotW = 0, kSlotK = 16384, kSlotU = 32768, kSlotMeta = 49152, kSlotGl = kSlotMeta + 512;
constexpr int kSlotBytes = kSlotGl + 16;
constexpr uint32_t kTileBytes = C * D * 2;   /* one [64][128] b16 tile, and one TMA pair of [64][64] boxes */

enum { kBarChain = 1, kBarPair0 = 2 };   /* named barriers of the output form's chain (0 is __syncthreads) */

/* The scratch: the sequence table (int32 r0[n], r1[n], base[n + 1]; base[i] is the number of chunks before
 * sequence i, capped at max_slots), the work counter, one ready flag per chunk slot and v-head, then the
 * chunk slots; each part padded to 256 bytes. */
int64_t table_bytes(int64_t n_seq) { return (3 * n_seq + 1) * 4 + 255 & ~(int64_t)255; }
constexpr int64_t kCtlBytes = 256;
int64_t flag_bytes(int64_t items) { return items * 4 + 255 & ~(int64_t)255; }

struct FillCtl {
    int next_item;    /* the transform's next (chunk slot, v-head) item */
};

/* Output form only: per (chunk slot, v-head), the state at the chunk's start S0 f16 [dv][SP] and the
 * corrected values U^T f16 [dv][TP] (rows of the chunk along the pitch), written by phase 2 for the
 * output kernel. */
constexpr int SP = D + 8;
constexpr int kOutS0 = 0, kOutU = D * SP * 2, kOutBytes = kOutU + D * TP * 2;

struct GdnPlan {
    RidgeFillGdn g;
    int32_t* tab;     /* the sequence table */
    FillCtl* ctl;     /* the work counter (zeroed by the plan kernel) */
    int* flags;       /* item i's slot is written (1) or not yet (0); zeroed by the plan kernel */
    uint8_t* slots;   /* the chunk slots */
    uint8_t* outws;   /* output form: S0 and U^T per chunk slot and v-head; null for the state-only fill */
    int max_slots;
    int head_block;   /* phase 1 takes the v-heads in blocks of this many (item_at); the chains the same (chain_at) */
};

/* Phase 1's item i (of slots x Hv, slots = every sequence's chunks): the v-heads in blocks of head_block, every
 * chunk slot of one block's heads before the next block's, slot-major inside a block. With head_block = the
 * number of chain CTAs, block b holds exactly the chains the chain CTAs run b-th (chain_at), so phase 1 makes
 * the chunks in the order the chains read them, however many heads the launch holds. */
__device__ __forceinline__ void item_at(const GdnPlan& p, int64_t item, int64_t slots, int64_t* slot, int64_t* h) {
    const int64_t hb = p.head_block, Hv = p.g.n_head_v;
    const int64_t blk = item / (slots * hb), j = item - blk * slots * hb;
    const int64_t nh = min(hb, Hv - blk * hb);
    *slot = j / nh;
    *h = blk * hb + j % nh;
}

/* Chain cid (of Hv x n_seq): the same head blocks; inside a block sequence-major, so chain CTA c (taking
 * chains c, c + head_block, ...) runs head b * head_block + c of every sequence in turn, block by block. */
__device__ __forceinline__ void chain_at(const GdnPlan& p, int64_t cid, int64_t* h, int64_t* seq) {
    const int64_t hb = p.head_block, Hv = p.g.n_head_v, n = p.g.n_seq;
    const int64_t blk = cid / (hb * n), r = cid - blk * hb * n;
    const int64_t nh = min(hb, Hv - blk * hb);
    *seq = r / nh;
    *h = blk * hb + r % nh;
}

__device__ __forceinline__ uint8_t* out_ptr(const GdnPlan& p, int64_t slot, int64_t h) {
    return p.outws + (slot * p.g.n_head_v + h) * (int64_t)kOutBytes;
}

__device__ __forceinline__ uint8_t* slot_ptr(const GdnPlan& p, int64_t slot, int64_t h) {
    return p.slots + (slot * p.g.n_head_v + h) * (int64_t)kSlotBytes;
}

/* cp.async of 4 bytes (src_bytes 0: zero fill). */
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(rf::saddr(dst)), "l"(src), "r"(src_bytes) : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
    return r;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) { asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory"); }
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}

/* Eight bf16 (one 16-byte chunk) times f, as eight f16; zero when !in. */
__device__ __forceinline__ uint4 scale_bf16x8_to_f16(uint4 raw, float f, bool in) {
    const uint32_t rw[4] = { raw.x, raw.y, raw.z, raw.w };
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
        o[e] = in ? rf::pack_f16(f * __uint_as_float(rw[e] << 16), f * __uint_as_float(rw[e] & 0xffff0000u)) : 0u;
    return make_uint4(o[0], o[1], o[2], o[3]);
}

/* ------------------------------------------------------------------ plan */

constexpr int kPlanThreads = 1024;

/* Sequence i's rows [r0, r1): cu_seqlens read on the device and clamped into [0, T] (a value the host
 * cannot check never sends a load outside the operands), and base[i] by a block-wide scan. */
__global__ void __launch_bounds__(kPlanThreads) gdn_plan_kernel(const GdnPlan p) {
    __shared__ long long warp_sum[32];
    __shared__ long long carry;
    const RidgeFillGdn& g = p.g;
    const int n = (int)g.n_seq, l = threadIdx.x & 31, w = threadIdx.x >> 5;
    int32_t* r0t = p.tab;
    int32_t* r1t = p.tab + n;
    int32_t* bt = p.tab + 2 * n;
    if (threadIdx.x == 0) {
        carry = 0;
        p.ctl->next_item = 0;
    }
    for (int64_t i = threadIdx.x; i < (int64_t)p.max_slots * g.n_head_v; i += kPlanThreads) p.flags[i] = 0;
    __syncthreads();
    for (int i0 = 0; i0 < n; i0 += kPlanThreads) {
        const int i = i0 + threadIdx.x;
        long long chunks = 0;
        if (i < n) {
            const int64_t a = min(max((int64_t)g.cu[i], (int64_t)0), g.T);
            const int64_t b = min(max((int64_t)g.cu[i + 1], a), g.T);
            r0t[i] = (int32_t)a;
            r1t[i] = (int32_t)b;
            chunks = (b - a + C - 1) / C;
        }
        long long x = chunks;
        for (int o = 1; o < 32; o <<= 1) {
            const long long y = __shfl_up_sync(0xffffffffu, x, o);
            if (l >= o) x += y;
        }
        if (l == 31) warp_sum[w] = x;
        __syncthreads();
        if (w == 0) {
            long long t = warp_sum[l];
            for (int o = 1; o < 32; o <<= 1) {
                const long long y = __shfl_up_sync(0xffffffffu, t, o);
                if (l >= o) t += y;
            }
            warp_sum[l] = t;
        }
        __syncthreads();
        const long long incl = carry + (w ? warp_sum[w - 1] : 0) + x;
        if (i < n) bt[i] = (int32_t)min(incl - chunks, (long long)p.max_slots);
        __syncthreads();
        if (threadIdx.x == kPlanThreads - 1) carry = incl;
        __syncthreads();
    }
    if (threadIdx.x == 0) bt[n] = (int32_t)min(carry, (long long)p.max_slots);
}

/* ------------------------------------------------------------------ phase 1 */

constexpr int kPrepThreads = 256;
/* The thread that issues a group's bulk copies (TMA loads, slot stores) and publishes its slots: lane 0 of warp
 * 4, which has no block of K K^T, so its waits on the stores overlap that product. */
constexpr int kStoreTid = 128;
constexpr int kSeqCache = 256;   /* sequences whose table rows a CTA keeps in shared memory */

struct PrepSmem {
    uint16_t kraw[2][2][C][C];   /* k rows of the current and the next item (TMA, 128-byte swizzled); then
                                    beta gamma k in f16 in place; then W (staging for the slot) */
    uint16_t vraw[2][2][C][C];   /* v rows; then beta v in f16 in place; then U~^T (staging) */
    uint16_t kt[2][C][C];        /* K~ [64 rows][128 dk] in the k tile's layout (staging for one bulk store) */
    float graw[2][C], braw[2][C];
    float a32[4][16][20];        /* the diagonal 16x16 blocks of A, f32 */
    uint16_t l16[C][TP];         /* A, f16 (its off-diagonal blocks are read) */
    uint16_t t16[C][TP];         /* T = (I + A)^-1, f16 */
    struct Meta {
        float G[C], beta[C], gl[4];
    } meta[2];                   /* the slot's meta per buffer, bulk-stored whole */
    uint16_t tmp[3][16][24];     /* per-warp 16x16 staging */
    int32_t r0[kSeqCache], base[kSeqCache + 1];
    uint64_t landed[2];          /* the k and v rows of buffer b have landed */
    int abort, ok, n_cached, claim, claim_next;   /* claim_next: the item after the current one */
};
static_assert(offsetof(PrepSmem, vraw) % 1024 == 0, "TMA 128-byte swizzle destinations");
static_assert(sizeof(PrepSmem::Meta) == kSlotBytes - kSlotMeta && offsetof(PrepSmem, meta) % 16 == 0, "the slot's meta, one bulk store");

/* Chunk `slot` (< the table's base[n]): its first row, length and sequence (when `seq` is given). The
 * sequence is the largest i with base[i] <= slot, searched in the first n_cached rows of the table
 * (r0c, basec: shared-memory copies) when the slot lies there, else in the table. */
__device__ void locate_chunk(const GdnPlan& p, const int32_t* r0c, const int32_t* basec, int n_cached, int64_t slot,
                             int64_t* row0, int* len, int* seq = nullptr) {
    const int n = (int)p.g.n_seq;
    const int32_t* r0t = p.tab;
    const int32_t* r1t = p.tab + n;
    const int32_t* bt = p.tab + 2 * n;
    int lo, hi, i;
    if (slot < basec[n_cached]) {
        lo = 0;
        hi = n_cached - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (basec[mid] <= slot) lo = mid;
            else hi = mid - 1;
        }
        i = lo;
        *row0 = r0c[i] + (slot - basec[i]) * C;
    } else {
        lo = n_cached;
        hi = n - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (bt[mid] <= slot) lo = mid;
            else hi = mid - 1;
        }
        i = lo;
        *row0 = r0t[i] + (slot - bt[i]) * C;
    }
    *len = (int)min((int64_t)C, (int64_t)r1t[i] - *row0);
    if (seq) *seq = i;
}

/* T[bi][bj] = -T[bi][bi] * sum_{k=bj}^{bi-1} L[bi][k] T[k][bj] for one 16x16 block, one warp (s: any shared
 * layout with the f16 tiles l16, t16 of pitch TP and per-warp staging tmp). */
template <class Smem>
__device__ void tri_offdiag_block(Smem& s, int bi, int bj, int w) {
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

/* Item i = (chunk slot, v-head) by item_at: start its k and v rows (two TMA boxes of [64 rows][64] each, rows
 * past the end read as zero) completing on landed[buf], and g, beta (cp.async; zero past the chunk). */
__device__ void prep_issue(const GdnPlan& p, const CUtensorMap* kmap, const CUtensorMap* vmap, PrepSmem& s, int64_t item,
                           int64_t slots, int buf, int tid) {
    const RidgeFillGdn& g = p.g;
    int64_t slot, h;
    item_at(p, item, slots, &slot, &h);
    const int64_t hk = h / (g.n_head_v / g.n_head_k);
    int64_t row0 = 0;
    int len = 0;
    locate_chunk(p, s.r0, s.base, s.n_cached, slot, &row0, &len);
    if (tid == kStoreTid) {
        rf::mbar_arrive_expect_tx(&s.landed[buf], 2 * kTileBytes);
        rf::tma_load_3d(&s.kraw[buf][0][0][0], kmap, &s.landed[buf], 0, (int)hk, (int)row0);
        rf::tma_load_3d(&s.kraw[buf][1][0][0], kmap, &s.landed[buf], C, (int)hk, (int)row0);
        rf::tma_load_3d(&s.vraw[buf][0][0][0], vmap, &s.landed[buf], 0, (int)h, (int)row0);
        rf::tma_load_3d(&s.vraw[buf][1][0][0], vmap, &s.landed[buf], C, (int)h, (int)row0);
    }
    if (tid < C) {
        const int r = tid;
        const int64_t row = row0 + (r < len ? r : 0);
        cp_async4(&s.graw[buf][r], g.g + row * g.g_row + h, r < len ? 4 : 0);
        cp_async4(&s.braw[buf][r], g.beta + row * g.b_row + h, r < len ? 4 : 0);
    }
}

/* The slot of flag `it` (chunk slot x Hv + v-head) is complete: its bulk stores (K~, then W, U~^T and the meta)
 * have completed (the caller waited for them); made visible at GPU scope, then flagged. One thread. */
__device__ void publish_item(const GdnPlan& p, int64_t it) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __threadfence();
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p.flags + it), "r"(1) : "memory");
}

/* Phase 1 for one group of 8 warps (thread `tid` of 256, named barrier `bar`): items claimed in increasing
 * order from the global counter, each slot flagged once it is written. It never waits on phase 2. */
__device__ void prep_role(const CUtensorMap& kmap, const CUtensorMap& vmap, const GdnPlan& p, PrepSmem& s, const int tid,
                          const int bar) {
    const RidgeFillGdn& g = p.g;
    const int w = tid >> 5, l = tid & 31, gq = l >> 2, tq = l & 3;
    auto sync = [&]() { rf::bar_sync(bar, kPrepThreads); };
    const int n_seq = (int)g.n_seq;
    const int n_cached = n_seq < kSeqCache ? n_seq : kSeqCache;
    for (int i = tid; i <= n_cached; i += kPrepThreads) {
        if (i < n_cached) s.r0[i] = p.tab[i];
        s.base[i] = p.tab[2 * n_seq + i];
    }
    if (tid == 0) {
        rf::mbar_init(&s.landed[0], 1);
        rf::mbar_init(&s.landed[1], 1);
        s.abort = 0;
        s.n_cached = n_cached;
        rf::mbar_init_fence();
        rf::tma_prefetch_map(&kmap);
        rf::tma_prefetch_map(&vmap);
        s.claim = atomicAdd(&p.ctl->next_item, 1);
        s.claim_next = atomicAdd(&p.ctl->next_item, 1);
    }
    sync();
    const int64_t slots = p.tab[3 * n_seq], items = slots * g.n_head_v;
    int64_t item = s.claim;

    if (item < items) prep_issue(p, &kmap, &vmap, s, item, slots, 0, tid);
    rf::cp_async_commit();
    int buf = 0;
    int64_t waited = 0, issued = item < items ? 1 : 0;
    int64_t pending = -1;   /* kStoreTid: the flag (slot x Hv + head) of the item whose slot stores are issued but
                               not yet published */
    int claim = 0;          /* kStoreTid: the item after the next one, claimed during this item */
    while (item < items) {
        rf::cp_async_wait<0>();
        if (tid == 0) s.ok = rf::mbar_wait(&s.landed[buf], (uint32_t)((waited >> 1) & 1), &s.abort, rf::kErrGdnWait);
        sync();
        if (!s.ok) break;
        const int64_t next = s.claim_next;   /* claimed an item ago (the counter's latency stays off the path) */
        ++waited;
        int64_t slot, h;
        item_at(p, item, slots, &slot, &h);
        int64_t row0 = 0;
        int len = 0;
        locate_chunk(p, s.r0, s.base, s.n_cached, slot, &row0, &len);
        uint8_t* out = slot_ptr(p, slot, h);
        const uint32_t ktile = rf::saddr(&s.kraw[buf][0][0][0]), vtile = rf::saddr(&s.vraw[buf][0][0][0]);

        /* G (inclusive cumulative log decay; zero past the chunk) by warp 0, two rows a lane; beta; gamma_L. */
        PrepSmem::Meta& mt = s.meta[buf];
        if (w == 0) {
            const float2 gg = *(const float2*)&s.graw[buf][2 * l];
            const float pair = gg.x + gg.y;
            float x = pair;
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, x, o);
                if (l >= o) x += y;
            }
            *(float2*)&mt.G[2 * l] = make_float2(x - pair + gg.x, x);
        } else if (w == 1) {
            *(float2*)&mt.beta[2 * l] = *(const float2*)&s.braw[buf][2 * l];
        }
        sync();
        const float gl = mt.G[len - 1];
        if (tid < 4) mt.gl[tid] = tid == 0 ? __expf(gl) : 0.0f;
        const float* G = mt.G;
        const float* beta = mt.beta;

        /* K K^T (bf16, exact inputs) and A: warp w, rows 16 (w & 3), columns 32 (w >> 2)..+32 (warps 4, 5
         * hold only blocks above the diagonal, which A does not use). */
        if (w != 4 && w != 5) {
            const int rb = 16 * (w & 3), cb = 32 * (w >> 2);
            float acc[4][4] = {};
            uint32_t fa[2][4], fbk[2][2][4];   /* fragments of k-step ks (buffer ks & 1), the next loaded ahead */
            rf::load_a_sw(fa[0], ktile, rb, 0);
            rf::load_b_nk_sw(fbk[0][0], ktile, cb, 0);
            rf::load_b_nk_sw(fbk[0][1], ktile, cb + 16, 0);
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
                const int cur = ks & 1, nx = cur ^ 1;
                if (ks + 1 < D / 16) {
                    rf::load_a_sw(fa[nx], ktile, rb, 16 * (ks + 1));
                    rf::load_b_nk_sw(fbk[nx][0], ktile, cb, 16 * (ks + 1));
                    rf::load_b_nk_sw(fbk[nx][1], ktile, cb + 16, 16 * (ks + 1));
                }
#pragma unroll
                for (int pr = 0; pr < 2; ++pr) {
                    rf::mma_bf16(acc[2 * pr], fa[cur], fbk[cur][pr][0], fbk[cur][pr][1]);
                    rf::mma_bf16(acc[2 * pr + 1], fa[cur], fbk[cur][pr][2], fbk[cur][pr][3]);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int i = rb + gq + 8 * hr, j = cb + 8 * nt + 2 * tq;
                    float v[2];
#pragma unroll
                    for (int e = 0; e < 2; ++e)
                        v[e] = (j + e < i && i < len) ? beta[i] * __expf(G[i] - G[j + e]) * acc[nt][2 * hr + e] : 0.0f;
                    *(uint32_t*)&s.l16[i][j] = rf::pack_f16(v[0], v[1]);
                    if ((i >> 4) == (j >> 4)) *(float2*)&s.a32[i >> 4][i & 15][j & 15] = make_float2(v[0], v[1]);
                }
        }
        /* While the other warps form K K^T: the previous item's slot stores are complete, so it is published,
         * the other k / v buffer and the K~ staging are free, and the next item's loads start. */
        if (tid == kStoreTid) {
            rf::bulk_store_wait();
            if (pending >= 0) publish_item(p, pending);
            pending = -1;
            claim = atomicAdd(&p.ctl->next_item, 1);   /* its result is first needed at the item's end */
        }
        if (next < items) {
            prep_issue(p, &kmap, &vmap, s, next, slots, buf ^ 1, tid);
            ++issued;
        }
        rf::cp_async_commit();
        sync();

        /* In place, 16-byte chunks at their swizzled places: k -> x1 = beta gamma k (f16); v -> x2 = beta v
         * (f16); and K~ = k exp(G_L - G) (f16) into the staging tile, in the k tile's own layout (the chain
         * reads it as an MN-major operand). Lane l of warp w holds row 32 (w & 1) + l. Rows past the chunk
         * zero. The blocks of T above the diagonal zero. */
        {
            const int r = 32 * (w & 1) + l;
            const bool in = r < len;
            const float gr = G[r], br = beta[r];
            const float fk = in ? __expf(gl - gr) : 0.0f, fx = in ? br * __expf(gr) : 0.0f;
            const uint32_t kst = rf::saddr(&s.kt[0][0][0]);
#pragma unroll
            for (int it = 0; it < 4; ++it) {
                const int seg = (w >> 1) + 4 * it;
                const uint32_t off = rf::sw128_off(r, seg * 8);
                const uint4 kr = lds128(ktile + off), vr = lds128(vtile + off);
                sts128(kst + off, scale_bf16x8_to_f16(kr, fk, in));
                sts128(ktile + off, scale_bf16x8_to_f16(kr, fx, in));
                sts128(vtile + off, scale_bf16x8_to_f16(vr, br, in));
            }
        }
        for (int i = tid; i < 6 * 16 * 8; i += kPrepThreads) {   /* blocks (0,1) (0,2) (0,3) (1,2) (1,3) (2,3) */
            const int blk = i >> 7, r = (i >> 3) & 15, cp = i & 7;
            const int bi = blk < 3 ? 0 : blk < 5 ? 1 : 2, bj = blk < 3 ? blk + 1 : blk < 5 ? blk - 1 : 3;
            *(uint32_t*)&s.t16[16 * bi + r][16 * bj + 2 * cp] = 0u;
        }
        rf::fence_proxy_async_smem();   /* K~ staged by every thread, for the bulk store */
        sync();
        if (tid == kStoreTid) {
            rf::bulk_store(out + kSlotK, &s.kt[0][0][0], kTileBytes);
            rf::bulk_store_commit();
        }

        /* Diagonal blocks of T, by substitution in f32: warp w solves block w >> 1 for columns
         * 8 (w & 1)..+8, lane l holding row l & 15 of 4 columns; row j is final at step j and is
         * broadcast to the rows below it. */
        {
            const int b = w >> 1, r = l & 15, c0 = 8 * (w & 1) + 4 * (l >> 4);
            float a[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 v = *(const float4*)&s.a32[b][r][4 * q];
                a[4 * q] = v.x;
                a[4 * q + 1] = v.y;
                a[4 * q + 2] = v.z;
                a[4 * q + 3] = v.w;
            }
            float x[4];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) x[cc] = r == c0 + cc ? 1.0f : 0.0f;
#pragma unroll
            for (int j = 0; j < 15; ++j)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    const float xj = __shfl_sync(0xffffffffu, x[cc], (l & 16) | j);
                    x[cc] = fmaf(-(j < r ? a[j] : 0.0f), xj, x[cc]);
                }
            *(uint2*)&s.t16[16 * b + r][16 * b + c0] = make_uint2(rf::pack_f16(x[0], x[1]), rf::pack_f16(x[2], x[3]));
        }
        sync();
        if (w < 3) tri_offdiag_block(s, w + 1, w, w);            /* T10, T21, T32 */
        sync();
        if (w < 2) tri_offdiag_block(s, w + 2, w, w);            /* T20, T31 */
        sync();
        if (w == 0) tri_offdiag_block(s, 3, 0, 0);               /* T30 */
        sync();

        /* W = T x1 (warp w: rows 16 (w & 3), dk 64 (w >> 2)..+64), staged over x1 once every warp has
         * read it. */
        {
            const int rb = 16 * (w & 3), cb = 64 * (w >> 2);
            uint32_t ta[4][4];
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) rf::load_a(ta[ks], &s.t16[0][0], TP, rb, 16 * ks);
            float acc[8][4] = {};
            uint32_t fw[2][4][4];   /* B fragments of column pair pr (buffer pr & 1), the next loaded ahead */
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) rf::load_b_kn_sw(fw[0][ks], ktile, 16 * ks, cb);
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                if (pr < 3)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) rf::load_b_kn_sw(fw[(pr + 1) & 1][ks], ktile, 16 * ks, cb + 16 * (pr + 1));
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    rf::mma_f16(acc[2 * pr], ta[ks], fw[pr & 1][ks][0], fw[pr & 1][ks][1]);
                    rf::mma_f16(acc[2 * pr + 1], ta[ks], fw[pr & 1][ks][2], fw[pr & 1][ks][3]);
                }
            }
            sync();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = cb + 8 * j + 2 * tq;
                sts32(ktile + rf::sw128_off(rb + gq, c), rf::pack_f16(acc[j][0], acc[j][1]));
                sts32(ktile + rf::sw128_off(rb + gq + 8, c), rf::pack_f16(acc[j][2], acc[j][3]));
            }
        }
        /* U~^T = x2^T T^T (warp w: dv rows 16 w..+16, all 64 chunk rows), staged over x2 the same way. */
        {
            float acc[8][4] = {};
            uint32_t fa[2][4], fu[2][4][4];   /* fragments of k-step ks (buffer ks & 1), the next loaded ahead */
            rf::load_a_t_sw(fa[0], vtile, 0, 16 * w);
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) rf::load_b_nk(fu[0][pr], &s.t16[0][0], TP, 16 * pr, 0);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const int cur = ks & 1, nx = cur ^ 1;
                if (ks < 3) {
                    rf::load_a_t_sw(fa[nx], vtile, 16 * (ks + 1), 16 * w);
#pragma unroll
                    for (int pr = 0; pr < 4; ++pr) rf::load_b_nk(fu[nx][pr], &s.t16[0][0], TP, 16 * pr, 16 * (ks + 1));
                }
#pragma unroll
                for (int pr = 0; pr < 4; ++pr) {
                    rf::mma_f16(acc[2 * pr], fa[cur], fu[cur][pr][0], fu[cur][pr][1]);
                    rf::mma_f16(acc[2 * pr + 1], fa[cur], fu[cur][pr][2], fu[cur][pr][3]);
                }
            }
            sync();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = 8 * j + 2 * tq;
                sts32(vtile + rf::sw128_off(16 * w + gq, c, 0), rf::pack_f16(acc[j][0], acc[j][1]));
                sts32(vtile + rf::sw128_off(16 * w + gq + 8, c, 0), rf::pack_f16(acc[j][2], acc[j][3]));
            }
        }
        rf::fence_proxy_async_smem();
        sync();
        if (tid == kStoreTid) {   /* W, U~^T and G|beta|gamma_L to the slot; published during the next item */
            rf::bulk_store(out + kSlotW, &s.kraw[buf][0][0][0], kTileBytes);
            rf::bulk_store(out + kSlotU, &s.vraw[buf][0][0][0], kTileBytes);
            rf::bulk_store(out + kSlotMeta, &mt, sizeof(mt));
            rf::bulk_store_commit();
            pending = slot * g.n_head_v + h;
            s.claim_next = claim;   /* read after the next item's first barrier */
        }
        item = next;
        buf ^= 1;
    }
    rf::cp_async_wait<0>();
    if (tid == kStoreTid) {
        rf::bulk_store_wait();
        if (pending >= 0 && s.ok) publish_item(p, pending);
        /* After a timed-out wait: let the copies already issued land before the CTA's shared memory is
         * released (bounded too). */
        for (int64_t i = waited; i < issued; ++i) {
            const uint64_t t0 = rf::global_ns();
            while (!rf::mbar_try_wait(&s.landed[i & 1], (uint32_t)((i >> 1) & 1)) && rf::global_ns() - t0 < rf::kWaitTimeoutNs) {
            }
        }
    }
}

__global__ void __launch_bounds__(kPrepThreads, 2)
gdn_prep_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const GdnPlan p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    prep_role(kmap, vmap, p, *(PrepSmem*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023), threadIdx.x, 1);
}

/* ------------------------------------------------------------------ phase 2 */

constexpr int kChainThreads = 160;   /* warps 0-3: the chain; warp 4: the loader */

struct Stage {                       /* one chunk's inputs, three bulk copies from its slot */
    uint16_t w[2][C][C];             /* W, swizzled */
    uint16_t kt[2][C][C];            /* K~, swizzled */
    uint16_t u[VS][C];               /* U~^T for this CTA's 32 dv rows, swizzled */
    float gl[32];                    /* gamma_L (first word) */
};

struct ChainSmem {
    Stage st[kStages];
    float part[2][4][16][PP];        /* the chain warps' partial V'^T, double-buffered */
    uint64_t landed[kStages], consumed[kStages];
    int abort, ok_chain;
};
static_assert(sizeof(Stage) % 128 == 0, "stage layout");

__global__ void __launch_bounds__(kChainThreads, 1) gdn_chain_kernel(const GdnPlan p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    ChainSmem& s = *(ChainSmem*)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
    const RidgeFillGdn& g = p.g;
    const int vsl = blockIdx.x;
    const int64_t h = blockIdx.y, seq = blockIdx.z;
    const int64_t state_slot = g.state_idx[seq * g.idx_pitch];
    if (state_slot < 0 || state_slot >= g.n_states) return;
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31, gq = l >> 2, tq = l & 3;
    const int v0 = vsl * VS;

    /* This sequence's rows and first chunk slot. Chunks past max_slots (only overlapping sequences
     * number that many) are not read. */
    const int n = (int)g.n_seq;
    const int64_t r0 = p.tab[seq], r1 = p.tab[n + seq], base = p.tab[2 * n + seq];
    const int64_t chunks = max((int64_t)0, min((r1 - r0 + C - 1) / C, (int64_t)p.max_slots - base));

    if (tid == 0) {
        for (int b = 0; b < kStages; ++b) {
            rf::mbar_init(&s.landed[b], 1);
            rf::mbar_init(&s.consumed[b], 4);
        }
        s.abort = 0;
        rf::mbar_init_fence();
    }
    __syncthreads();

    if (w == 4) {
        /* ------------------------------------------------------------ the loader (one lane) */
        if (l != 0) return;
        int64_t issued = 0;
        for (int64_t c = 0; c < chunks; ++c) {
            const int st = (int)(c % kStages);
            if (c >= kStages && !rf::mbar_wait(&s.consumed[st], (uint32_t)((c / kStages - 1) & 1), &s.abort, rf::kErrGdnWait))
                break;
            const uint8_t* src = slot_ptr(p, base + c, h);
            Stage& sg = s.st[st];
            rf::mbar_arrive_expect_tx(&s.landed[st], 2 * kTileBytes + (uint32_t)sizeof(sg.u) + 16);
            rf::bulk_load(&sg.w[0][0][0], src + kSlotW, 2 * kTileBytes, &s.landed[st]);
            rf::bulk_load(&sg.u[0][0], src + kSlotU + vsl * (int)sizeof(sg.u), sizeof(sg.u), &s.landed[st]);
            rf::bulk_load(&sg.gl[0], src + kSlotGl, 16, &s.landed[st]);
            ++issued;
        }
        /* Before the CTA's shared memory is released: the copies of the last stages have landed (only the
         * most recent copy of a stage can still be in flight; bounded). */
        for (int64_t i = issued > kStages ? issued - kStages : 0; i < issued; ++i) {
            const uint64_t t0 = rf::global_ns();
            while (!rf::mbar_try_wait(&s.landed[i % kStages], (uint32_t)((i / kStages) & 1)) &&
                   rf::global_ns() - t0 < rf::kWaitTimeoutNs) {
            }
        }
        return;
    }

    /* -------------------------------------------------------------- the chain */
    const int vh = w & 1, kh = w >> 1;
    /* The state slice: S[v0 + 16 vh + m][64 kh + n] as C tiles over dk (8 tiles of 8 columns). */
    float S[8][4];
    float* stp = g.state + state_slot * g.st_slot + h * g.st_head;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int v = v0 + 16 * vh + gq + 8 * hr, k = 64 * kh + 8 * j + 2 * tq;
            const float2 x = *(const float2*)(stp + (int64_t)v * D + k);
            S[j][2 * hr] = x.x;
            S[j][2 * hr + 1] = x.y;
        }
    bool ok = true;
    for (int64_t c = 0; c < chunks; ++c) {
        const int st = (int)(c % kStages), b = (int)(c & 1);
        if (tid == 0) s.ok_chain = rf::mbar_wait(&s.landed[st], (uint32_t)((c / kStages) & 1), &s.abort, rf::kErrGdnWait);
        rf::bar_sync(kBarChain, 128);
        if (!(ok = s.ok_chain)) break;
        const Stage& sg = s.st[st];
        const uint32_t wtile = rf::saddr(&sg.w[0][0][0]), kttile = rf::saddr(&sg.kt[0][0][0]), utile = rf::saddr(&sg.u[0][0]);
        uint8_t* ow = p.outws ? out_ptr(p, base + c, h) : nullptr;

        /* V'^T partial over this warp's dk half: [16 dv rows] x [64 chunk rows] = S W^T. */
        float pv[8][4] = {};
        uint32_t fb[2][4][4];   /* B fragments of k-step ks (buffer ks & 1), the next step's loaded ahead */
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) rf::load_b_nk_sw(fb[0][pr], wtile, 16 * pr, 64 * kh);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            if (ks < 3)
#pragma unroll
                for (int pr = 0; pr < 4; ++pr) rf::load_b_nk_sw(fb[(ks + 1) & 1][pr], wtile, 16 * pr, 64 * kh + 16 * (ks + 1));
            uint32_t a[4];
            rf::c_to_a(a, S[2 * ks], S[2 * ks + 1]);
            if (ow) {   /* output form: S0 in f16, this warp's quarter */
                uint16_t* s0 = (uint16_t*)(ow + kOutS0);
                const int vr = v0 + 16 * vh + gq, kc = 64 * kh + 16 * ks + 2 * tq;
                *(uint32_t*)&s0[vr * SP + kc] = a[0];
                *(uint32_t*)&s0[(vr + 8) * SP + kc] = a[1];
                *(uint32_t*)&s0[vr * SP + kc + 8] = a[2];
                *(uint32_t*)&s0[(vr + 8) * SP + kc + 8] = a[3];
            }
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                rf::mma_f16(pv[2 * pr], a, fb[ks & 1][pr][0], fb[ks & 1][pr][1]);
                rf::mma_f16(pv[2 * pr + 1], a, fb[ks & 1][pr][2], fb[ks & 1][pr][3]);
            }
        }
        /* K~'s first k-step, ahead of the exchange (K~ [rows][dk]: B[k = row][n = dk], transposing loads). */
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) rf::load_b_kn_sw(fb[0][pr], kttile, 0, 64 * kh + 16 * pr);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            *(float2*)&s.part[b][w][gq][8 * j + 2 * tq] = make_float2(pv[j][0], pv[j][1]);
            *(float2*)&s.part[b][w][gq + 8][8 * j + 2 * tq] = make_float2(pv[j][2], pv[j][3]);
        }
        rf::bar_sync(kBarPair0 + vh, 64);
        const float gamma_l = sg.gl[0];
        /* V' = U~ - (both halves of S W^T). */
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                const int m = gq + 8 * hr, nn = 8 * j + 2 * tq;
                const uint32_t uw = lds32(utile + rf::sw128_off(16 * vh + m, nn, 0));
                const float2 uf = __half22float2(*(const __half2*)&uw);
                const float2 pt = *(const float2*)&s.part[b][w ^ 2][m][nn];
                pv[j][2 * hr] = uf.x - (pv[j][2 * hr] + pt.x);
                pv[j][2 * hr + 1] = uf.y - (pv[j][2 * hr + 1] + pt.y);
            }

        /* S <- gamma_L S + V'^T K~ over this warp's dk half. */
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) S[j][e] *= gamma_l;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            if (ks < 3)
#pragma unroll
                for (int pr = 0; pr < 4; ++pr) rf::load_b_kn_sw(fb[(ks + 1) & 1][pr], kttile, 16 * (ks + 1), 64 * kh + 16 * pr);
            uint32_t a[4];
            rf::c_to_a(a, pv[2 * ks], pv[2 * ks + 1]);
            if (ow && (ks >> 1) == kh) {   /* output form: U^T in f16 (the two dk halves hold the same V') */
                uint16_t* ut = (uint16_t*)(ow + kOutU);
                const int vr = v0 + 16 * vh + gq, rc = 16 * ks + 2 * tq;
                *(uint32_t*)&ut[vr * TP + rc] = a[0];
                *(uint32_t*)&ut[(vr + 8) * TP + rc] = a[1];
                *(uint32_t*)&ut[vr * TP + rc + 8] = a[2];
                *(uint32_t*)&ut[(vr + 8) * TP + rc + 8] = a[3];
            }
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                rf::mma_f16(S[2 * pr], a, fb[ks & 1][pr][0], fb[ks & 1][pr][1]);
                rf::mma_f16(S[2 * pr + 1], a, fb[ks & 1][pr][2], fb[ks & 1][pr][3]);
            }
        }
        __syncwarp();
        if (l == 0) rf::mbar_arrive(&s.consumed[st]);
    }
    if (!ok) return;   /* a hand-over timed out (recorded in ridgefill_device_error): leave the state as it was */
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int v = v0 + 16 * vh + gq + 8 * hr, k = 64 * kh + 8 * j + 2 * tq;
            *(float2*)(stp + (int64_t)v * D + k) = make_float2(S[j][2 * hr], S[j][2 * hr + 1]);
        }
}

/* ------------------------------------------------------------------ phase 2 on tensor memory (state-only form) */

/* One CTA per (v-head, sequence): the whole 128 x 128 state in tensor memory, the chunk's two products as
 * tcgen05.mma (kind::f16, f32 accumulation, operands in 128-byte-swizzled shared memory, K~ MN-major):
 *     D1 = S W^T           (M 128 dv, N 64 chunk rows, K 128 dk)      eight K-16 steps
 *     D2 += V'^T K~        (M 128 dv, N 128 dk, K 64 chunk rows)      four K-16 steps, D2 = gamma_L S before
 * Roles, handing over through mbarriers only (every wait bounded):
 *   warps 0-7   tensor-memory lane quarter w & 3 (dv rows 32 (w & 3)..+32), column half w >> 2; a thread is
 *               one dv row: V' = U~ - D1 in f16 (the second product's A), then the next chunk's f16 state
 *               (the first product's A) and gamma_L(next) S back into D2
 *   warp 8      lane 0 keeps three chunks' inputs in flight (bulk copies of the slot's W|K~, U~^T, gamma_L)
 *   warp 9      lane 0 issues the products as their operands are ready */
constexpr int kTcEpi = 8, kTcThreads = 32 * (kTcEpi + 2), kTcStages = 3;
/* Tensor-memory columns: D1 (64), the f16 state A_S (64: two dk a column), D2 (128), V'^T A_V (32). */
constexpr uint32_t kTmemTc = 512, kColD1 = 0, kColAs = 64, kColD2 = 128, kColAv = 256;
/* Instruction descriptors, kind::f16: D f32 (bit 4), A and B f16, both K-major, N >> 3 at bit 17, M >> 4 at 24. */
constexpr uint32_t kIdescPv = (1u << 4) | ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t kIdescUp = (1u << 4) | (1u << 16) /* B MN-major */ | ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

struct TcStage {
    uint16_t w[2][C][C];       /* W [64 rows][128 dk]: two 64-column halves */
    uint16_t kt[2][C][C];      /* K~ [64 rows][128 dk]: two 64-column halves (an MN-major operand) */
    uint16_t u[D][C];          /* U~^T [128 dv][64 rows] */
    float gl[256];             /* gamma_L (first word); the stage padded to 1024 bytes */
};

struct TcSmem {
    TcStage st[kTcStages];
    uint64_t landed[kTcStages], consumed[kTcStages];
    uint64_t d1_full, d2_full;           /* a product completed (tcgen05.commit) */
    uint64_t as_ready, av_ready, d2_ready; /* the lanes wrote A_S / A_V / gamma S into D2 (one arrival a warp) */
    uint32_t tmem;
    int abort;
};
/* the hardware swizzles by shared-memory address bits: every tile starts on 1024 bytes */
static_assert(offsetof(TcSmem, st) % 1024 == 0 && sizeof(TcStage) % 1024 == 0, "tile alignment");

__device__ __forceinline__ int ld_acquire(const int* ptr) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}

/* Wait (bounded) until item `it`'s slot is flagged written, then order the async-proxy reads that follow. */
__device__ bool wait_item(const GdnPlan& p, int64_t it, volatile int* abort) {
    if (ld_acquire(p.flags + it) == 0) {
        const uint64_t t0 = rf::global_ns();
        while (ld_acquire(p.flags + it) == 0) {
            if (*abort) return false;
            if (rf::global_ns() - t0 > rf::kWaitTimeoutNs) {
                *abort = 1;
                atomicCAS(&rf::g_device_error, 0, (int)rf::kErrGdnWait);
                return false;
            }
            __nanosleep(100);
        }
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
    return true;
}

/* The chains first, first + step, ... (chain = v-head + Hv * sequence) on threads 0..kTcThreads-1 of one CTA.
 * Every stage and hand-over index runs on across chains (k: the chunks this CTA has taken so far). */
__device__ void chain_tc_role(const GdnPlan& p, TcSmem& s, int64_t first, int64_t step) {
    const RidgeFillGdn& g = p.g;
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
    const int n = (int)g.n_seq;
    const int64_t n_chains = g.n_head_v * g.n_seq;
    auto role_sync = [&]() { rf::bar_sync(3, kTcThreads); };
    if (tid == 0) {
        for (int b = 0; b < kTcStages; ++b) {
            rf::mbar_init(&s.landed[b], 1);
            rf::mbar_init(&s.consumed[b], 1);
        }
        rf::mbar_init(&s.d1_full, 1);
        rf::mbar_init(&s.d2_full, 1);
        rf::mbar_init(&s.as_ready, kTcEpi);
        rf::mbar_init(&s.av_ready, kTcEpi);
        rf::mbar_init(&s.d2_ready, kTcEpi);
        s.abort = 0;
        rf::mbar_init_fence();
    }
    if (w == 0) rf::tmem_alloc<kTmemTc>(&s.tmem);
    rf::tc_fence_before();
    role_sync();
    rf::tc_fence_after();
    const uint32_t tmem = s.tmem;
    volatile int* abort = &s.abort;
    int64_t k0 = 0;          /* chunks taken by this CTA before the current chain */
    int64_t issued = 0;      /* the loader's copies */
    for (int64_t cid = first; cid < n_chains && !*abort; cid += step) {
        int64_t h, seq;
        chain_at(p, cid, &h, &seq);
        const int64_t state_slot = g.state_idx[seq * g.idx_pitch];
        if (state_slot < 0 || state_slot >= g.n_states) continue;
        const int64_t r0 = p.tab[seq], r1 = p.tab[n + seq], base = p.tab[2 * n + seq];
        const int64_t chunks = max((int64_t)0, min((r1 - r0 + C - 1) / C, (int64_t)p.max_slots - base));
        if (chunks == 0) continue;

        if (w == kTcEpi) {
            /* -------------------------------------------------------- the loader (one lane) */
            if (l == 0) {
                for (int64_t c = 0; c < chunks; ++c) {
                    const int64_t k = k0 + c;
                    const int st = (int)(k % kTcStages);
                    if (k >= kTcStages && !rf::mbar_wait(&s.consumed[st], (uint32_t)((k / kTcStages - 1) & 1), abort, rf::kErrGdnWait))
                        break;
                    if (!wait_item(p, (base + c) * g.n_head_v + h, abort)) break;
                    const uint8_t* src = slot_ptr(p, base + c, h);
                    TcStage& sg = s.st[st];
                    rf::mbar_arrive_expect_tx(&s.landed[st], 3 * kTileBytes + 16);
                    rf::bulk_load(&sg.w[0][0][0], src + kSlotW, 2 * kTileBytes, &s.landed[st]);   /* W and K~ */
                    rf::bulk_load(&sg.u[0][0], src + kSlotU, kTileBytes, &s.landed[st]);
                    rf::bulk_load(&sg.gl[0], src + kSlotGl, 16, &s.landed[st]);
                    ++issued;
                }
            }
        } else if (w == kTcEpi + 1) {
            /* -------------------------------------------------------- the product issuer (one lane) */
            if (l == 0) {
                for (int64_t c = 0; c < chunks; ++c) {
                    const int64_t k = k0 + c;
                    const int st = (int)(k % kTcStages);
                    const uint32_t par = (uint32_t)(k & 1);
                    const uint32_t wt = rf::saddr(&s.st[st].w[0][0][0]), kt = rf::saddr(&s.st[st].kt[0][0][0]);
                    /* D1 = S W^T: the chunk's inputs landed and the lanes wrote this chunk's f16 state */
                    if (!rf::mbar_wait(&s.landed[st], (uint32_t)((k / kTcStages) & 1), abort, rf::kErrGdnWait) ||
                        !rf::mbar_wait(&s.as_ready, par, abort, rf::kErrGdnWait))
                        break;
                    rf::tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        rf::umma_f16_ts(tmem + kColD1, tmem + kColAs + 8 * kk, rf::sw128_kmajor_desc(wt + (kk >> 2) * 8192 + (kk & 3) * 32),
                                        kIdescPv, kk > 0);
                    rf::mma_commit(&s.d1_full);
                    /* D2 += V'^T K~: the lanes wrote V' and put gamma_L S into D2 */
                    if (!rf::mbar_wait(&s.av_ready, par, abort, rf::kErrGdnWait) ||
                        !rf::mbar_wait(&s.d2_ready, par, abort, rf::kErrGdnWait))
                        break;
                    rf::tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        rf::umma_f16_ts(tmem + kColD2, tmem + kColAv + 8 * kk, rf::sw128_mnmajor_desc(kt + kk * 2048, 8192), kIdescUp, 1);
                    rf::mma_commit(&s.consumed[st]);   /* the stage is free once these products have read it */
                    rf::mma_commit(&s.d2_full);
                }
            }
        } else {
            /* -------------------------------------------------------- the lanes (warps 0-7) */
            const int q = w & 3, ch = w >> 2, i = 32 * q + l;   /* dv row i; columns of half ch */
            const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
            const uint32_t d1 = lane_base + kColD1 + 32 * ch, d2 = lane_base + kColD2 + 64 * ch;
            const uint32_t as = lane_base + kColAs + 32 * ch, av = lane_base + kColAv + 16 * ch;
            float* srow = g.state + state_slot * g.st_slot + h * g.st_head + (int64_t)i * D + 64 * ch;
            auto arrive = [&](uint64_t* bar) {   /* this warp's writes are done: one arrival a warp */
                __syncwarp();
                if (l == 0) rf::mbar_arrive(bar);
            };
            auto put_as = [&](const uint32_t (&r)[2][32]) {   /* f16 state into the first product's A (tensor memory) */
                uint32_t o[32];
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    o[e] = rf::pack_f16(__uint_as_float(r[e >> 4][(2 * e) & 31]), __uint_as_float(r[e >> 4][(2 * e + 1) & 31]));
                rf::tmem_st32(as, o);
                rf::tmem_st_wait();
                rf::tc_fence_before();
            };
            auto put_d2 = [&](uint32_t (&r)[2][32], float gam) {   /* gamma * S into D2 */
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) r[hf][e] = __float_as_uint(gam * __uint_as_float(r[hf][e]));
                    rf::tmem_st32(d2 + 32 * hf, r[hf]);
                }
                rf::tmem_st_wait();
                rf::tc_fence_before();
            };

            uint32_t r[2][32];
#pragma unroll
            for (int hf = 0; hf < 2; ++hf)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 x = *(const float4*)(srow + 32 * hf + 4 * j);
                    r[hf][4 * j] = __float_as_uint(x.x);
                    r[hf][4 * j + 1] = __float_as_uint(x.y);
                    r[hf][4 * j + 2] = __float_as_uint(x.z);
                    r[hf][4 * j + 3] = __float_as_uint(x.w);
                }
            put_as(r);
            arrive(&s.as_ready);
            bool ok = rf::mbar_wait(&s.landed[k0 % kTcStages], (uint32_t)((k0 / kTcStages) & 1), abort, rf::kErrGdnWait);
            if (ok) {
                put_d2(r, s.st[k0 % kTcStages].gl[0]);
                arrive(&s.d2_ready);
            }
            for (int64_t c = 0; c < chunks && ok; ++c) {
                const int64_t k = k0 + c;
                const uint32_t par = (uint32_t)(k & 1);
                const uint32_t ut = rf::saddr(&s.st[k % kTcStages].u[0][0]);
                /* V' = U~ - D1 for rows 32 ch..+32 of the chunk, f16 into the second product's A */
                if (!(ok = rf::mbar_wait(&s.d1_full, par, abort, rf::kErrGdnWait))) break;
                rf::tc_fence_after();
                {
                    uint32_t d[32], o[16];
                    rf::tmem_ld32(d1, d);
                    rf::tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint4 uu = lds128(ut + rf::sw128_off(i, 32 * ch + 8 * j, 0));
                        const uint32_t uw[4] = { uu.x, uu.y, uu.z, uu.w };
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 uf = __half22float2(*(const __half2*)&uw[e]);
                            o[4 * j + e] = rf::pack_f16(uf.x - __uint_as_float(d[8 * j + 2 * e]), uf.y - __uint_as_float(d[8 * j + 2 * e + 1]));
                        }
                    }
                    rf::tmem_st16(av, o);   /* V'^T, f16, into the second product's A (tensor memory) */
                    rf::tmem_st_wait();
                }
                rf::tc_fence_before();
                arrive(&s.av_ready);
                /* the updated state: the next chunk's f16 state first (its first product waits on it), then
                 * gamma_L(next) S into D2; the final state to memory */
                if (!(ok = rf::mbar_wait(&s.d2_full, par, abort, rf::kErrGdnWait))) break;
                rf::tc_fence_after();
                rf::tmem_ld32(d2, r[0]);
                rf::tmem_ld32(d2 + 32, r[1]);
                rf::tmem_ld_wait();
                if (c + 1 == chunks) {
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            *(float4*)(srow + 32 * hf + 4 * j) = make_float4(__uint_as_float(r[hf][4 * j]), __uint_as_float(r[hf][4 * j + 1]),
                                                                             __uint_as_float(r[hf][4 * j + 2]), __uint_as_float(r[hf][4 * j + 3]));
                    break;
                }
                put_as(r);
                arrive(&s.as_ready);
                const int nst = (int)((k + 1) % kTcStages);
                if (!(ok = rf::mbar_wait(&s.landed[nst], (uint32_t)(((k + 1) / kTcStages) & 1), abort, rf::kErrGdnWait))) break;
                put_d2(r, s.st[nst].gl[0]);
                arrive(&s.d2_ready);
            }
            /* D2's reads of the last chunk precede the next chain's first stores into it (a later barrier) */
            rf::tc_fence_before();
        }
        k0 += chunks;
        role_sync();   /* every role is done with the chain before the next one starts */
    }
    /* the loader's copies still in flight land before the CTA leaves (bounded) */
    if (w == kTcEpi && l == 0)
        for (int64_t i = issued > kTcStages ? issued - kTcStages : 0; i < issued; ++i) {
            const uint64_t t0 = rf::global_ns();
            while (!rf::mbar_try_wait(&s.landed[i % kTcStages], (uint32_t)((i / kTcStages) & 1)) &&
                   rf::global_ns() - t0 < rf::kWaitTimeoutNs) {
            }
        }
    rf::tc_fence_before();
    role_sync();
    if (w == 0) {
        rf::tc_fence_after();
        rf::tmem_free<kTmemTc>(tmem);
    }
}

/* ------------------------------------------------------------------ the state-only fill, one kernel */

/* One CTA per SM, launched cooperatively (all resident): CTAs [0, chain_ctas) run the tensor-memory chains,
 * the others run phase 1 as two independent 8-warp groups. The chains read each chunk's slot once phase 1
 * has flagged it; phase 1 never waits on the chains. */
constexpr int kFusedThreads = 2 * kPrepThreads;
constexpr int kPrepStride = (int)((sizeof(PrepSmem) + 1023) / 1024 * 1024);
constexpr int kFusedSmem = (sizeof(TcSmem) > 2 * (size_t)kPrepStride ? (int)sizeof(TcSmem) : 2 * kPrepStride) + 1024;
static_assert(kTcThreads <= kFusedThreads, "roles fit the block");

__global__ void __launch_bounds__(kFusedThreads, 1)
gdn_fill_fused_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const GdnPlan p,
                      int chain_ctas) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    if ((int)blockIdx.x < chain_ctas) {
        if (threadIdx.x < kTcThreads) chain_tc_role(p, *(TcSmem*)base, blockIdx.x, chain_ctas);
    } else {
        const int grp = threadIdx.x / kPrepThreads;
        prep_role(kmap, vmap, p, *(PrepSmem*)(base + grp * kPrepStride), threadIdx.x % kPrepThreads, 1 + grp);
    }
}

/* ------------------------------------------------------------------ the state-only fill, one CTA a head
 *
 * For launches with many chains (every DeltaNet layer of a pass side by side: hundreds of v-heads), one
 * persistent CTA per SM takes whole chains (v-head, sequence) in turn and runs both phases of each itself, the
 * transform of chunk c + 1 beside the chain's products of chunk c, handing everything over in shared and tensor
 * memory (no workspace, no flags, no cross-CTA waits; a plain launch).
 *
 *   warps 0-7   the transform (lane quarter w & 3, column half w >> 2): G, beta; x2 = beta v and, once K K^T is
 *               in tensor memory, the rows of A (warps 0, 1, 4, 5: rows 32 (w & 1).., columns 32 (w >> 2)..)
 *               beside x1 = beta gamma k and K~ = exp(G_L - G) k (warps 2, 3, 6, 7), all f16 in shared memory;
 *               T = (I + A)^-1 by the blocked inversion of phase 1; T as a K-major operand; then W^T from tensor
 *               memory into the chain's B operand (f16, MN-major [dk][rows]). The transform's steps are short
 *               dependent chains: eight warps (two a sub-partition) hide each other's latencies
 *   warps 8-15  the chain's lanes (quarter w & 3, column half (w - 8) >> 2): V'^T = U~^T - S W^T straight from
 *               tensor memory (U~^T never leaves it), the f16 state, gamma_L S; the final state to memory
 *   warp 16     the loader: k and v rows by TMA, g and beta by cp.async, two chunks in flight
 *   warp 17     lane 0 issues the products (kind::f16, f32 accumulation; K K^T by warp 18):
 *                 K K^T   (M 128 rows of k (the upper 64 unused), N 64, K 128 dk; bf16)    -> tensor memory
 *                 W^T     = x1^T T^T  (M 128 dk, N 64 rows, K 64; A MN-major)               -> tensor memory
 *                 U~^T    = x2^T T^T  (M 128 dv, N 64, K 64; A MN-major)                    -> tensor memory
 *                 D1      = S W^T     (M 128 dv, N 64, K 128; A the f16 state in tensor memory, B MN-major)
 *                 D2     += V'^T K~   (M 128 dv, N 128 dk, K 64; B MN-major; D2 = gamma_L S before)
 *               in the order D1(c), D2(c), W^T(c+1), U~^T(c+1)
 *   warp 18     lane 0 issues each chunk's K K^T as soon as its rows have landed and the transform has read the
 *               previous one (kk_free)
 * Every hand-over is an mbarrier with a bounded wait; no barrier can run two phases ahead of a waiter (each
 * completion needs the waiter's own previous step). */
constexpr int kHdP = 8, kHdC = 8, kHdLoad = kHdP + kHdC, kHdMma = kHdLoad + 1, kHdKkw = kHdMma + 1;
constexpr int kHdThreads = 32 * (kHdKkw + 1);
/* Tensor-memory columns: D1 (64), the f16 state A_S (64), D2 (128), K K^T (64), W^T (64), U~^T (64), V'^T A_V (32). */
constexpr uint32_t kHdD1 = 0, kHdAs = 64, kHdD2 = 128, kHdKk = 256, kHdWt = 320, kHdUt = 384, kHdAv = 448;
constexpr uint32_t kIdescKk = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t kIdescWu = (1u << 4) | (1u << 15) /* A MN-major */ | ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t kIdescD1 = (1u << 4) | (1u << 16) /* B MN-major */ | ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
/* Launches of at least this many chains take this form (fewer chains leave SMs idle; the cooperative form
 * spreads a few chains' transforms over every SM). */
constexpr int64_t kHeadFormChains = 64;

struct HdStage {                 /* one chunk's inputs; x1 and x2 replace k and v in place */
    uint16_t k[2][C][C];
    uint16_t v[2][C][C];
    float g[C], b[C];            /* g and beta (zero past the chunk), by cp.async */
    float G[C], gl[4];           /* the inclusive cumulative log decay and G_L, by the loader */
    uint8_t pad[1024 - 3 * C * 4 - 16];
};
constexpr int kHdStages = 3;     /* chunks of input in flight (the loader two ahead of the transform) */

struct HdSmem {
    HdStage in[kHdStages];
    uint16_t kt[2][2][C][C];     /* K~ [rows][dk] (the k tile's layout), by chunk parity */
    uint16_t wt[2][D][C];        /* W^T [dk][rows], 128-byte swizzled rows, by chunk parity */
    struct Work {                /* one transform group's inversion workspace (group = chunk parity) */
        uint16_t l16[C][TP];     /* A, f16; once T is formed, its first 8 KB hold T [rows][rows] as a 128-byte
                                    swizzled K-major operand (tile()) */
        uint16_t t16[C][TP];     /* T, f16 */
        float a32[4][16][20];    /* A's diagonal blocks, f32 */
        uint16_t tmp[4][16][24];
        __device__ uint16_t* tile() { return &l16[0][0]; }
    } work[2];
    struct Meta {
        float gl[4];             /* gamma_L = exp(G_L) */
    } meta[2];                   /* by chunk parity: the chain's lanes read it after the stage may be reused; the
                                    transform writes chunk q's only after buf_free of chunk q - 2 */
    uint64_t landed[kHdStages], stage_free[kHdStages], buf_free[2];
    uint64_t kk_full, kk_free, t_ready[2], wt_full, ut_full, tsw_free[2], w_ready[2], d1_full, d2_full, as_ready, av_ready,
        d2_ready;
    uint32_t tmem;
    int abort;
};
static_assert(sizeof(HdStage) % 1024 == 0 && offsetof(HdSmem, kt) % 1024 == 0 && offsetof(HdSmem, wt) % 1024 == 0 &&
              offsetof(HdSmem, work) % 1024 == 0 && sizeof(HdSmem::Work) % 1024 == 0, "operand tiles on 1024 bytes");
static_assert(sizeof(HdSmem) + 1024 <= 227 * 1024, "one CTA a SM");
constexpr int kHdSmem = (int)sizeof(HdSmem) + 1024;

struct HdChain {
    int64_t h, seq, slot, r0, r1, chunks;
};

/* Chain `cid` (v-head cid % Hv of sequence cid / Hv): its rows (cu_seqlens clamped into [0, T]) and state slot;
 * chunks 0 when the slot lies outside the pool or the sequence is empty (the chain is skipped). */
__device__ HdChain hd_chain(const RidgeFillGdn& g, int64_t cid) {
    HdChain c;
    c.h = cid % g.n_head_v;
    c.seq = cid / g.n_head_v;
    c.r0 = min(max((int64_t)g.cu[c.seq], (int64_t)0), g.T);
    c.r1 = min(max((int64_t)g.cu[c.seq + 1], c.r0), g.T);
    c.slot = g.state_idx[c.seq * g.idx_pitch];
    c.chunks = (c.slot < 0 || c.slot >= g.n_states) ? 0 : (c.r1 - c.r0 + C - 1) / C;
    return c;
}

__global__ void __launch_bounds__(kHdThreads, 1)
gdn_fill_heads_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const RidgeFillGdn g) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    HdSmem& s = *(HdSmem*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
    const int64_t n_chains = g.n_head_v * g.n_seq;
    volatile int* abort = &s.abort;
    if (tid == 0) {
        for (int b = 0; b < kHdStages; ++b) {
            rf::mbar_init(&s.landed[b], 1 + 32);   /* the TMA bytes' arrival and the loader's 32 lanes */
            rf::mbar_init(&s.stage_free[b], 1);
        }
        for (int b = 0; b < 2; ++b) rf::mbar_init(&s.buf_free[b], 1);
        rf::mbar_init(&s.kk_full, 1);
        rf::mbar_init(&s.kk_free, 2);   /* the two warps of a group that read K K^T's rows */
        rf::mbar_init(&s.wt_full, 1);
        rf::mbar_init(&s.ut_full, 1);
        for (int b = 0; b < 2; ++b) {
            rf::mbar_init(&s.tsw_free[b], 1);
            rf::mbar_init(&s.t_ready[b], kHdP / 2);   /* one arrival a warp of the chunk's group */
            rf::mbar_init(&s.w_ready[b], kHdP / 2);
        }
        rf::mbar_init(&s.d1_full, 1);
        rf::mbar_init(&s.d2_full, 1);
        rf::mbar_init(&s.as_ready, kHdC);
        rf::mbar_init(&s.av_ready, kHdC);
        rf::mbar_init(&s.d2_ready, kHdC);
        s.abort = 0;
        rf::mbar_init_fence();
    }
    if (w == kHdMma) rf::tmem_alloc<512>(&s.tmem);
    /* T's blocks above the diagonal stay zero (nothing writes them) */
    for (int i = tid; i < 2 * C * TP / 2; i += kHdThreads) ((uint32_t*)&s.work[i / (C * TP / 2)].t16[0][0])[i % (C * TP / 2)] = 0u;
    rf::tc_fence_before();
    __syncthreads();
    rf::tc_fence_after();
    const uint32_t tmem = s.tmem;
    /* every role walks the same chains and numbers their chunks q = 0, 1, ... across them */
    int64_t total = 0;
    for (int64_t cid = blockIdx.x; cid < n_chains; cid += gridDim.x) total += hd_chain(g, cid).chunks;

    if (w == kHdLoad) {
        /* ------------------------------------------------------------ the loader (whole warp) */
        int64_t q = 0;
        bool ok = true;
        for (int64_t cid = blockIdx.x; cid < n_chains && ok; cid += gridDim.x) {
            const HdChain ch = hd_chain(g, cid);
            const int64_t hk = ch.h / (g.n_head_v / g.n_head_k);
            for (int64_t j = 0; j < ch.chunks; ++j, ++q) {
                const int st = (int)(q % kHdStages);
                if (q >= kHdStages)
                    ok = rf::mbar_wait(&s.stage_free[st], (uint32_t)((q / kHdStages - 1) & 1), abort, rf::kErrGdnWait);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                const int64_t row0 = ch.r0 + j * C;
                const int len = (int)min((int64_t)C, ch.r1 - row0);
                HdStage& sg = s.in[st];
                if (l == 0) {
                    rf::mbar_arrive_expect_tx(&s.landed[st], 2 * kTileBytes);
                    rf::tma_load_3d(&sg.k[0][0][0], &kmap, &s.landed[st], 0, (int)hk, (int)row0);
                    rf::tma_load_3d(&sg.k[1][0][0], &kmap, &s.landed[st], C, (int)hk, (int)row0);
                    rf::tma_load_3d(&sg.v[0][0][0], &vmap, &s.landed[st], 0, (int)ch.h, (int)row0);
                    rf::tma_load_3d(&sg.v[1][0][0], &vmap, &s.landed[st], C, (int)ch.h, (int)row0);
                }
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int r = l + 32 * hf;
                    const int64_t row = row0 + (r < len ? r : 0);
                    cp_async4(&sg.g[r], g.g + row * g.g_row + ch.h, r < len ? 4 : 0);
                    cp_async4(&sg.b[r], g.beta + row * g.b_row + ch.h, r < len ? 4 : 0);
                }
                rf::cp_async_wait_all();
                __syncwarp();   /* every lane's g is in */
                {
                    /* G (inclusive cumulative log decay; zero past the chunk), two rows a lane, and G_L */
                    const float2 gg = *(const float2*)&sg.g[2 * l];
                    const float pair = gg.x + gg.y;
                    float x = pair;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const float y = __shfl_up_sync(0xffffffffu, x, o);
                        if (l >= o) x += y;
                    }
                    *(float2*)&sg.G[2 * l] = make_float2(x - pair + gg.x, x);
                    const float last = __shfl_sync(0xffffffffu, (len - 1) & 1 ? x : x - pair + gg.x, (len - 1) >> 1);
                    if (l == 0) sg.gl[0] = last;
                }
                rf::mbar_arrive(&s.landed[st]);
            }
        }
        /* copies still in flight land before the CTA leaves (bounded) */
        if (l == 0)
            for (int64_t i = q > kHdStages ? q - kHdStages : 0; i < q; ++i) {
                const uint64_t t0 = rf::global_ns();
                while (!rf::mbar_try_wait(&s.landed[i % kHdStages], (uint32_t)((i / kHdStages) & 1)) &&
                       rf::global_ns() - t0 < rf::kWaitTimeoutNs) {
                }
            }
    } else if (w == kHdMma || w == kHdKkw) {
        /* ------------------------------------------------------------ the product issuers: warp 18 K K^T, warp 17 the rest */
        auto kkt = [&](int64_t q) -> bool {   /* K K^T of chunk q */
                const int st = (int)(q % kHdStages);
                if (!rf::mbar_wait(&s.landed[st], (uint32_t)((q / kHdStages) & 1), abort, rf::kErrGdnWait)) return false;
                rf::tc_fence_after();
                const uint32_t kt = rf::saddr(&s.in[st].k[0][0][0]);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t d = rf::sw128_kmajor_desc(kt + (kk >> 2) * 8192 + (kk & 3) * 32);
                    rf::umma_f16(tmem + kHdKk, d, d, kIdescKk, kk > 0);
                }
                rf::mma_commit(&s.kk_full);
                return true;
        };
        if (w == kHdKkw) {
            /* K K^T of each chunk as soon as its rows have landed and the transform has read the previous one's rows
             * (kk_free), so it is ready long before the transform needs it. A warp of its own: a lane of the issuer's
             * warp spinning beside lane 0 would wait its turn behind lane 0's waits */
            if (l == 0)
                for (int64_t q = 0; q < total; ++q) {
                    if (q >= 1 && !rf::mbar_wait(&s.kk_free, (uint32_t)((q - 1) & 1), abort, rf::kErrGdnWait)) break;
                    if (!kkt(q)) break;
                }
        } else if (l == 0 && total > 0) {
            auto wu = [&](int64_t q) -> bool {   /* W^T and U~^T of chunk q */
                if (!rf::mbar_wait(&s.t_ready[q & 1], (uint32_t)((q >> 1) & 1), abort, rf::kErrGdnWait)) return false;
                rf::tc_fence_after();
                const int st = (int)(q % kHdStages);
                const uint32_t x1 = rf::saddr(&s.in[st].k[0][0][0]), x2 = rf::saddr(&s.in[st].v[0][0][0]);
                const uint32_t tt = rf::saddr(s.work[q & 1].tile());
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    rf::umma_f16(tmem + kHdWt, rf::sw128_mnmajor_desc(x1 + kk * 2048, 8192), rf::sw128_kmajor_desc(tt + kk * 32),
                                 kIdescWu, kk > 0);
                rf::mma_commit(&s.wt_full);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    rf::umma_f16(tmem + kHdUt, rf::sw128_mnmajor_desc(x2 + kk * 2048, 8192), rf::sw128_kmajor_desc(tt + kk * 32),
                                 kIdescWu, kk > 0);
                rf::mma_commit(&s.ut_full);
                rf::mma_commit(&s.stage_free[st]);
                rf::mma_commit(&s.tsw_free[q & 1]);
                return true;
            };
            bool ok = wu(0);
            for (int64_t q = 0; q < total && ok; ++q) {
                const uint32_t par = (uint32_t)(q & 1);
                /* D1 = S W^T: the lanes wrote this chunk's f16 state, the transform its W^T tile */
                if (!(ok = rf::mbar_wait(&s.as_ready, par, abort, rf::kErrGdnWait) &&
                           rf::mbar_wait(&s.w_ready[par], (uint32_t)((q >> 1) & 1), abort, rf::kErrGdnWait)))
                    break;
                rf::tc_fence_after();
                const uint32_t wt = rf::saddr(&s.wt[par][0][0]);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    rf::umma_f16_ts(tmem + kHdD1, tmem + kHdAs + 8 * kk, rf::sw128_mnmajor_desc(wt + kk * 2048, 8192), kIdescD1, kk > 0);
                rf::mma_commit(&s.d1_full);
                /* D2 += V'^T K~: the lanes wrote V' and put gamma_L S into D2 */
                if (!(ok = rf::mbar_wait(&s.av_ready, par, abort, rf::kErrGdnWait) &&
                           rf::mbar_wait(&s.d2_ready, par, abort, rf::kErrGdnWait)))
                    break;
                rf::tc_fence_after();
                const uint32_t kt = rf::saddr(&s.kt[par][0][0][0]);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    rf::umma_f16_ts(tmem + kHdD2, tmem + kHdAv + 8 * kk, rf::sw128_mnmajor_desc(kt + kk * 2048, 8192), kIdescUp, 1);
                rf::mma_commit(&s.d2_full);
                rf::mma_commit(&s.buf_free[par]);   /* K~ and W^T of this parity are read */
                if (q + 1 < total) ok = wu(q + 1);
            }
        }
    } else if (w < kHdP) {
        /* ------------------------------------------------------------ the transform (warps 0-7) */
        /* Two groups of four warps, group grp = (w >> 2) taking the chunks of parity grp, so two chunks' transforms
         * are in flight: each is a string of short dependent steps that one chunk alone cannot spread over the SM.
         * Within a group, warp lw = w & 3 is lane quarter lw of the tensor memory. */
        const int grp = w >> 2, lw = w & 3, gt = tid & 127;
        HdSmem::Work& wk = s.work[grp];
        auto psync = [&]() { rf::bar_sync(1 + grp, 128); };
        /* a barrier of the group's four warps that also tells all of them whether any thread's wait gave up */
        auto failed = [&](bool ok) { return rf::bar_any(1 + grp, 128, !ok || *abort); };
        /* W^T of chunk qq (this group's) from tensor memory into its parity's B tile of D1: thread = dk row 32 lw + l,
         * the 64 columns in two halves; true if a wait gave up */
        auto read_back_wt = [&](int64_t qq) -> bool {
            if (failed(rf::mbar_wait(&s.wt_full, (uint32_t)(qq & 1), abort, rf::kErrGdnWait))) return true;
            rf::tc_fence_after();
            const uint32_t wtile = rf::saddr(&s.wt[qq & 1][0][0]);
            const int dk = 32 * lw + l;
#pragma unroll 1
            for (int ch = 0; ch < 2; ++ch) {
                uint32_t wv[32];
                rf::tmem_ld32(tmem + ((uint32_t)(32 * lw) << 16) + kHdWt + 32 * ch, wv);
                rf::tmem_ld_wait();
#pragma unroll
                for (int c8 = 0; c8 < 4; ++c8) {
                    const uint32_t* x = &wv[c8 * 8];
                    sts128(wtile + rf::sw128_off(dk, 8 * (4 * ch + c8)),
                           make_uint4(rf::pack_f16(__uint_as_float(x[0]), __uint_as_float(x[1])),
                                      rf::pack_f16(__uint_as_float(x[2]), __uint_as_float(x[3])),
                                      rf::pack_f16(__uint_as_float(x[4]), __uint_as_float(x[5])),
                                      rf::pack_f16(__uint_as_float(x[6]), __uint_as_float(x[7]))));
                }
            }
            rf::tc_fence_before();
            rf::fence_proxy_async_smem();
            __syncwarp();
            if (l == 0) rf::mbar_arrive(&s.w_ready[grp]);
            return false;
        };
        int64_t q = 0;
        bool stop = false;
        for (int64_t cid = blockIdx.x; cid < n_chains && !stop; cid += gridDim.x) {
            const HdChain ch = hd_chain(g, cid);
            for (int64_t j = 0; j < ch.chunks; ++j, ++q) {
                if ((q & 1) != grp) continue;   /* the other group's chunk */
                const int st = (int)(q % kHdStages), par = grp;
                const int len = (int)min((int64_t)C, ch.r1 - (ch.r0 + j * C));
                HdStage& sg = s.in[st];
                HdSmem::Meta& mt = s.meta[par];
                /* the chunk's k, v, g, beta and (by the loader) G and G_L are in */
                if ((stop = failed(rf::mbar_wait(&s.landed[st], (uint32_t)((q / kHdStages) & 1), abort, rf::kErrGdnWait)))) break;
                const float gl = sg.gl[0];
                const uint32_t ktile = rf::saddr(&sg.k[0][0][0]), vtile = rf::saddr(&sg.v[0][0][0]);
                /* x2 = beta v in place: row gt & 63, column half gt >> 6; four segments' loads before their stores
                 * (the shared-memory helpers keep their order as written) */
                {
                    const int r = gt & 63;
                    const bool in = r < len;
                    const float br = sg.b[r];
#pragma unroll
                    for (int b4 = 0; b4 < 8; b4 += 4) {
                        uint4 raw[4];
                        uint32_t off[4];
#pragma unroll
                        for (int it = 0; it < 4; ++it) {
                            off[it] = rf::sw128_off(r, (8 * (gt >> 6) + b4 + it) * 8);
                            raw[it] = lds128(vtile + off[it]);
                        }
#pragma unroll
                        for (int it = 0; it < 4; ++it) sts128(vtile + off[it], scale_bf16x8_to_f16(raw[it], br, in));
                    }
                }
                /* K K^T landed in tensor memory (so x1 may replace the k tile); this parity's K~ tile free once D2 of
                 * two chunks ago has read it; this group's A / T tile free once W^T and U~^T of its previous chunk
                 * have read T from it */
                bool ok = rf::mbar_wait(&s.kk_full, (uint32_t)(q & 1), abort, rf::kErrGdnWait);
                if (q >= 2) {
                    ok = ok && rf::mbar_wait(&s.buf_free[par], (uint32_t)(((q >> 1) - 1) & 1), abort, rf::kErrGdnWait);
                    ok = ok && rf::mbar_wait(&s.tsw_free[grp], (uint32_t)(((q >> 1) - 1) & 1), abort, rf::kErrGdnWait);
                }
                if ((stop = failed(ok))) break;
                /* gamma_L for the chain's lanes, written only now: they read this parity's value of two chunks ago
                 * before their d2_ready of that chunk, and buf_free (waited above) completes after its D2 */
                if (gt == 0) mt.gl[0] = __expf(gl);
                rf::tc_fence_after();
                if (lw < 2) {
                    /* A's rows: thread = row i (lane quarter lw), its 64 columns from tensor memory, 32 at a time */
                    const int i = 32 * lw + l;
                    const bool rowin = i < len;
                    const float Gi = sg.G[i], bi = sg.b[i];
                    const uint32_t base = tmem + ((uint32_t)(32 * lw) << 16) + kHdKk;
#pragma unroll 1
                    for (int j0 = 0; j0 < C; j0 += 16) {
                        float gv[16];   /* G of the 16 columns, in registers (no load between the stores below) */
#pragma unroll
                        for (int x = 0; x < 4; ++x) *(float4*)&gv[4 * x] = *(const float4*)&sg.G[j0 + 4 * x];
                        uint32_t kk[16];
                        rf::tmem_ld16(base + j0, kk);
                        rf::tmem_ld_wait();
                        if (j0 + 16 == C) {
                            rf::tc_fence_before();
                            __syncwarp();
                            if (l == 0) rf::mbar_arrive(&s.kk_free);   /* the next chunk's K K^T may overwrite it */
                        }
                        uint32_t pk[8];
#pragma unroll
                        for (int jj = 0; jj < 16; jj += 2) {
                            const int jc = j0 + jj;
                            float v[2];
#pragma unroll
                            for (int e = 0; e < 2; ++e)
                                v[e] = (jc + e < i && rowin) ? bi * __expf(Gi - gv[jj + e]) * __uint_as_float(kk[jj + e]) : 0.0f;
                            pk[jj >> 1] = rf::pack_f16(v[0], v[1]);
                            if ((jc >> 4) == (i >> 4)) *(float2*)&wk.a32[i >> 4][i & 15][jc & 15] = make_float2(v[0], v[1]);
                        }
                        *(uint4*)&wk.l16[i][j0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                        *(uint4*)&wk.l16[i][j0 + 8] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                    }
                } else {
                    /* x1 = beta gamma k in place and K~ = exp(G_L - G) k into this parity's tile: thread = row r */
                    const int r = gt - 64;
                    const bool in = r < len;
                    const float gr = sg.G[r], br = sg.b[r];
                    const float fk = in ? __expf(gl - gr) : 0.0f, fx = in ? br * __expf(gr) : 0.0f;
                    const uint32_t kst = rf::saddr(&s.kt[par][0][0][0]);
#pragma unroll 1
                    for (int b4 = 0; b4 < 16; b4 += 4) {   /* four segments' loads before their stores */
                        uint4 kr[4];
                        uint32_t off[4];
#pragma unroll
                        for (int it = 0; it < 4; ++it) {
                            off[it] = rf::sw128_off(r, (b4 + it) * 8);
                            kr[it] = lds128(ktile + off[it]);
                        }
#pragma unroll
                        for (int it = 0; it < 4; ++it) {
                            sts128(kst + off[it], scale_bf16x8_to_f16(kr[it], fk, in));
                            sts128(ktile + off[it], scale_bf16x8_to_f16(kr[it], fx, in));
                        }
                    }
                }
                psync();
                /* diagonal blocks of T by substitution in f32: warp lw block lw, lane l row l & 15 of 8 columns */
                {
                    const int r = l & 15, c0 = 8 * (l >> 4);
                    float a[16];
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const float4 v = *(const float4*)&wk.a32[lw][r][4 * q4];
                        a[4 * q4] = v.x;
                        a[4 * q4 + 1] = v.y;
                        a[4 * q4 + 2] = v.z;
                        a[4 * q4 + 3] = v.w;
                    }
                    float x[8];
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) x[cc] = r == c0 + cc ? 1.0f : 0.0f;
#pragma unroll
                    for (int jj = 0; jj < 15; ++jj)
#pragma unroll
                        for (int cc = 0; cc < 8; ++cc) {
                            const float xj = __shfl_sync(0xffffffffu, x[cc], (l & 16) | jj);
                            x[cc] = fmaf(-(jj < r ? a[jj] : 0.0f), xj, x[cc]);
                        }
                    *(uint4*)&wk.t16[16 * lw + r][16 * lw + c0] = make_uint4(rf::pack_f16(x[0], x[1]), rf::pack_f16(x[2], x[3]),
                                                                             rf::pack_f16(x[4], x[5]), rf::pack_f16(x[6], x[7]));
                }
                psync();
                if (lw < 3) tri_offdiag_block(wk, lw + 1, lw, lw);   /* T10, T21, T32 */
                psync();
                if (lw < 2) tri_offdiag_block(wk, lw + 2, lw, lw);   /* T20, T31 */
                psync();
                if (lw == 0) tri_offdiag_block(wk, 3, 0, 0);         /* T30 */
                psync();
                /* T into its operand tile over A's first 8 KB (A is no longer read) */
                {
                    const uint32_t tt = rf::saddr(wk.tile());
                    const int r = gt >> 1;
                    uint4 v[4];
#pragma unroll
                    for (int c4 = 0; c4 < 4; ++c4) v[c4] = *(const uint4*)&wk.t16[r][8 * (4 * (gt & 1) + c4)];
#pragma unroll
                    for (int c4 = 0; c4 < 4; ++c4) sts128(tt + rf::sw128_off(r, 8 * (4 * (gt & 1) + c4)), v[c4]);
                }
                rf::fence_proxy_async_smem();   /* x1, x2, K~ and T for the tensor cores */
                __syncwarp();
                if (l == 0) rf::mbar_arrive(&s.t_ready[grp]);
                /* W^T (the product issued once t_ready is complete) into its tile */
                if ((stop = read_back_wt(q))) break;
            }
        }
    } else if (w < kHdLoad) {
        /* ------------------------------------------------------------ the chain's lanes (warps 8-15) */
        const int qd = w & 3, hf = (w - kHdP) >> 2, i = 32 * qd + l;   /* dv row i; columns of half hf */
        const uint32_t lane_base = tmem + ((uint32_t)(32 * qd) << 16);
        const uint32_t d1 = lane_base + kHdD1 + 32 * hf, d2 = lane_base + kHdD2 + 64 * hf, ut = lane_base + kHdUt + 32 * hf;
        const uint32_t as = lane_base + kHdAs + 32 * hf, av = lane_base + kHdAv + 16 * hf;
        auto arrive = [&](uint64_t* bar) {   /* this warp's writes are done: one arrival a warp */
            __syncwarp();
            if (l == 0) rf::mbar_arrive(bar);
        };
        /* a wait the whole warp leaves together (its tensor-memory accesses are warp-wide) */
        auto wwait = [&](uint64_t* bar, uint32_t par) {
            return __all_sync(0xffffffffu, rf::mbar_wait(bar, par, abort, rf::kErrGdnWait));
        };
        /* The state row is moved 32 columns at a time (a half of this thread's 64), so no more than 32 of its values
         * are live: into the first product's A as f16, and gamma S back into D2 (D2 is re-read for that: the tensor
         * cores write it again only after this warp's d2_ready). */
        auto as_half = [&](const uint32_t (&r)[32], int h2) {   /* f16 pairs of 32 state values into A_S */
            uint32_t o[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = rf::pack_f16(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
            rf::tmem_st16(as + 16 * h2, o);
        };
        auto load_row = [&](const float* src, uint32_t (&r)[32]) {   /* 32 state values from memory */
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                const float4 x = *(const float4*)(src + 4 * jj);
                r[4 * jj] = __float_as_uint(x.x);
                r[4 * jj + 1] = __float_as_uint(x.y);
                r[4 * jj + 2] = __float_as_uint(x.z);
                r[4 * jj + 3] = __float_as_uint(x.w);
            }
        };
        auto scale_into_d2 = [&](uint32_t (&r)[32], int h2, float gam) {
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(gam * __uint_as_float(r[e]));
            rf::tmem_st32(d2 + 32 * h2, r);
        };
        int64_t q = 0;
        bool ok = true;
        for (int64_t cid = blockIdx.x; cid < n_chains && ok; cid += gridDim.x) {
            const HdChain ch = hd_chain(g, cid);
            if (ch.chunks == 0) continue;
            float* srow = g.state + ch.slot * g.st_slot + ch.h * g.st_head + (int64_t)i * D + 64 * hf;
            /* the chain's start state: f16 into A_S, then (gamma_L of its first chunk known) gamma S into D2 */
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
                uint32_t r[32];
                load_row(srow + 32 * h2, r);
                as_half(r, h2);
            }
            rf::tmem_st_wait();
            rf::tc_fence_before();
            arrive(&s.as_ready);
            if (!(ok = wwait(&s.ut_full, (uint32_t)(q & 1)))) break;
            {
                const float gam = s.meta[q & 1].gl[0];
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    uint32_t r[32];
                    load_row(srow + 32 * h2, r);
                    scale_into_d2(r, h2, gam);
                }
                rf::tmem_st_wait();
                rf::tc_fence_before();
            }
            arrive(&s.d2_ready);
            for (int64_t j = 0; j < ch.chunks && ok; ++j, ++q) {
                const uint32_t par = (uint32_t)(q & 1);
                /* V'^T = U~^T - D1 for rows 32 hf..+32 of the chunk, f16 into the second product's A */
                if (!(ok = wwait(&s.d1_full, par))) break;
                rf::tc_fence_after();
#pragma unroll
                for (int x = 0; x < 2; ++x) {   /* 16 columns at a time: fewer live registers */
                    uint32_t d[16], u[16], o[8];
                    rf::tmem_ld16(d1 + 16 * x, d);
                    rf::tmem_ld16(ut + 16 * x, u);
                    rf::tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        o[e] = rf::pack_f16(__uint_as_float(u[2 * e]) - __uint_as_float(d[2 * e]),
                                            __uint_as_float(u[2 * e + 1]) - __uint_as_float(d[2 * e + 1]));
                    rf::tmem_st8(av + 8 * x, o);
                }
                rf::tmem_st_wait();
                rf::tc_fence_before();
                arrive(&s.av_ready);
                /* the updated state: the next chunk's f16 state first, then gamma_L(next) S into D2; at the chain's
                 * last chunk the state to memory */
                if (!(ok = wwait(&s.d2_full, par))) break;
                rf::tc_fence_after();
                if (j + 1 == ch.chunks) {
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        uint32_t r[32];
                        rf::tmem_ld32(d2 + 32 * h2, r);
                        rf::tmem_ld_wait();
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj)
                            *(float4*)(srow + 32 * h2 + 4 * jj) =
                                make_float4(__uint_as_float(r[4 * jj]), __uint_as_float(r[4 * jj + 1]),
                                            __uint_as_float(r[4 * jj + 2]), __uint_as_float(r[4 * jj + 3]));
                    }
                    rf::tc_fence_before();
                    continue;
                }
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    uint32_t r[32];
                    rf::tmem_ld32(d2 + 32 * h2, r);
                    rf::tmem_ld_wait();
                    as_half(r, h2);
                }
                rf::tmem_st_wait();
                rf::tc_fence_before();
                arrive(&s.as_ready);
                if (!(ok = wwait(&s.ut_full, (uint32_t)((q + 1) & 1)))) break;
                {
                    const float gam = s.meta[(q + 1) & 1].gl[0];
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        uint32_t r[32];
                        rf::tmem_ld32(d2 + 32 * h2, r);
                        rf::tmem_ld_wait();
                        scale_into_d2(r, h2, gam);
                    }
                    rf::tmem_st_wait();
                    rf::tc_fence_before();
                }
                arrive(&s.d2_ready);
            }
        }
    }
    rf::tc_fence_before();
    __syncthreads();
    if (w == kHdMma) {
        rf::tc_fence_after();
        rf::tmem_free<512>(tmem);
    }
}

/* ------------------------------------------------------------------ output (o present) */

/* o_i = scale * S_i q_i over a chunk, from its start state S0 and corrected values U:
 *     S_i = Gamma_i S0 + sum_{j <= i} exp(G_i - G_j) U_j k_j^T,   Gamma_i = exp(G_i)
 * so  O = scale * (diag(Gamma) Q S0^T + ((Q K^T) .* Dm) U),   Dm_ij = exp(G_i - G_j) for j <= i, else 0.
 * Every (chunk, v-head) in parallel, persistent CTAs: q and k rows by TMA (128-byte swizzled), S0, U^T
 * and G from the scratch by bulk copy; Q K^T on bf16 tensor cores, then q in f16 for the f16 products. */
constexpr int kOutThreads = 256;

struct OutSmem {
    uint16_t qraw[2][C][C];      /* q rows: two 128-byte-swizzled halves (then f16 in place) */
    uint16_t kraw[2][C][C];      /* k rows */
    uint16_t s0[D][SP];          /* S0, f16 */
    uint16_t ut[D][TP];          /* U^T, f16 */
    float meta[2 * C];           /* G, beta of the chunk */
    uint16_t pm[C][TP];          /* (Q K^T) .* Dm, f16 */
    int32_t r0[kSeqCache], base[kSeqCache + 1];
    uint64_t landed;
    int abort, ok, n_cached;
};
static_assert(offsetof(OutSmem, s0) % 16 == 0 && offsetof(OutSmem, ut) % 16 == 0 && offsetof(OutSmem, meta) % 16 == 0,
              "bulk destinations");

__global__ void __launch_bounds__(kOutThreads, 2)
gdn_out_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap, const GdnPlan p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    OutSmem& s = *(OutSmem*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const RidgeFillGdn& g = p.g;
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31, gq = l >> 2, tq = l & 3;
    const int n_seq = (int)g.n_seq;
    const int n_cached = n_seq < kSeqCache ? n_seq : kSeqCache;
    for (int i = tid; i <= n_cached; i += kOutThreads) {
        if (i < n_cached) s.r0[i] = p.tab[i];
        s.base[i] = p.tab[2 * n_seq + i];
    }
    if (tid == 0) {
        rf::mbar_init(&s.landed, 1);
        s.abort = 0;
        s.n_cached = n_cached;
        rf::mbar_init_fence();
        rf::tma_prefetch_map(&qmap);
        rf::tma_prefetch_map(&kmap);
    }
    __syncthreads();
    const int64_t items = (int64_t)p.tab[3 * n_seq] * g.n_head_v;
    const uint32_t qtile = rf::saddr(&s.qraw[0][0][0]), ktile = rf::saddr(&s.kraw[0][0][0]);
    int64_t waited = 0, issued = 0;
    for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
        const int64_t slot = item / g.n_head_v, h = item % g.n_head_v, hk = h / (g.n_head_v / g.n_head_k);
        int64_t row0 = 0;
        int len = 0, sq = 0;
        locate_chunk(p, s.r0, s.base, s.n_cached, slot, &row0, &len, &sq);
        const int64_t state_slot = g.state_idx[(int64_t)sq * g.idx_pitch];
        if (state_slot < 0 || state_slot >= g.n_states) continue;   /* a skipped sequence: its o rows are left as they are */
        if (tid == 0) {
            const uint8_t* ow = out_ptr(p, slot, h);
            rf::mbar_arrive_expect_tx(&s.landed, 2 * kTileBytes + (uint32_t)(sizeof(s.s0) + sizeof(s.ut) + sizeof(s.meta)));
            rf::tma_load_3d(&s.qraw[0][0][0], &qmap, &s.landed, 0, (int)hk, (int)row0);
            rf::tma_load_3d(&s.qraw[1][0][0], &qmap, &s.landed, C, (int)hk, (int)row0);
            rf::tma_load_3d(&s.kraw[0][0][0], &kmap, &s.landed, 0, (int)hk, (int)row0);
            rf::tma_load_3d(&s.kraw[1][0][0], &kmap, &s.landed, C, (int)hk, (int)row0);
            rf::bulk_load(&s.s0[0][0], ow + kOutS0, sizeof(s.s0), &s.landed);
            rf::bulk_load(&s.ut[0][0], ow + kOutU, sizeof(s.ut), &s.landed);
            rf::bulk_load(&s.meta[0], slot_ptr(p, slot, h) + kSlotMeta, sizeof(s.meta), &s.landed);
            ++issued;
            s.ok = rf::mbar_wait(&s.landed, (uint32_t)(waited & 1), &s.abort, rf::kErrGdnWait);
        }
        __syncthreads();
        if (!s.ok) break;
        ++waited;
        const float* G = s.meta;

        {   /* (Q K^T) .* Dm (warp w: rows 16 (w & 3), columns 32 (w >> 2)..+32), f16 */
            const int rb = 16 * (w & 3), cb = 32 * (w >> 2);
            float acc[4][4] = {};
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
                uint32_t a[4];
                rf::load_a_sw(a, qtile, rb, 16 * ks);
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
                for (int hr = 0; hr < 2; ++hr) {
                    const int i = rb + gq + 8 * hr, j = cb + 8 * nt + 2 * tq;
                    const float v0 = (j <= i && i < len) ? __expf(G[i] - G[j]) * acc[nt][2 * hr] : 0.0f;
                    const float v1 = (j + 1 <= i && i < len) ? __expf(G[i] - G[j + 1]) * acc[nt][2 * hr + 1] : 0.0f;
                    *(uint32_t*)&s.pm[i][j] = rf::pack_f16(v0, v1);
                }
        }
        __syncthreads();
        /* q to f16 in place (16-byte chunks keep their swizzled places) */
        for (int i = tid; i < C * (D / 8); i += kOutThreads) {
            const int r = i >> 4, seg = i & 15;
            const uint32_t a = rf::sw128_addr(qtile, r, seg * 8);
            uint4 raw;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(raw.x), "=r"(raw.y), "=r"(raw.z), "=r"(raw.w) : "r"(a));
            const uint32_t rw[4] = { raw.x, raw.y, raw.z, raw.w };
            uint32_t hh[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) hh[e] = rf::pack_f16(__uint_as_float(rw[e] << 16), __uint_as_float(rw[e] & 0xffff0000u));
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(hh[0]), "r"(hh[1]), "r"(hh[2]), "r"(hh[3]) : "memory");
        }
        __syncthreads();
        {   /* O = scale * (diag(Gamma) Q S0^T + Pm U) (warp w: rows 16 (w & 3), dv columns 64 (w >> 2)..+64) */
            const int rb = 16 * (w & 3), cb = 64 * (w >> 2);
            float acc[8][4] = {};
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
                uint32_t a[4];
                rf::load_a_sw(a, qtile, rb, 16 * ks);
#pragma unroll
                for (int pr = 0; pr < 4; ++pr) {
                    uint32_t b[4];
                    rf::load_b_nk(b, &s.s0[0][0], SP, cb + 16 * pr, 16 * ks);
                    rf::mma_f16(acc[2 * pr], a, b[0], b[1]);
                    rf::mma_f16(acc[2 * pr + 1], a, b[2], b[3]);
                }
            }
            const float ga = __expf(G[rb + gq]), gb = __expf(G[rb + gq + 8]);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                acc[j][0] *= ga;
                acc[j][1] *= ga;
                acc[j][2] *= gb;
                acc[j][3] *= gb;
            }
#pragma unroll
            for (int ks = 0; ks < C / 16; ++ks) {
                uint32_t a[4];
                rf::load_a(a, &s.pm[0][0], TP, rb, 16 * ks);
#pragma unroll
                for (int pr = 0; pr < 4; ++pr) {
                    uint32_t b[4];
                    rf::load_b_nk(b, &s.ut[0][0], TP, cb + 16 * pr, 16 * ks);
                    rf::mma_f16(acc[2 * pr], a, b[0], b[1]);
                    rf::mma_f16(acc[2 * pr + 1], a, b[2], b[3]);
                }
            }
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                const int i = rb + gq + 8 * hr;
                if (i >= len) continue;
                uint16_t* orow = g.o + (row0 + i) * g.o_row + h * g.o_head + cb + 2 * tq;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    *(uint32_t*)(orow + 8 * j) = rf::pack_bf16(g.scale * acc[j][2 * hr], g.scale * acc[j][2 * hr + 1]);
            }
        }
        __syncthreads();   /* every read of this item's shared memory precedes the next item's loads */
    }
    /* After a timed-out wait: let the copies already issued land before the CTA's shared memory is
     * released (bounded too). */
    if (tid == 0)
        for (int64_t i = waited; i < issued; ++i) {
            const uint64_t t0 = rf::global_ns();
            while (!rf::mbar_try_wait(&s.landed, (uint32_t)(i & 1)) && rf::global_ns() - t0 < rf::kWaitTimeoutNs) {
            }
        }
}

/* ------------------------------------------------------------------ small heads (dk, dv <= 64)

 * The rule row by row, for heads too narrow for the chunked tensor-core form (the reference's CPU mini
 * model has head dims 32): one CTA per (v-head, sequence), thread i < dv holding state row S[i][0..dk) in
 * registers; each row's k (and q) staged in shared memory by the CTA, then per thread
 *     S_i <- exp(g_t) S_i;   S_i <- S_i + beta_t (v_ti - S_i.k_t) k_t;   o_ti = scale * S_i.q_t
 * in f32. Needs no workspace. */
template <int DK>
__global__ void __launch_bounds__(64) gdn_small_kernel(const RidgeFillGdn g) {
    __shared__ float kq[2][DK];
    const int64_t h = blockIdx.x, seq = blockIdx.y;
    const int64_t slot = g.state_idx[seq * g.idx_pitch];
    if (slot < 0 || slot >= g.n_states) return;
    const int64_t a = min(max((int64_t)g.cu[seq], (int64_t)0), g.T);
    const int64_t b = min(max((int64_t)g.cu[seq + 1], a), g.T);
    const int i = threadIdx.x, dk = (int)g.dk;
    const bool mine = i < g.dv;
    const int64_t hk = h / (g.n_head_v / g.n_head_k);
    float* srow = g.state + slot * g.st_slot + h * g.st_head + (int64_t)i * dk;
    float S[DK];
#pragma unroll
    for (int j = 0; j < DK; ++j) S[j] = (mine && j < dk) ? srow[j] : 0.0f;
    for (int64_t t = a; t < b; ++t) {
        __syncthreads();   /* the previous row's k and q are read */
        for (int j = i; j < DK; j += blockDim.x) {
            kq[0][j] = j < dk ? ridgefill_bf16_to_f32(g.k[t * g.k_row + hk * g.k_head + j]) : 0.0f;
            kq[1][j] = (g.o && j < dk) ? ridgefill_bf16_to_f32(g.q[t * g.q_row + hk * g.q_head + j]) : 0.0f;
        }
        __syncthreads();
        if (!mine) continue;
        const float decay = expf(g.g[t * g.g_row + h]), beta = g.beta[t * g.b_row + h];
        float pred = 0.0f;
#pragma unroll
        for (int j = 0; j < DK; ++j) {
            S[j] *= decay;
            pred = fmaf(S[j], kq[0][j], pred);
        }
        const float u = beta * (ridgefill_bf16_to_f32(g.v[t * g.v_row + h * g.v_head + i]) - pred);
        float out = 0.0f;
#pragma unroll
        for (int j = 0; j < DK; ++j) {
            S[j] = fmaf(u, kq[0][j], S[j]);
            out = fmaf(S[j], kq[1][j], out);
        }
        if (g.o) g.o[t * g.o_row + h * g.o_head + i] = rf::f32_to_bf16_bits(g.scale * out);
    }
    if (mine)
#pragma unroll
        for (int j = 0; j < DK; ++j)
            if (j < dk) srow[j] = S[j];
}

int launch_small(const RidgeFillGdn& g, cudaStream_t stream) {
    const dim3 grid((unsigned)g.n_head_v, (unsigned)g.n_seq);
    const unsigned threads = g.dv > 32 ? 64 : 32;
    if (g.dk <= 16) gdn_small_kernel<16><<<grid, threads, 0, stream>>>(g);
    else if (g.dk <= 32) gdn_small_kernel<32><<<grid, threads, 0, stream>>>(g);
    else gdn_small_kernel<64><<<grid, threads, 0, stream>>>(g);
    return rf::launch_status();
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

/* The state-only form with at least kHeadFormChains chains runs one CTA a head and needs no workspace. */
bool head_form(const RidgeFillGdn& g) { return !g.o && g.n_head_v * g.n_seq >= kHeadFormChains; }

}  // namespace

extern "C" int64_t ridgefill_gdn_fill_scratch(const RadArgs* a) {
    RidgeFillGdn g;
    if (ridgefill_gdn_parse(a, &g) != RAD_OK || g.dk != D || head_form(g)) return 0;   /* the per-row and per-head forms need none */
    const int64_t items = max_slots_of(g) * g.n_head_v;
    return table_bytes(g.n_seq) + kCtlBytes + flag_bytes(items) + items * (kSlotBytes + (g.o ? kOutBytes : 0));
}

extern "C" int ridgefill_gdn_fill_device(const RadArgs* a, RadStream s) {
    RidgeFillGdn g;
    const int rc = ridgefill_gdn_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.n_seq == 0 || g.T == 0) return RAD_OK;
    if (g.n_seq > 65535 || g.n_head_v > 65535 || g.T > 0x7fffffffLL) return RAD_E_SHAPE;
    if (g.dk != D) return launch_small(g, rf::as_stream(s));
    /* k and v are read through TMA tensor maps: positive strides below 2^39 elements. */
    const int64_t lim = 1LL << 39;
    if (g.k_row <= 0 || g.k_head <= 0 || g.v_row <= 0 || g.v_head <= 0 || g.k_row >= lim || g.k_head >= lim ||
        g.v_row >= lim || g.v_head >= lim || (g.q && (g.q_row <= 0 || g.q_head <= 0 || g.q_row >= lim || g.q_head >= lim)))
        return RAD_E_STRIDE;
    CUtensorMap kmap, vmap, qmap;
    if (!head_rows_map(&kmap, g.k, g.T, g.n_head_k, g.k_row, g.k_head, C, true) ||
        !head_rows_map(&vmap, g.v, g.T, g.n_head_v, g.v_row, g.v_head, C, true) ||
        (g.q && !head_rows_map(&qmap, g.q, g.T, g.n_head_k, g.q_row, g.q_head, C, true)))
        return RAD_E_DEVICE;
    if (head_form(g)) {
        /* one CTA per SM, each taking whole chains (no workspace, no cross-CTA waits) */
        if (cudaFuncSetAttribute(gdn_fill_heads_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kHdSmem) != cudaSuccess)
            return RAD_E_DEVICE;
        static int resident = -1;   /* CTAs a SM can hold (registers, shared memory): the form needs exactly 1 */
        if (resident < 0 &&
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, gdn_fill_heads_kernel, kHdThreads, kHdSmem) != cudaSuccess)
            return RAD_E_DEVICE;
        if (resident != 1) return RAD_E_DEVICE;
        const int64_t chains = g.n_head_v * g.n_seq;
        const int grid = (int)(chains < rf::sm_count() ? chains : rf::sm_count());
        gdn_fill_heads_kernel<<<grid, kHdThreads, kHdSmem, rf::as_stream(s)>>>(kmap, vmap, g);
        return rf::launch_status();
    }
    const int64_t slots = max_slots_of(g), items = slots * g.n_head_v;
    const int64_t head = table_bytes(g.n_seq) + kCtlBytes + flag_bytes(items);
    const int64_t need = head + items * (kSlotBytes + (g.o ? kOutBytes : 0));
    if (!a->scratch || a->scratch_bytes < need || (uintptr_t)a->scratch % 16) return RAD_E_INVAL;
    if (items > 0x7fffffffLL) return RAD_E_SHAPE;
    GdnPlan p;
    p.g = g;
    uint8_t* ws = (uint8_t*)a->scratch;
    p.tab = (int32_t*)ws;
    p.ctl = (FillCtl*)(ws + table_bytes(g.n_seq));
    p.flags = (int*)(ws + table_bytes(g.n_seq) + kCtlBytes);
    p.slots = ws + head;
    p.outws = g.o ? p.slots + items * (int64_t)kSlotBytes : nullptr;
    p.max_slots = (int)slots;
    p.head_block = (int)g.n_head_v;   /* the output form: slot-major over every head */
    cudaStream_t stream = rf::as_stream(s);
    const int smem1 = (int)sizeof(PrepSmem) + 1024, smem2 = (int)sizeof(ChainSmem) + 128, smem3 = (int)sizeof(OutSmem) + 1024;
    if (cudaFuncSetAttribute(gdn_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1) != cudaSuccess ||
        cudaFuncSetAttribute(gdn_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2) != cudaSuccess ||
        cudaFuncSetAttribute(gdn_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem3) != cudaSuccess)
        return RAD_E_DEVICE;
    gdn_plan_kernel<<<1, kPlanThreads, 0, stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return RAD_E_DEVICE;
    if (!g.o) {
        /* The state-only form: one cooperative kernel, one CTA per SM (all resident); a quarter of them
         * (at most one a chain) run the chains, the rest phase 1. */
        if (cudaFuncSetAttribute(gdn_fill_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFusedSmem) != cudaSuccess)
            return RAD_E_DEVICE;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gdn_fill_fused_kernel, kFusedThreads, kFusedSmem) != cudaSuccess ||
            per_sm < 1)
            return RAD_E_DEVICE;
        const int grid = per_sm * rf::sm_count();
        const int64_t chains = g.n_head_v * g.n_seq;
        int chain_ctas = (int)(chains < grid / 4 ? chains : grid / 4);
        if (chain_ctas < 1) chain_ctas = 1;
        if (chain_ctas >= grid) return RAD_E_DEVICE;
        p.head_block = chain_ctas;   /* phase 1 makes the chunks in the order the chain CTAs read them */
        void* args[] = { (void*)&kmap, (void*)&vmap, (void*)&p, (void*)&chain_ctas };
        if (cudaLaunchCooperativeKernel((const void*)gdn_fill_fused_kernel, dim3((unsigned)grid), dim3(kFusedThreads), args,
                                        kFusedSmem, stream) != cudaSuccess)
            return RAD_E_DEVICE;
        return rf::launch_status();
    }
    /* The output form: phase 1 (its grid sized by the rows alone: the chunk count is on the device, CTAs
     * past it find no item), the register chain, the output kernel. */
    const int64_t grid1 = items < 2LL * rf::sm_count() ? items : 2LL * rf::sm_count();
    gdn_prep_kernel<<<(unsigned)grid1, kPrepThreads, smem1, stream>>>(kmap, vmap, p);
    if (cudaGetLastError() != cudaSuccess) return RAD_E_DEVICE;
    gdn_chain_kernel<<<dim3(D / VS, (unsigned)g.n_head_v, (unsigned)g.n_seq), kChainThreads, smem2, stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return RAD_E_DEVICE;
    gdn_out_kernel<<<(unsigned)grid1, kOutThreads, smem3, stream>>>(qmap, kmap, p);
    return rf::launch_status();
}

namespace {

/* The two waits the fill's kernels block on, each against something nothing completes: an mbarrier phase
 * nobody arrives on (every tensor-core hand-over) and a slot flag nobody sets (a chain waiting for phase 1).
 * Each gives up after its limit, records kErrGdnWait and reports false; status[0], status[1] get the two
 * outcomes (1 = completed). */
__global__ void wait_selftest_kernel(int* flag, int* status) {
    __shared__ uint64_t bar;
    __shared__ int abort;
    if (threadIdx.x == 0) {
        rf::mbar_init(&bar, 1);
        abort = 0;
        rf::mbar_init_fence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        status[0] = rf::mbar_wait(&bar, 0, &abort, rf::kErrGdnWait) ? 1 : 0;
        abort = 0;
        GdnPlan p{};
        p.flags = flag;
        status[1] = wait_item(p, 0, &abort) ? 1 : 0;
    }
}

}  // namespace

/* Failure detection without a fault: see include/ridgefill.h. */
extern "C" int ridgefill_wait_selftest(int* flag, int* status, RadStream s) {
    if (!flag || !status) return RAD_E_INVAL;
    wait_selftest_kernel<<<1, 32, 0, rf::as_stream(s)>>>(flag, status);
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
 * array of kNoAllocScratchBytes (64 MiB), which every GPU that loads the library holds until the
 * process exits. The fill's workspace is 48.5 KiB per 64-row chunk and value head (one chunk more per
 * sequence), plus 52 KiB more per chunk and head when the output o is asked for. So 64 MiB holds a
 * one-sequence 2,048-row call -- the engine's default chunk -- at up to 40 value heads for the state
 * alone, or up to 19 value heads with o; a 4,096-row call at up to 20 (state only). Heads of at most 64
 * dims need no workspace at all. A call that needs more returns RAD_E_SHAPE and launches nothing.
 *
 * The first call on each device resolves the array's device address there (cudaGetSymbolAddress, with
 * that device current), and again whenever the device's current context is not the one it was resolved
 * in (after a cudaDeviceReset the library's module is loaded anew and the array may move); make that first
 * call before any stream capture. No call allocates or frees device memory. Every call shares the one
 * array and the array keeps the last call's contents: nothing in it needs to start at zero (each call
 * writes every byte of the workspace it reads before reading it, in stream order), but two calls that
 * overlap on the GPU -- on different streams, or from different threads, without an ordering between
 * them -- race on it.
 */
namespace {
constexpr int64_t kNoAllocScratchBytes = 64ll << 20;
constexpr int kNoAllocMaxDevices = 64;
}   // namespace

static __device__ __align__(256) uint8_t g_gdn_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mutex;
struct NoAllocEntry {
    void* context;   /* the driver context the address was resolved in */
    void* address;
};
NoAllocEntry g_noalloc[kNoAllocMaxDevices];

/* The current driver context (cuCtxGetCurrent through the runtime's entry-point query); null when there is
 * none yet or the query is unavailable. */
void* current_context() {
    typedef int (*CtxGetCurrent)(void**);
    static CtxGetCurrent fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (CtxGetCurrent)f;
    }
    void* ctx = nullptr;
    return fn && fn(&ctx) == 0 ? ctx : nullptr;
}

/* The array's device address on the current device, resolved on the first call there and again when the
 * device's context changed. */
int noalloc_workspace(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return RAD_E_DEVICE;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoAllocEntry& e = g_noalloc[dev];
    void* ctx = current_context();
    if (!e.address || !ctx || ctx != e.context) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_gdn_noalloc_scratch) != cudaSuccess || !ptr) return RAD_E_DEVICE;
        e.address = ptr;
        e.context = current_context();   /* the resolution above made the context current if there was none */
    }
    *out = e.address;
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
