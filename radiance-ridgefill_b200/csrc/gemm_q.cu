/* gemm_q.cu -- the int8 projector on B200: ridgefill_gemm_nt_q, ridgefill_gemm_nt_q_bias, the DeltaNet block's
 * fused k|v in-projection ridgefill_gdn_in_proj and the activation quantiser ridgefill_quant_act_i8g.
 *
 * The reference forwards this GEMM to radiance libr4d's int8 gemm_nt_q (kernels/forward.cpp:53-57;
 * issue site arch/ridgefill_layer.h:73-80), whose source is not available; its schema
 * (kernels/rows.cpp:72-76, 161-167) and its test's arithmetic comment (tests/kernel_test.cpp:2114-2117:
 * int32 within a 128-K block, f32 fold, one bf16 rounding) are the contract. This library fixes the
 * fold exactly:
 *     acc = 0;  for each K block j in order:  acc = fma(float(dot_j) * a_scale[m, j], b_scale[j, n], acc)
 *     y = bf16(acc);   with a bias: y = bf16(float(y) + bias[n])
 * so the result is reproducible bit for bit by the CPU oracle.
 *
 * Kernel: persistent 2-CTA clusters, one CTA per SM; a pair computes a 256 x 256 output tile with
 * tcgen05.mma.cta_group::2 (each CTA holds 128 rows of A and 128 rows of B, so a CTA's shared memory moves
 * half the operand bytes a one-CTA 128 x 256 tile needs), 128-byte K steps.
 *   warp 0      TMA producer, both CTAs: this CTA's A [128 x 128] and B [128 x 128] int8 tiles, 128-byte
 *               swizzle, 4-stage ring, the bytes completing on the even CTA's barrier
 *   warp 1      tensor-memory allocator (both CTAs) and, in the even CTA, the MMA issuer: kind::i8 M256
 *               N256 K32, four a step, int32 accumulators in each CTA's tensor memory (its 128 rows), two
 *               256-column buffers so a block's MMAs overlap the previous block's fold; its commits release
 *               the stage and hand over the accumulator in both CTAs
 *   warps 2-17  epilogue: each warp owns a 32-lane quarter of the tile rows and a 64-column slice;
 *               it folds each finished K block into f32 registers and, at the tile's end, writes its
 *               32 x 64 bf16 block into its own 128-byte-swizzled staging tile in shared memory and
 *               stores it with a TMA tile store (rows and columns past y's edge are clipped); with a row
 *               selection (the optional rows operand, ridgefill_select's mask) each lane instead stores its
 *               own row's 64 columns straight to y when the row is selected, so the projection lands only
 *               in the approximated rows of the block input and no separate select pass reads it back
 * The in-projection form (ridgefill_gdn_in_proj) runs the same pipeline over row tiles that overlap by three rows:
 * a CTA projects rows [m_c - 3, m_c + 125), so each of its 125 output rows finds the three rows before it (the
 * causal convolution's window) in the CTA's own tile. Its epilogue rounds the projection to bf16 into a row-major
 * tile in shared memory (the staging space), writes each sequence's last three rows to `tail` (what the conv-state
 * update reads), and then, a warp per head and 16 rows and a lane per 4 channels (conv_prep's layout), computes
 * conv_prep's arithmetic on them instruction for instruction, so the bits agree: the width-4 convolution (the rows
 * before a sequence's start from its conv-state slot or zero), SiLU, the L2 norm of each k head, k and v to bf16 --
 * the projection's rows never go to HBM.
 * The bf16 GEMM with N <= 64 (the DeltaNet block's a|b projection) runs M256 N64 pair tiles: the same pipeline,
 * a quarter of the wide tile's MMA work, which at that width would mostly multiply the B tile's zero rows.
 * A K block is `group` columns: 128 for the projector folder's i8*bf16[1x128] encoding, K itself
 * for per-row / per-column scaling (one fold a tile, the int32 accumulation running over all of K).
 */
#include <cudaTypedefs.h>

#include "common.cuh"
#include "mma.cuh"
#include "sm100.cuh"

#include <cuda_bf16.h>

namespace {

constexpr int BM = 128, BM2 = 2 * BM, BN = 256, BK = 128;   /* a CTA's rows, a pair's rows and columns, K bytes a step */
constexpr int kStages = 4;
constexpr int kABytes = BM * BK, kBBytes = (BN / 2) * BK, kStageBytes = kABytes + kBBytes;   /* one CTA's halves */
constexpr uint32_t kTmemCols = 512;
constexpr int kEpiWarps = 16;
constexpr int kWarpCols = BN * 4 / kEpiWarps;         /* columns an epilogue warp owns (of its 32 lanes' rows) */
constexpr int kBoxes = kWarpCols / 64;                /* its [32 rows][64 cols] bf16 store boxes */
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr int kOutBox = 32 * 64 * 2;                  /* one [32 rows][64 cols] bf16 store box */
constexpr int kStageOut = kEpiWarps * kBoxes * kOutBox;        /* the epilogue warps' staging tiles */
constexpr int kScaleSlots = kEpiWarps * 2 * kWarpCols * 4;     /* each epilogue warp's b_scale values of two K blocks */
constexpr int kMetaBytes = 2 * BM * 4;                         /* the in-projection's per-row sequence start and slot */
constexpr int kSmemBytes = kStages * kStageBytes + kStageOut + kScaleSlots + kMetaBytes + 1024 /* alignment slack */ +
                           256 /* barriers */;
constexpr int kConvRows = BM - 3;   /* the in-projection's output rows a CTA: its tile less the 3-row window */
/* The in-projection's epilogue warps: the 16 that fold also convolve; more that only convolve are possible (at 80
 * registers a thread for 4 more) but measured no faster -- the convolution is bound by the SFU's exp and reciprocal. */
constexpr int kConvWarps = kEpiWarps;
constexpr int kEpiBar = 1;          /* named barrier of the 16 epilogue warps */

/* Instruction descriptor of the pair's M256 N256 product: D s32 (bits 4-5 = 2), A and B signed int8 (bits
 * 7-9, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24. */
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM2 >> 4) << 24);

/* kind::f16 with bf16 A and B (bits 7-9, 10-12 = 1), D f32 (bit 4): the bf16 GEMM (ridgefill_gemm_nt_bias), N columns. */
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM2 >> 4) << 24);
}

struct GemmPlan {
    RidgeFillGemmQ g;       /* the int8 form */
    RidgeFillGemmBias gb;   /* the bf16 form */
    RidgeFillInProj c;      /* the in-projection form (g = c.gemm) */
    int n_tiles, tiles, folds, steps_per_fold;
};

/* kBf16 false: the int8 projector (kind::i8, int32 sums folded with the scales); true: the bf16 GEMM of
 * ridgefill_gemm_nt_bias (kind::f16 with bf16 operands, f32 sums, one fold). The same tiles, the same
 * 128-byte K steps (128 int8 or 64 bf16 columns), the same roles. */
/* A warp's [32 rows][64 columns] staging boxes to y at (n0, y0); a box that starts past the matrix is not issued
 * (one that overlaps its edge is clipped by the copy). */
__device__ __forceinline__ void store_boxes(const CUtensorMap* map_y, const uint8_t* stg, int64_t n0, int32_t y0, int64_t M,
                                            int64_t N) {
    if (y0 < M) {
#pragma unroll
        for (int b = 0; b < kBoxes; ++b)
            if (n0 + 64 * b < N) rf::tma_store_2d(map_y, stg + b * kOutBox, (int32_t)(n0 + 64 * b), y0);
    }
    rf::bulk_store_commit();
}

/* Eight columns of a finished K block folded into a lane's f32 sums: acc = fma(float(dot) * sa, sb[n], acc), the
 * product and the fma two columns an instruction (packed f32x2, each lane rounded as the scalar form). */
__device__ __forceinline__ void fold8(const uint32_t (&r)[8], float* acc8, const float* sb8, float sa) {
    const float4 s0 = *(const float4*)sb8, s1 = *(const float4*)(sb8 + 4);
    const float sv[8] = { s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w };
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
        float t0, t1;
        rf::mul2_rn(t0, t1, __int2float_rn((int)r[e]), __int2float_rn((int)r[e + 1]), sa, sa);
        rf::fma2_rn(acc8[e], acc8[e + 1], t0, t1, sv[e], sv[e + 1]);
    }
}

/* One finished K block (the lane's kWarpCols accumulator columns at `taddr`) folded into its f32 sums, eight
 * columns a tensor-memory load. kDump: also the block's int32 sums into g.acc (the optional acc operand). */
template <bool kDump>
__device__ __forceinline__ void fold_block(uint32_t taddr, float (&acc)[kWarpCols], const float* sb, float sa,
                                           const RidgeFillGemmQ& g, int64_t m, int64_t n0, bool row_live, int f, int blocks) {
#pragma unroll
    for (int c = 0; c < kWarpCols / 8; ++c) {
        uint32_t r[8];
        rf::tmem_ld8(taddr + c * 8, r);
        rf::tmem_ld_wait();
        if (kDump && row_live)
            for (int i = 0; i < 8; ++i)
                if (n0 + c * 8 + i < g.N) g.acc[(m * g.N + n0 + c * 8 + i) * blocks + f] = (int32_t)r[i];
        fold8(r, acc + c * 8, sb + c * 8, sa);
    }
}

/* The kernel's forms: the bf16 GEMM, the int8 projector, the int8 projector writing out its int32 block sums
 * (the optional acc operand), the int8 projector writing only the selected rows (the optional rows operand), and
 * the DeltaNet in-projection with the convolution in its epilogue. Separate instantiations keep each form's
 * registers to itself. */
enum GemmMode {
    kModeBf16 = 0, kModeI8 = 1, kModeI8Dump = 2, kModeI8Rows = 3, kModeI8Conv = 4, kModeBf16Narrow = 5,
    kModeI8One = 6, kModeI8RowsOne = 7,   /* kModeI8 / kModeI8Rows with one K block (group = K): the streamed fold */
    kModeCount = 8
};

/* A pair tile's columns: 256, or 64 for the narrow bf16 form (N <= 64, e.g. the DeltaNet a|b projection), whose
 * M256 N64 products leave the MMAs a quarter of the wide form's work when it would mostly multiply zero rows. */
template <int kMode>
__host__ __device__ constexpr int bn_of() { return kMode == kModeBf16Narrow ? 64 : BN; }

/* Threads a CTA of each form: the producer and MMA warps, then the epilogue warps. */
template <int kMode>
constexpr int threads_of() { return 32 * (2 + (kMode == kModeI8Conv ? kConvWarps : kEpiWarps)); }

/* The first row a CTA projects: 256-row pair tiles, or for the in-projection 250-row pair tiles each CTA of which
 * starts three rows before its 125 output rows (a negative start reads zeros). */
template <int kMode>
__device__ __forceinline__ int64_t tile_row0(int tile, int n_tiles, uint32_t rank) {
    if constexpr (kMode == kModeI8Conv) return (int64_t)(tile / n_tiles) * (2 * kConvRows) + (int64_t)rank * kConvRows - 3;
    else return (int64_t)(tile / n_tiles) * BM2 + (int64_t)rank * BM;
}

/* The 16-byte chunk j (of 32) of row t in the in-projection's row-major [128][256] bf16 tile: XOR-swizzled by the
 * row's low three bits, so a warp's lanes writing one chunk of 32 rows, or reading 16 chunks of a row, meet no
 * bank conflict. */
__device__ __forceinline__ int conv_chunk(int t, int j) { return t * 512 + ((j ^ (t & 7)) << 4); }

/* The K blocks of one tile folded into a lane's f32 sums. The scales of block f + 1 are fetched while block f waits
 * and folds: a_scale into a register, this warp's b_scale values (four a lane) by asynchronous copy into the warp's
 * other shared-memory slot (columns past N read as zero). Each accumulator buffer goes back to the MMA warp once
 * read. False when a wait gave up. */
template <bool kDump>
__device__ __forceinline__ bool fold_tile(const GemmPlan& p, float (&acc)[kWarpCols], float* slots, uint32_t lane_addr, int lane,
                                          int64_t m, int64_t n0, bool row_live, uint32_t& fold, volatile int* abort,
                                          uint64_t* acc_full, uint64_t* acc_empty) {
    const RidgeFillGemmQ& g = p.g;
    const bool copies = lane < kWarpCols / 4;
    const uint32_t col_bytes = copies && n0 + lane * 4 < g.N ? 16u : 0u;   /* N is a multiple of 16 */
#pragma unroll
    for (int i = 0; i < kWarpCols; ++i) acc[i] = 0.0f;
    __syncwarp();   /* the previous tile's reads of the slots are done */
    if (copies) rf::cp_async16_zfill(slots + lane * 4, g.b_scale + (col_bytes ? n0 + lane * 4 : 0), col_bytes);
    float sa_next = row_live ? g.a_scale[m * g.ldas] : 0.0f;
    for (int f = 0; f < p.folds; ++f, ++fold) {
        const uint32_t buf = fold & 1, use = (fold >> 1) & 1;
        const float* sb = slots + (f & 1) * kWarpCols;
        rf::cp_async_wait_all();
        __syncwarp();   /* block f's scales are in, and every lane is done with block f - 1's slot */
        const float sa = sa_next;
        if (f + 1 < p.folds) {
            if (copies)
                rf::cp_async16_zfill(slots + ((f + 1) & 1) * kWarpCols + lane * 4,
                                     g.b_scale + (col_bytes ? (int64_t)(f + 1) * g.N + n0 + lane * 4 : 0), col_bytes);
            sa_next = row_live ? g.a_scale[m * g.ldas + f + 1] : 0.0f;
        }
        if (!rf::mbar_wait(&acc_full[buf], use, abort, rf::kErrGemmWaitEpilogue)) return false;
        rf::tc_fence_after();
        fold_block<kDump>(lane_addr + buf * BN, acc, sb, sa, g, m, n0, row_live, f, p.folds);
        rf::tc_fence_before();
        __syncwarp();
        if (lane == 0) rf::mbar_arrive_cluster_relaxed(rf::map_rank(rf::smem_addr(&acc_empty[buf]), 0));
    }
    return true;
}

/* Two f32 as a bf16 pair, rounded to nearest even by the hardware conversion: conv_prep's output rounding. */
__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *(const uint32_t*)&v;
}

__device__ __forceinline__ void unpack4(uint2 v, float (&f)[4]) {
    f[0] = __uint_as_float(v.x << 16);
    f[1] = __uint_as_float(v.x & 0xffff0000u);
    f[2] = __uint_as_float(v.y << 16);
    f[3] = __uint_as_float(v.y & 0xffff0000u);
}

/* One output row of the in-projection's convolution for a lane's 4 channels, conv_prep's arithmetic (so the bits
 * agree): x0..x3 the input rows r - 3 .. r; per channel u = bias, u = fma(w_j, x_j, u) for j = 0..3, y = silu(u); for a
 * k head y *= rsqrt(ss + 1e-6), ss the lane's four squares by fma, then the warp's butterfly (xor 16, 8, 4, 2, 1: the
 * warp is the head). The output row `dst`. */
__device__ __forceinline__ void conv_out(const float (&w)[4][4], const float (&bs)[4], const float (&x0)[4], const float (&x1)[4],
                                         const float (&x2)[4], const float (&x3)[4], bool is_k, bool col_live, uint16_t* dst) {
    float y[4];
#pragma unroll
    for (int e = 0; e < 4; e += 2) {   /* two channels an instruction (packed f32x2, each rounded as the scalar fma) */
        float u0 = bs[e], u1 = bs[e + 1];
        rf::fma2_rn(u0, u1, w[e][0], w[e + 1][0], x0[e], x0[e + 1]);
        rf::fma2_rn(u0, u1, w[e][1], w[e + 1][1], x1[e], x1[e + 1]);
        rf::fma2_rn(u0, u1, w[e][2], w[e + 1][2], x2[e], x2[e + 1]);
        rf::fma2_rn(u0, u1, w[e][3], w[e + 1][3], x3[e], x3[e + 1]);
        y[e] = rf::silu(u0);
        y[e + 1] = rf::silu(u1);
    }
    if (is_k) {
        float ss = 0.0f;
#pragma unroll
        for (int e = 0; e < 4; ++e) ss = fmaf(y[e], y[e], ss);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = rsqrtf(ss + 1e-6f);
        rf::mul2_rn(y[0], y[1], y[0], y[1], inv, inv);
        rf::mul2_rn(y[2], y[3], y[2], y[3], inv, inv);
    }
    if (col_live) *(uint2*)dst = make_uint2(bf16x2(y[0], y[1]), bf16x2(y[2], y[3]));
}

/* The in-projection's convolution over one CTA tile (rows_tile: the projection's rows m0 .. m0 + 127 as bf16; meta:
 * each row's sequence start, -1 outside every sequence, and its history slot, -1 for none). Epilogue warp cw takes
 * one of the tile's two 128-channel heads (cw & 1) over a run of output rows (16 rows for 16 warps), lane l its
 * channels 4 l .. 4 l + 3 -- conv_prep's layout. Rows go in groups of four: when the four lie in one sequence (the
 * common case) their seven input rows are loaded and widened once and the four rows computed side by side;
 * otherwise row by row. An input row before the sequence's start comes from its conv-state slot, or is zero. */
__device__ __forceinline__ void conv_rows(const GemmPlan& p, const uint8_t* rows_tile, const int32_t* meta_s0,
                                          const int32_t* meta_slot, int64_t m0, int64_t nt0, int cw, int lane) {
    const RidgeFillInProj& c = p.c;
    const int64_t M = p.g.M, N = p.g.N;
    const int hcol = cw & 1;
    const int64_t cn = nt0 + hcol * 128 + lane * 4;
    const bool col_live = cn < N, is_k = cn < c.n_k;   /* both the same over the warp */
    float w[4][4], bs[4];   /* channel e's taps w[e][0..3] and bias, widened once a tile */
    {
        uint4 wv[2] = {};
        uint2 bv = {};
        if (col_live) {
            wv[0] = __ldg((const uint4*)(c.w + cn * 4));
            wv[1] = __ldg((const uint4*)(c.w + cn * 4 + 8));
            if (c.bias) bv = __ldg((const uint2*)(c.bias + cn));
        }
        const uint32_t ww[8] = { wv[0].x, wv[0].y, wv[0].z, wv[0].w, wv[1].x, wv[1].y, wv[1].z, wv[1].w };
#pragma unroll
        for (int e = 0; e < 4; ++e)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t word = ww[2 * e + (j >> 1)];
                w[e][j] = __uint_as_float((j & 1) ? (word & 0xffff0000u) : (word << 16));
            }
        unpack4(bv, bs);
    }
    uint16_t* out;
    int64_t out_row;
    if (is_k) {
        out = c.k + (cn >> 7) * c.k_head + (cn & 127);
        out_row = c.k_row;
    } else {
        const int64_t vc = cn - c.n_k;
        out = c.v + (vc >> 7) * c.v_head + (vc & 127);
        out_row = c.v_row;
    }
    const uint8_t* my_tile = rows_tile + (lane & 1) * 8;
    const int chunk = hcol * 16 + (lane >> 1);
    /* input row t_in of an output row in the sequence starting at s0 with history slot `slot` */
    auto fetch = [&](int t_in, int s0, int slot, float (&f)[4]) {
        const int64_t rr = m0 + t_in;
        uint2 v = make_uint2(0u, 0u);
        if (rr >= s0) v = *(const uint2*)(my_tile + conv_chunk(t_in, chunk));
        else if (slot >= 0 && col_live) v = *(const uint2*)(c.state + slot * c.st_slot + (3 - (s0 - rr)) * c.st_row + cn);
        unpack4(v, f);
    };
    constexpr int kRowsPer = (kConvRows + kConvWarps / 2 - 1) / (kConvWarps / 2);
    const int tb = 3 + (cw >> 1) * kRowsPer, te = min(tb + kRowsPer, BM);
    for (int t = tb; t < te; t += 4) {
        const int n = min(4, te - t);
        const int s0 = meta_s0[t];
        bool group = n == 4 && s0 >= 0 && m0 + t + 3 < M;
#pragma unroll
        for (int i = 1; i < 4; ++i) group = group && meta_s0[min(t + i, BM - 1)] == s0;
        if (group) {
            float x[7][4];
            if (m0 + t - 3 >= s0) {   /* the whole window inside the tile: plain loads */
#pragma unroll
                for (int j = 0; j < 7; ++j) unpack4(*(const uint2*)(my_tile + conv_chunk(t - 3 + j, chunk)), x[j]);
            } else {
                const int slot = meta_slot[t];
#pragma unroll
                for (int j = 0; j < 7; ++j) fetch(t - 3 + j, s0, slot, x[j]);
            }
            uint16_t* dst = out + (m0 + t) * out_row;
#pragma unroll
            for (int i = 0; i < 4; ++i) conv_out(w, bs, x[i], x[i + 1], x[i + 2], x[i + 3], is_k, col_live, dst + i * out_row);
        } else {
            for (int i = 0; i < n; ++i) {
                const int ti = t + i;
                if (m0 + ti >= M) break;
                const int si = meta_s0[ti];
                if (si < 0) continue;   /* outside every sequence: left untouched */
                const int sl = meta_slot[ti];
                float x0[4], x1[4], x2[4], x3[4];
                fetch(ti - 3, si, sl, x0);
                fetch(ti - 2, si, sl, x1);
                fetch(ti - 1, si, sl, x2);
                fetch(ti, si, sl, x3);
                conv_out(w, bs, x0, x1, x2, x3, is_k, col_live, out + (m0 + ti) * out_row);
            }
        }
    }
}

/* The in-projection's epilogue warps (kConvWarps of them; the first kEpiWarps also fold). Per tile (one K block:
 * group = K): a folding lane's row waits for its sums and looks up its sequence; the epilogue barrier, which also
 * agrees on a failed wait (every warp then leaves together), ensures every warp is done with the previous tile's
 * rows; the folding warps fold their sums 32 columns a tensor-memory load (the b_scale values prefetched into the
 * warp's shared-memory slot), round them to bf16 into the row tile (each sequence's last three rows also to `tail`)
 * and hand the accumulator back to the MMA warp; a second barrier; every warp convolves. False when a wait gave up. */
__device__ __forceinline__ bool conv_epilogue(const GemmPlan& p, uint8_t* rows_tile, float* scale_slots, int32_t* meta,
                                              uint32_t lane_addr, int warp, int lane, int pair, int pairs, uint32_t rank,
                                              volatile int* abort, uint64_t* acc_full, uint64_t* acc_empty) {
    const RidgeFillGemmQ& g = p.g;
    const RidgeFillInProj& c = p.c;
    const int ew = warp - 2, slice = ew >> 2, row = (warp & 3) * 32 + lane;
    const bool folds = ew < kEpiWarps;
    float* sb = scale_slots + ew * 2 * kWarpCols;   /* a folding warp's b_scale values */
    int32_t* meta_s0 = meta;
    int32_t* meta_slot = meta + BM;
    uint32_t fold = 0;
    for (int tile = pair; tile < p.tiles; tile += pairs, ++fold) {
        const int64_t m0 = tile_row0<kModeI8Conv>(tile, p.n_tiles, rank), nt0 = (int64_t)(tile % p.n_tiles) * BN;
        const int64_t m = m0 + row, n0 = nt0 + slice * kWarpCols;
        const bool row_live = folds && m >= 0 && m < g.M;
        const uint32_t buf = fold & 1, use = (fold >> 1) & 1;
        float sa = 0.0f;
        bool ok = true;
        int64_t s0 = -1, e0 = -1;
        int seq = -1;
        int32_t slot = -1;
        if (folds) {
            sa = row_live ? g.a_scale[m * g.ldas] : 0.0f;
            /* this warp's 64 b_scale values into its shared-memory slot while the sums are computed (the slot's reads
             * of the previous tile ended before its second barrier); columns past N read as zero */
            if (lane < kWarpCols / 4) {
                const bool in = n0 + lane * 4 < g.N;   /* N is a multiple of 128 */
                rf::cp_async16_zfill(sb + lane * 4, g.b_scale + (in ? n0 + lane * 4 : 0), in ? 16u : 0u);
            }
            ok = rf::mbar_wait(&acc_full[buf], use, abort, rf::kErrGemmWaitEpilogue);
            /* the row's sequence and the conv-state slot of its history */
            seq = ok && row_live ? rf::find_seq(c.cu, c.n_seq, g.M, m, &s0, &e0) : -1;
            if (seq >= 0 && c.ctx && c.ctx[seq] > 0) {
                const int64_t sl = c.idx[seq * c.idx_pitch];
                if (sl >= 0 && sl < c.n_states) slot = (int32_t)sl;
            }
            rf::cp_async_wait_all();
        }
        if (rf::bar_any(kEpiBar, 32 * kConvWarps, !ok)) return false;
        if (folds) {
            rf::tc_fence_after();
            const bool tail_row = row >= 3 && seq >= 0 && m >= e0 - 3;
#pragma unroll 1
            for (int h = 0; h < kWarpCols / 32; ++h) {   /* 32 columns a tensor-memory load */
                uint32_t r[32];
                rf::tmem_ld32(lane_addr + buf * BN + h * 32, r);
                rf::tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int v = h * 4 + j;
                    const int64_t n = n0 + v * 8;
                    float a8[8] = {};
                    fold8(*(const uint32_t(*)[8])(r + j * 8), a8, sb + v * 8, sa);
                    /* the hardware's round to nearest even: the GEMM's rounding for every value but a NaN (made
                     * the canonical one) */
                    const uint4 q = make_uint4(bf16x2(a8[0], a8[1]), bf16x2(a8[2], a8[3]), bf16x2(a8[4], a8[5]),
                                               bf16x2(a8[6], a8[7]));
                    *(uint4*)(rows_tile + conv_chunk(row, slice * (kWarpCols / 8) + v)) = q;
                    if (tail_row && n < g.N) *(uint4*)(g.y + m * g.ldy + n) = q;
                }
            }
            rf::tc_fence_before();
            __syncwarp();
            if (lane == 0) rf::mbar_arrive_cluster_relaxed(rf::map_rank(rf::smem_addr(&acc_empty[buf]), 0));
            if (slice == 0) {
                meta_s0[row] = seq >= 0 ? (int32_t)s0 : -1;
                meta_slot[row] = slot;
            }
        }
        rf::bar_sync(kEpiBar, 32 * kConvWarps);
        conv_rows(p, rows_tile, meta_s0, meta_slot, m0, nt0, ew, lane);
    }
    return true;
}

/* Eight bf16 columns n0 + 8 v .. + 7 of a lane's row (its f32 sums a8), the bias added and rounded again, into the
 * warp's staging tile (box v >> 3, row lane, 16-byte chunk v & 7 at its 128-byte-swizzled place) or, direct, into
 * the row of y itself when the row is selected. The hardware's round to nearest even: the fold's rounding for every
 * value but a NaN (made the canonical one). */
template <bool kDirect>
__device__ __forceinline__ void emit8(const RidgeFillGemmQ& g, uint8_t* stg, bool write_row, int64_t m, int64_t n0, int lane, int v,
                                      const float* a8) {
    const int64_t n = n0 + v * 8;
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = bf16x2(a8[2 * e], a8[2 * e + 1]);
    if (g.bias && n < g.N) {
        const uint4 bv = __ldg((const uint4*)(g.bias + n));
        const uint32_t bw[4] = { bv.x, bv.y, bv.z, bv.w };
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float lo = __fadd_rn(__uint_as_float(o[e] << 16), __uint_as_float(bw[e] << 16));
            const float hi = __fadd_rn(__uint_as_float(o[e] & 0xffff0000u), __uint_as_float(bw[e] & 0xffff0000u));
            o[e] = bf16x2(lo, hi);
        }
    }
    if constexpr (kDirect) {
        if (write_row && n < g.N) *(uint4*)(g.y + m * g.ldy + n) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
        *(uint4*)(stg + (v >> 3) * kOutBox + lane * 128 + (((v & 7) ^ (lane & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

template <int kMode>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(threads_of<kMode>(), 1)
gemm_q_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
              const __grid_constant__ CUtensorMap map_y, const GemmPlan p) {
    constexpr bool kBf16 = kMode == kModeBf16 || kMode == kModeBf16Narrow;
    constexpr int kBN = bn_of<kMode>();
    constexpr uint32_t kTxBytes = 2 * (kABytes + (kBN / 2) * BK);   /* both CTAs' A and B halves a stage */
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* tile_a = smem;
    uint8_t* tile_b = smem + kStages * kABytes;
    uint8_t* stage_out = smem + kStages * kStageBytes;   /* 1024-byte aligned: kStageBytes is */
    float* scale_slots = (float*)(stage_out + kStageOut);
    int32_t* meta = (int32_t*)(stage_out + kStageOut + kScaleSlots);
    uint64_t* full = (uint64_t*)(stage_out + kStageOut + kScaleSlots + kMetaBytes);
    uint64_t* empty = full + kStages;
    uint64_t* acc_full = empty + kStages;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = (uint32_t*)(acc_empty + 2);
    volatile int* abort = (volatile int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = rf::cluster_rank();   /* 0: the CTA that issues the pair's MMAs */
    const int pair = (int)rf::cluster_id_x(), pairs = (int)rf::cluster_count_x();
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            rf::mbar_init(&full[s], 1);    /* rank 0's: its producer's expect_tx, both CTAs' bytes */
            rf::mbar_init(&empty[s], 1);   /* each CTA's: the MMA warp's commit */
        }
        for (int b = 0; b < 2; ++b) {
            rf::mbar_init(&acc_full[b], 1);                /* each CTA's: the MMA warp's commit */
            rf::mbar_init(&acc_empty[b], 2 * kEpiWarps);   /* rank 0's: both CTAs' epilogue warps */
        }
        *abort = 0;
        rf::mbar_init_fence();
        rf::tma_prefetch_map(&map_a);
        rf::tma_prefetch_map(&map_b);
        rf::tma_prefetch_map(&map_y);
    }
    if (warp == 1) rf::tmem_alloc_pair<kTmemCols>(tmem_slot);
    rf::tc_fence_before();
    rf::cluster_sync_all();   /* both CTAs' barriers are initialised before either signals the other's */
    rf::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const RidgeFillGemmQ& g = p.g;

    if (warp == 0) {
        /* ---------------------------------------------------------- producer (both CTAs) */
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            int64_t issued = 0;
            const int steps = p.folds * p.steps_per_fold;
            for (int tile = pair; tile < p.tiles && !*abort; tile += pairs) {
                const int m0 = (int)tile_row0<kMode>(tile, p.n_tiles, rank), n0 = (tile % p.n_tiles) * kBN + (int)rank * (kBN / 2);
                for (int ks = 0; ks < steps; ++ks) {
                    if (!rf::mbar_wait(&empty[stage], phase ^ 1, abort, rf::kErrGemmWaitProducer)) break;
                    if (rank == 0) rf::mbar_arrive_expect_tx(&full[stage], kTxBytes);
                    const int kx = ks * (kBf16 ? BK / 2 : BK);   /* the K step's first column, in elements */
                    const uint32_t bar = rf::map_rank(rf::smem_addr(&full[stage]), 0);   /* rank 0's */
                    rf::tma_load_2d_pair(tile_a + stage * kABytes, &map_a, bar, kx, m0);
                    rf::tma_load_2d_pair(tile_b + stage * kBBytes, &map_b, bar, kx, n0);
                    ++issued;
                    if (++stage == kStages) { stage = 0; phase ^= 1; }
                }
            }
            /* Drain: the MMAs have released every stage this CTA loaded (so its loads have landed and the
             * pair's MMAs no longer read its shared memory) before the CTA leaves. One deadline. */
            const int64_t first = issued > kStages ? issued - kStages : 0;
            const uint64_t t0 = rf::global_ns();
            for (int64_t i = first; i < issued; ++i) {
                while (!rf::mbar_try_wait(&empty[i % kStages], (uint32_t)((i / kStages) & 1))) {
                    if (rf::global_ns() - t0 > rf::kWaitTimeoutNs) {
                        atomicCAS(&rf::g_device_error, 0, (int)rf::kErrGemmDrain);
                        break;
                    }
                }
            }
        }
    } else if (warp == 1) {
        /* ---------------------------------------------------------- MMA issuer (rank 0) */
        if (lane == 0 && rank == 0) {
            uint32_t stage = 0, phase = 0, fold = 0;
            bool ok = true;
            for (int tile = pair; tile < p.tiles && ok; tile += pairs) {
                for (int f = 0; f < p.folds && ok; ++f, ++fold) {
                    const uint32_t buf = fold & 1, use = (fold >> 1) & 1;
                    if (!(ok = rf::mbar_wait(&acc_empty[buf], use ^ 1, abort, rf::kErrGemmWaitMma))) break;
                    rf::tc_fence_after();
                    const uint32_t d = tmem_base + buf * BN;
                    for (int ks = 0; ks < p.steps_per_fold; ++ks) {
                        if (!(ok = rf::mbar_wait(&full[stage], phase, abort, rf::kErrGemmWaitMma))) break;
                        rf::tc_fence_after();
                        const uint32_t a_addr = rf::smem_addr(tile_a + stage * kABytes);
                        const uint32_t b_addr = rf::smem_addr(tile_b + stage * kBBytes);
#pragma unroll
                        for (int kk = 0; kk < BK / 32; ++kk) {   /* 32 bytes of K a product: 32 int8 or 16 bf16 */
                            if constexpr (kBf16)
                                rf::umma_f16_pair(d, rf::sw128_kmajor_desc(a_addr + kk * 32), rf::sw128_kmajor_desc(b_addr + kk * 32),
                                                  idesc_bf16(kBN), (ks | kk) != 0);
                            else
                                rf::mma_i8_pair(d, rf::sw128_kmajor_desc(a_addr + kk * 32), rf::sw128_kmajor_desc(b_addr + kk * 32),
                                                kIdesc, (ks | kk) != 0);
                        }
                        /* the stage is free in both CTAs once these MMAs have read it */
                        rf::mma_commit_pair(rf::smem_addr(&empty[stage]));
                        rf::mma_commit_pair(rf::map_rank(rf::smem_addr(&empty[stage]), 1));
                        if (++stage == kStages) { stage = 0; phase ^= 1; }
                    }
                    if (ok) {   /* the block's sums are final, in both CTAs' tensor memory */
                        rf::mma_commit_pair(rf::smem_addr(&acc_full[buf]));
                        rf::mma_commit_pair(rf::map_rank(rf::smem_addr(&acc_full[buf]), 1));
                    }
                }
            }
        }
    } else {
        /* ---------------------------------------------------------- epilogue */
        const int quarter = warp & 3, slice = (warp - 2) >> 2;   /* a warp reads tensor-memory lanes 32 (warp % 4).. */
        const int row = quarter * 32 + lane;
        const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16) + slice * kWarpCols;
        uint32_t fold = 0;
        bool ok = true;
        if constexpr (kBf16) {
            /* y = res + act(acc + bias): 32 columns at a time from tensor memory, each rounding to bf16 where
             * ridgefill_gemm_nt_bias rounds, into the staging tiles; the accumulator is released after its
             * last read. */
            const RidgeFillGemmBias& gb = p.gb;
            for (int tile = pair; tile < p.tiles && ok; tile += pairs, ++fold) {
                const int64_t m = (int64_t)(tile / p.n_tiles) * BM2 + rank * BM + row;
                const int64_t n0 = (int64_t)(tile % p.n_tiles) * kBN + slice * kWarpCols;
                const uint32_t buf = fold & 1, use = (fold >> 1) & 1;
                if (!(ok = rf::mbar_wait(&acc_full[buf], use, abort, rf::kErrGemmWaitEpilogue))) break;
                if (n0 >= gb.N) {   /* a slice past y's last column (the narrow form's slices 1-3): nothing to write */
                    rf::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) rf::mbar_arrive_cluster_relaxed(rf::map_rank(rf::smem_addr(&acc_empty[buf]), 0));
                    continue;
                }
                rf::tc_fence_after();
                uint8_t* stg = stage_out + (warp - 2) * kBoxes * kOutBox;
                if (lane == 0) rf::bulk_store_wait_read();
                __syncwarp();
#pragma unroll 1
                for (int c = 0; c < kWarpCols / 32; ++c) {
                    uint32_t r[32];
                    rf::tmem_ld32(lane_addr + buf * BN + c * 32, r);
                    rf::tmem_ld_wait();
                    if (c == kWarpCols / 32 - 1) {
                        rf::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) rf::mbar_arrive_cluster_relaxed(rf::map_rank(rf::smem_addr(&acc_empty[buf]), 0));
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int cc = c * 32 + j * 8;   /* column within this warp's slice */
                        const int64_t n = n0 + cc;
                        float bv[8] = {}, rv[8] = {};
                        if (n < gb.N) {
                            if (gb.bias_f32) {
                                const float4 b0 = __ldg((const float4*)((const float*)gb.bias + n));
                                const float4 b1 = __ldg((const float4*)((const float*)gb.bias + n + 4));
                                bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
                                bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
                            } else {
                                const uint4 bb = __ldg((const uint4*)((const uint16_t*)gb.bias + n));
                                const uint32_t bw[4] = { bb.x, bb.y, bb.z, bb.w };
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    bv[2 * e] = __uint_as_float(bw[e] << 16);
                                    bv[2 * e + 1] = __uint_as_float(bw[e] & 0xffff0000u);
                                }
                            }
                            if (gb.res && m < gb.M) {
                                const uint4 rr = *(const uint4*)(gb.res + m * gb.ldr + n);
                                const uint32_t rw[4] = { rr.x, rr.y, rr.z, rr.w };
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    rv[2 * e] = __uint_as_float(rw[e] << 16);
                                    rv[2 * e + 1] = __uint_as_float(rw[e] & 0xffff0000u);
                                }
                            }
                        }
                        uint32_t o[4];
#pragma unroll
                        for (int e = 0; e < 8; e += 2) {
                            float v[2];
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                float x = rf::bf16_bits_to_f32(rf::f32_to_bf16_bits(__fadd_rn(__uint_as_float(r[j * 8 + e + h]), bv[e + h])));
                                if (gb.act == RIDGEFILL_ACT_SILU)
                                    x = rf::bf16_bits_to_f32(rf::f32_to_bf16_bits(__fdiv_rn(x, __fadd_rn(1.0f, expf(-x)))));
                                if (gb.res) x = __fadd_rn(x, rv[e + h]);
                                v[h] = x;
                            }
                            o[e >> 1] = rf::pack_bf16(v[0], v[1]);
                        }
                        *(uint4*)(stg + (cc >> 6) * kOutBox + lane * 128 + ((((cc & 63) >> 3) ^ (lane & 7)) << 4)) =
                            make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
                rf::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    const int32_t y0 = (int32_t)((tile / p.n_tiles) * BM2 + rank * BM + quarter * 32);
                    store_boxes(&map_y, stg, n0, y0, gb.M, gb.N);
                }
            }
        }
        if constexpr (kMode == kModeI8Conv)
            ok = conv_epilogue(p, stage_out, scale_slots, meta, lane_addr, warp, lane, pair, pairs, rank, abort, acc_full,
                               acc_empty);
        for (int tile = pair; tile < p.tiles && ok && !kBf16 && kMode != kModeI8Conv; tile += pairs) {
            const int64_t m = (int64_t)(tile / p.n_tiles) * BM2 + rank * BM + row;
            const int64_t n0 = (int64_t)(tile % p.n_tiles) * BN + slice * kWarpCols;
            const bool row_live = m < g.M;
            /* bf16 (and the bias) into this warp's staging tiles, once the previous tile's stores have read them; or,
             * with a row selection, straight from the lanes into the selected rows of y (a lane is one row). */
            constexpr bool direct = kMode == kModeI8Rows || kMode == kModeI8RowsOne;
            constexpr bool kOne = kMode == kModeI8One || kMode == kModeI8RowsOne;
            if constexpr (kOne) {
                uint8_t* stg = stage_out + (warp - 2) * kBoxes * kOutBox;
                /* one K block (per-row and per-column scales): the sums folded 32 columns a tensor-memory load and
                 * stored as they come, the b_scale values prefetched into the warp's shared-memory slot */
                const bool write_row = direct && row_live && __ldg(g.rows + m) == 1;
                float* sb = scale_slots + (warp - 2) * 2 * kWarpCols;
                __syncwarp();   /* the previous tile's reads of the slot are done */
                if (lane < kWarpCols / 4) {
                    const bool in = n0 + lane * 4 < g.N;   /* N is a multiple of 16 */
                    rf::cp_async16_zfill(sb + lane * 4, g.b_scale + (in ? n0 + lane * 4 : 0), in ? 16u : 0u);
                }
                const float sa = row_live ? g.a_scale[m * g.ldas] : 0.0f;
                const uint32_t buf = fold & 1, use = (fold >> 1) & 1;
                ++fold;
                if (!(ok = rf::mbar_wait(&acc_full[buf], use, abort, rf::kErrGemmWaitEpilogue))) break;
                rf::cp_async_wait_all();
                if constexpr (!direct) {
                    if (lane == 0) rf::bulk_store_wait_read();
                }
                __syncwarp();
                rf::tc_fence_after();
#pragma unroll 1
                for (int h = 0; h < kWarpCols / 32; ++h) {
                    uint32_t r[32];
                    rf::tmem_ld32(lane_addr + buf * BN + h * 32, r);
                    rf::tmem_ld_wait();
                    if (h == kWarpCols / 32 - 1) {   /* the accumulator's last read: back to the MMA warp */
                        rf::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) rf::mbar_arrive_cluster_relaxed(rf::map_rank(rf::smem_addr(&acc_empty[buf]), 0));
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float a8[8] = {};
                        fold8(*(const uint32_t(*)[8])(r + j * 8), a8, sb + (h * 4 + j) * 8, sa);
                        emit8<direct>(g, stg, write_row, m, n0, lane, h * 4 + j, a8);
                    }
                }
            } else {
                float acc[kWarpCols];
                if (!(ok = fold_tile<kMode == kModeI8Dump>(p, acc, scale_slots + (warp - 2) * 2 * kWarpCols, lane_addr, lane, m,
                                                             n0, row_live, fold, abort, acc_full, acc_empty)))
                    break;
                uint8_t* stg = stage_out + (warp - 2) * kBoxes * kOutBox;
                const bool write_row = direct && row_live && __ldg(g.rows + m) == 1;
                if constexpr (!direct) {
                    if (lane == 0) rf::bulk_store_wait_read();
                    __syncwarp();
                }
#pragma unroll
                for (int v = 0; v < kWarpCols / 8; ++v) {
                    const int64_t n = n0 + v * 8;
                    uint32_t o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        o[e] = (uint32_t)rf::f32_to_bf16_bits(acc[v * 8 + 2 * e]) |
                               ((uint32_t)rf::f32_to_bf16_bits(acc[v * 8 + 2 * e + 1]) << 16);
                    if (g.bias && n < g.N) {
                        const uint4 bv = __ldg((const uint4*)(g.bias + n));
                        const uint32_t bw[4] = { bv.x, bv.y, bv.z, bv.w };
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float lo = __fadd_rn(__uint_as_float(o[e] << 16), __uint_as_float(bw[e] << 16));
                            const float hi = __fadd_rn(__uint_as_float(o[e] & 0xffff0000u), __uint_as_float(bw[e] & 0xffff0000u));
                            o[e] = (uint32_t)rf::f32_to_bf16_bits(lo) | ((uint32_t)rf::f32_to_bf16_bits(hi) << 16);
                        }
                    }
                    if constexpr (direct) {
                        if (write_row && n < g.N) *(uint4*)(g.y + m * g.ldy + n) = make_uint4(o[0], o[1], o[2], o[3]);
                    } else {
                        *(uint4*)(stg + (v >> 3) * kOutBox + lane * 128 + (((v & 7) ^ (lane & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
            }
            uint8_t* stg = stage_out + (warp - 2) * kBoxes * kOutBox;
            if constexpr (direct) continue;
            rf::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                const int32_t y0 = (int32_t)((tile / p.n_tiles) * BM2 + rank * BM + quarter * 32);
                store_boxes(&map_y, stg, n0, y0, g.M, g.N);
            }
        }
        if (lane == 0) rf::bulk_store_wait();   /* the tile stores are complete before the CTA leaves */
    }

    /* Neither CTA leaves while the other may still signal its barriers; then both free the pair's columns. */
    rf::tc_fence_before();
    __syncwarp();
    rf::cluster_sync_all();
    if (warp == 1) {
        rf::tc_fence_after();
        rf::tmem_free_pair<kTmemCols>(tmem_base);
    }
}

/* ------------------------------------------------------------------ quantiser */

/* One warp per (row, group); lane l reads 4-element chunks l, l + 32, ... of the group (coalesced
 * 256-byte warp reads). Pass 1 finds the group's absmax, pass 2 writes the codes. */
__global__ void __launch_bounds__(256) quant_kernel(RidgeFillQuant g) {
    const int lane = threadIdx.x & 31;
    const int64_t groups = g.K / g.group, work = g.M * groups;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int chunks = (int)(g.group / 4);
    for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < work; w += warps) {
        const int64_t m = w / groups, j = w - m * groups;
        const uint16_t* x = g.x + m * g.ldx + j * g.group;
        float amax = 0.0f;
        for (int c = lane; c < chunks; c += 32) {
            const uint2 v = *(const uint2*)(x + 4 * c);
            amax = fmaxf(amax, fabsf(__uint_as_float(v.x << 16)));
            amax = fmaxf(amax, fabsf(__uint_as_float(v.x & 0xffff0000u)));
            amax = fmaxf(amax, fabsf(__uint_as_float(v.y << 16)));
            amax = fmaxf(amax, fabsf(__uint_as_float(v.y & 0xffff0000u)));
        }
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float s = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
        if (lane == 0) g.s[m * g.lds + j] = s;
        int8_t* q = g.q + m * g.ldq + j * g.group;
        for (int c = lane; c < chunks; c += 32) {
            const uint2 v = *(const uint2*)(x + 4 * c);
            const float xs[4] = { __uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                                  __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u) };
            uint32_t packed = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                int r = __float2int_rn(__fdiv_rn(xs[e], s));
                r = r > 127 ? 127 : (r < -127 ? -127 : r);
                packed |= (uint32_t)(uint8_t)(int8_t)r << (8 * e);
            }
            *(uint32_t*)(q + 4 * c) = packed;
        }
    }
}

/* One pass over HBM when the groups tile 2,048-column segments (K % 2048 == 0, group a power of two
 * <= 2048): a CTA takes a segment of a row at a time, thread t holds columns 8t..8t+7 (one 16-byte load),
 * a group's absmax is reduced in the warp (group <= 256) or over its warps in shared memory, then every
 * thread writes its 8 codes and each group's first thread its scale. The same arithmetic as quant_kernel. */
constexpr int kQSeg = 2048, kQThreads = kQSeg / 8, kQRows = 4;

__global__ void __launch_bounds__(kQThreads) quant_seg_kernel(RidgeFillQuant g) {
    __shared__ float wmax[kQRows][kQThreads / 32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t segs = g.K / kQSeg, work = g.M * segs;
    const int tpg = (int)(g.group / 8);   /* threads a group: a power of two, 1..256 */
    const int lanes = tpg < 32 ? tpg : 32;
    /* kQRows segments an iteration, their loads issued together */
    for (int64_t w0 = (int64_t)blockIdx.x * kQRows; w0 < work; w0 += (int64_t)gridDim.x * kQRows) {
        uint4 v[kQRows];
#pragma unroll
        for (int r = 0; r < kQRows; ++r) {
            const int64_t wk = w0 + r < work ? w0 + r : work - 1;
            const int64_t m = wk / segs, c0 = (wk - m * segs) * kQSeg + 8 * t;
            v[r] = *(const uint4*)(g.x + m * g.ldx + c0);
        }
        float amax[kQRows];
#pragma unroll
        for (int r = 0; r < kQRows; ++r) {
            const uint32_t vw[4] = { v[r].x, v[r].y, v[r].z, v[r].w };
            float a = 0.0f;
#pragma unroll
            for (int e = 0; e < 4; ++e) a = fmaxf(a, fmaxf(fabsf(__uint_as_float(vw[e] << 16)), fabsf(__uint_as_float(vw[e] & 0xffff0000u))));
            for (int o = 1; o < lanes; o <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
            amax[r] = a;
        }
        if (tpg > 32) {
            const int wpg = tpg / 32, g0 = warp / wpg * wpg;
            if (lane == 0)
#pragma unroll
                for (int r = 0; r < kQRows; ++r) wmax[r][warp] = amax[r];
            __syncthreads();
#pragma unroll
            for (int r = 0; r < kQRows; ++r) {
                float a = wmax[r][g0];
                for (int q = 1; q < wpg; ++q) a = fmaxf(a, wmax[r][g0 + q]);
                amax[r] = a;
            }
            __syncthreads();   /* wmax is read before the next iteration writes it */
        }
#pragma unroll
        for (int r = 0; r < kQRows; ++r) {
            if (w0 + r >= work) break;
            const int64_t wk = w0 + r, m = wk / segs, c0 = (wk - m * segs) * kQSeg + 8 * t;
            const float sc = amax[r] == 0.0f ? 1.0f : __fdiv_rn(amax[r], 127.0f);
            if ((t & (tpg - 1)) == 0) g.s[m * g.lds + c0 / g.group] = sc;
            const uint32_t vw[4] = { v[r].x, v[r].y, v[r].z, v[r].w };
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float x = __uint_as_float((e & 1) ? (vw[e >> 1] & 0xffff0000u) : (vw[e >> 1] << 16));
                int q = __float2int_rn(__fdiv_rn(x, sc));
                q = q > 127 ? 127 : (q < -127 ? -127 : q);
                if (e < 4) lo |= (uint32_t)(uint8_t)(int8_t)q << (8 * e);
                else hi |= (uint32_t)(uint8_t)(int8_t)q << (8 * (e - 4));
            }
            *(uint2*)(g.q + m * g.ldq + c0) = make_uint2(lo, hi);
        }
    }
}

/* The int8 codes of eight bf16 values (a 16-byte chunk) at scale sc (inv = 1 / sc, rounded), packed in order:
 * rint(x / sc) with the quotient correctly rounded, clamped to [-127, 127] — the oracle's arithmetic. The fast
 * path forms y = fma(x, inv, 1.5 * 2^23), which rounds the exact product x * inv to an integer (to nearest, ties
 * to even) in y's low mantissa bits, so y's low byte is the code in two's complement (|x * inv| <= 127 (1 + 2^-23)
 * here: no clamp), and e = fma(x, inv, -(y - 1.5 * 2^23)), the product's distance from that integer. The exact
 * product lies within 2^-17 of the exact quotient and the rounded quotient within 2^-17 of it, so both round to
 * the same integer unless |e| is within 2^-16 of 1/2; a chunk with any |e| above 1/2 - 2^-15 (or not finite)
 * forms every quotient exactly. */
__device__ __forceinline__ uint2 quant_chunk8(uint4 v, float sc, float inv) {
    constexpr float kMagic = 12582912.0f;   /* 1.5 * 2^23 */
    const uint32_t vw[4] = { v.x, v.y, v.z, v.w };
    uint32_t rb[8];
    bool near = false;
#pragma unroll
    for (int p = 0; p < 4; ++p) {   /* elements 2 p, 2 p + 1 two an instruction (packed f32x2, the same roundings) */
        const float x0 = __uint_as_float(vw[p] << 16), x1 = __uint_as_float(vw[p] & 0xffff0000u);
        float y0 = kMagic, y1 = kMagic, d0, d1;
        rf::fma2_rn(y0, y1, x0, x1, inv, inv);                  /* y = x inv + 1.5 2^23 */
        rf::sub2_rn(d0, d1, kMagic, kMagic, y0, y1);            /* -(y - 1.5 2^23), exact */
        rf::fma2_rn(d0, d1, x0, x1, inv, inv);                  /* e = x inv - (y - 1.5 2^23) */
        near |= !(fabsf(d0) <= 0.5f - 0x1p-15f) | !(fabsf(d1) <= 0.5f - 0x1p-15f);
        rb[2 * p] = __float_as_uint(y0);
        rb[2 * p + 1] = __float_as_uint(y1);
    }
    if (near) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float xv = __uint_as_float((e & 1) ? (vw[e >> 1] & 0xffff0000u) : (vw[e >> 1] << 16));
            const int r = __float2int_rn(__fdiv_rn(xv, sc));
            rb[e] = (uint32_t)(r > 127 ? 127 : (r < -127 ? -127 : r));
        }
    }
    const uint32_t lo = __byte_perm(__byte_perm(rb[0], rb[1], 0x0040), __byte_perm(rb[2], rb[3], 0x0040), 0x5410);
    const uint32_t hi = __byte_perm(__byte_perm(rb[4], rb[5], 0x0040), __byte_perm(rb[6], rb[7], 0x0040), 0x5410);
    return make_uint2(lo, hi);
}

/* One pass over HBM for a group of 256 NV columns held in registers: a warp per (row, group), lane l holds
 * the 16-byte chunks l, l + 32, ... (coalesced 512-byte warp loads); absmax by shuffles, then the codes
 * (quant_chunk8). The same arithmetic as quant_kernel. */
template <int NV>
__global__ void __launch_bounds__(256) quant_reg_kernel(RidgeFillQuant g) {
    const int lane = threadIdx.x & 31;
    const int64_t groups = g.K / g.group, work = g.M * groups;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < work; w += warps) {
        const int64_t m = w / groups, j = w - m * groups;
        const uint16_t* x = g.x + m * g.ldx + j * g.group;
        uint4 v[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = *(const uint4*)(x + 8 * (lane + 32 * i));
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const uint32_t vw[4] = { v[i].x, v[i].y, v[i].z, v[i].w };
#pragma unroll
            for (int e = 0; e < 4; ++e)
                amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(vw[e] << 16)), fabsf(__uint_as_float(vw[e] & 0xffff0000u))));
        }
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float sc = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
        if (lane == 0) g.s[m * g.lds + j] = sc;
        const float inv = __frcp_rn(sc);
        int8_t* q = g.q + m * g.ldq + j * g.group;
#pragma unroll
        for (int i = 0; i < NV; ++i) *(uint2*)(q + 8 * (lane + 32 * i)) = quant_chunk8(v[i], sc, inv);
    }
}

/* The same one-pass quantiser with the data in shared memory instead of registers: a warp per (row, group) of
 * 256 NV columns, the next item's columns copied asynchronously into the warp's other shared-memory slot while
 * the current one is reduced and coded (its columns read from shared memory twice: the absmax, then the codes),
 * so two items a warp are in flight with few registers (more warps a SM than the register form allows). The
 * same arithmetic (quant_chunk8). The items are taken last row first: a producer that wrote x in row order
 * (the projector's tiles) left its last rows in L2, and what reads x next in row order finds its first rows
 * there. */
constexpr int kQStageThreads = 256;
template <int NV>
__global__ void __launch_bounds__(kQStageThreads) quant_stage_kernel(RidgeFillQuant g) {
    extern __shared__ uint4 qstage[];   /* [warp][2][NV * 32] */
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    uint4* slots = qstage + wib * 2 * NV * 32;
    const int64_t groups = g.K / g.group, work = g.M * groups;
    const int64_t warps = (int64_t)gridDim.x * (kQStageThreads >> 5);
    int64_t w = (int64_t)blockIdx.x * (kQStageThreads >> 5) + wib;
    auto fetch = [&](int64_t item, int slot) {
        const int64_t r = work - 1 - item, m = r / groups, j = r - m * groups;
        const uint16_t* x = g.x + m * g.ldx + j * g.group;
#pragma unroll
        for (int i = 0; i < NV; ++i)
            rf::cp_async16_zfill(&slots[slot * NV * 32 + lane + 32 * i], x + 8 * (lane + 32 * i), 16u);
    };
    if (w < work) fetch(w, 0);
    rf::cp_async_commit();
    for (int slot = 0; w < work; w += warps, slot ^= 1) {
        __syncwarp();   /* every lane is done with the other slot (the item before this one) */
        if (w + warps < work) fetch(w + warps, slot ^ 1);
        rf::cp_async_commit();
        rf::cp_async_wait<1>();   /* this item's copies are in */
        __syncwarp();
        const uint4* cur = slots + slot * NV * 32;
        /* absmax two values an instruction: the magnitudes' bf16 pairs (sign bits cleared) by the bf16x2 max, whose
         * result is one of its inputs (exact); a NaN is passed over as fmaxf passes it */
        __nv_bfloat162 m2 = __floats2bfloat162_rn(0.0f, 0.0f);
#pragma unroll 4
        for (int i = 0; i < NV; ++i) {
            const uint4 v = cur[lane + 32 * i];
            const uint32_t vw[4] = { v.x & 0x7fff7fffu, v.y & 0x7fff7fffu, v.z & 0x7fff7fffu, v.w & 0x7fff7fffu };
#pragma unroll
            for (int e = 0; e < 4; ++e) m2 = __hmax2(m2, *(const __nv_bfloat162*)&vw[e]);
        }
        float amax = fmaxf(__low2float(m2), __high2float(m2));
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const int64_t r = work - 1 - w, m = r / groups, j = r - m * groups;
        const float sc = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
        if (lane == 0) g.s[m * g.lds + j] = sc;
        const float inv = __frcp_rn(sc);
        int8_t* q = g.q + m * g.ldq + j * g.group;
#pragma unroll 2
        for (int i = 0; i < NV; ++i) *(uint2*)(q + 8 * (lane + 32 * i)) = quant_chunk8(cur[lane + 32 * i], sc, inv);
    }
    rf::cp_async_wait_all();
}

/* ------------------------------------------------------------------ host side */

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)f;
    }
    return fn;
}

/* y bf16 [M, N] with row pitch `pitch` elements, written in [32 rows][64 cols] boxes from 128-byte-swizzled
 * shared memory. */
bool bf16_store_map(CUtensorMap* map, void* base, int64_t rows, int64_t cols, int64_t pitch) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = { (cuuint64_t)cols, (cuuint64_t)rows };
    const cuuint64_t strides[1] = { (cuuint64_t)pitch * 2 };
    const cuuint32_t box[2] = { 64, 32 };
    const cuuint32_t estr[2] = { 1, 1 };
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

/* A [rows, cols] int8 matrix with row pitch `pitch` bytes, read in [box_rows, 128] tiles with 128-byte
 * swizzle; rows past the end read as zero. */
bool int8_tile_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t pitch, uint32_t box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = { (cuuint64_t)cols, (cuuint64_t)rows };
    const cuuint64_t strides[1] = { (cuuint64_t)pitch };
    const cuuint32_t box[2] = { (cuuint32_t)BK, box_rows };
    const cuuint32_t estr[2] = { 1, 1 };
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

/* One 2-CTA cluster per pair tile, as many pairs as the device holds at once (persistent). */
template <int kMode>
int launch_pairs(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap& map_y, const GemmPlan& p,
                 cudaStream_t stream) {
    static int max_pairs[kModeCount] = {};   /* per form: clusters of two a GPU can hold */
    if (cudaFuncSetAttribute(gemm_q_kernel<kMode>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
        return RAD_E_DEVICE;
    if (!max_pairs[kMode]) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (unsigned)(rf::sm_count() / 2));
        cfg.blockDim = dim3(threads_of<kMode>());
        cfg.dynamicSmemBytes = kSmemBytes;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_q_kernel<kMode>, &cfg) != cudaSuccess || n <= 0) return RAD_E_DEVICE;
        max_pairs[kMode] = n;
    }
    int pairs = p.tiles < max_pairs[kMode] ? p.tiles : max_pairs[kMode];
    if constexpr (kMode != kModeBf16 && kMode != kModeBf16Narrow) {
        if (p.g.max_ctas > 0 && p.g.max_ctas / 2 < pairs) pairs = p.g.max_ctas / 2 > 0 ? (int)(p.g.max_ctas / 2) : 1;
    }
    gemm_q_kernel<kMode><<<2 * pairs, threads_of<kMode>(), kSmemBytes, stream>>>(map_a, map_b, map_y, p);
    return rf::launch_status();
}

int launch_gemm(const RidgeFillGemmQ& g, cudaStream_t stream) {
    if (g.M == 0) return RAD_OK;
    if (g.M > 0x7fffffffLL || g.N > 0x7fffffffLL || g.K > 0x7fffffffLL) return RAD_E_SHAPE;
    CUtensorMap map_a, map_b, map_y;
    if (!int8_tile_map(&map_a, g.a, g.M, g.K, g.lda, BM) || !int8_tile_map(&map_b, g.b, g.N, g.K, g.ldb, BN / 2) ||
        !bf16_store_map(&map_y, g.y, g.M, g.N, g.ldy))
        return RAD_E_DEVICE;
    GemmPlan p;
    p.g = g;
    p.n_tiles = (int)((g.N + BN - 1) / BN);
    const int64_t tiles = ((g.M + BM2 - 1) / BM2) * p.n_tiles;
    if (tiles > 0x7fffffffLL) return RAD_E_SHAPE;
    p.tiles = (int)tiles;
    p.folds = (int)(g.K / g.group);
    p.steps_per_fold = (int)(g.group / BK);
    if (g.acc) return launch_pairs<kModeI8Dump>(map_a, map_b, map_y, p, stream);
    const bool one = p.folds == 1;   /* per-row and per-column scales: the streamed one-block fold */
    if (g.rows) return one ? launch_pairs<kModeI8RowsOne>(map_a, map_b, map_y, p, stream)
                           : launch_pairs<kModeI8Rows>(map_a, map_b, map_y, p, stream);
    return one ? launch_pairs<kModeI8One>(map_a, map_b, map_y, p, stream) : launch_pairs<kModeI8>(map_a, map_b, map_y, p, stream);
}

/* The in-projection: 250-row pair tiles (each CTA's 128 rows start 3 before its 125 output rows), one fold a
 * tile (per-row and per-column scaling). */
int launch_in_proj(const RidgeFillInProj& c, cudaStream_t stream) {
    const RidgeFillGemmQ& g = c.gemm;
    if (g.M == 0) return RAD_OK;
    if (g.M > 0x7fffffffLL || g.N > 0x7fffffffLL || g.K > 0x7fffffffLL) return RAD_E_SHAPE;
    CUtensorMap map_a, map_b, map_y;
    if (!int8_tile_map(&map_a, g.a, g.M, g.K, g.lda, BM) || !int8_tile_map(&map_b, g.b, g.N, g.K, g.ldb, BN / 2) ||
        !bf16_store_map(&map_y, g.y, g.M, g.N, g.ldy))
        return RAD_E_DEVICE;
    GemmPlan p{};
    p.g = g;
    p.c = c;
    p.n_tiles = (int)((g.N + BN - 1) / BN);
    const int64_t tiles = ((g.M + 2 * kConvRows - 1) / (2 * kConvRows)) * p.n_tiles;
    if (tiles > 0x7fffffffLL) return RAD_E_SHAPE;
    p.tiles = (int)tiles;
    p.folds = 1;
    p.steps_per_fold = (int)(g.K / BK);
    return launch_pairs<kModeI8Conv>(map_a, map_b, map_y, p, stream);
}

/* A [rows, cols] bf16 matrix with row pitch `pitch` elements, read in [box_rows, 64] tiles (128 bytes of K)
 * with 128-byte swizzle; rows past the end read as zero. */
bool bf16_tile_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t pitch, uint32_t box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = { (cuuint64_t)cols, (cuuint64_t)rows };
    const cuuint64_t strides[1] = { (cuuint64_t)pitch * 2 };
    const cuuint32_t box[2] = { (cuuint32_t)(BK / 2), box_rows };
    const cuuint32_t estr[2] = { 1, 1 };
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_gemm_bf16(const RidgeFillGemmBias& g, cudaStream_t stream) {
    if (g.M == 0) return RAD_OK;
    if (g.M > 0x7fffffffLL || g.N > 0x7fffffffLL || g.K > 0x7fffffffLL) return RAD_E_SHAPE;
    const bool narrow = g.N <= bn_of<kModeBf16Narrow>();
    const int bn = narrow ? bn_of<kModeBf16Narrow>() : BN;
    CUtensorMap map_a, map_b, map_y;
    if (!bf16_tile_map(&map_a, g.a, g.M, g.K, g.lda, BM) || !bf16_tile_map(&map_b, g.b, g.N, g.K, g.ldb, bn / 2) ||
        !bf16_store_map(&map_y, g.y, g.M, g.N, g.ldy))
        return RAD_E_DEVICE;
    GemmPlan p{};
    p.gb = g;
    p.n_tiles = (int)((g.N + BN - 1) / BN);
    const int64_t tiles = ((g.M + BM2 - 1) / BM2) * p.n_tiles;
    if (tiles > 0x7fffffffLL) return RAD_E_SHAPE;
    p.tiles = (int)tiles;
    p.folds = 1;
    p.steps_per_fold = (int)((g.K + BK / 2 - 1) / (BK / 2));   /* a ragged last step reads zeros past K */
    return narrow ? launch_pairs<kModeBf16Narrow>(map_a, map_b, map_y, p, stream)
                  : launch_pairs<kModeBf16>(map_a, map_b, map_y, p, stream);
}

}  // namespace

extern "C" int ridgefill_gemm_nt_q_device(const RadArgs* a, RadStream s) {
    RidgeFillGemmQ g;
    const int rc = ridgefill_gemm_q_parse(a, 0, &g);
    return rc != RAD_OK ? rc : launch_gemm(g, rf::as_stream(s));
}

extern "C" int ridgefill_gemm_nt_q_bias_device(const RadArgs* a, RadStream s) {
    RidgeFillGemmQ g;
    const int rc = ridgefill_gemm_q_parse(a, 1, &g);
    return rc != RAD_OK ? rc : launch_gemm(g, rf::as_stream(s));
}

extern "C" int ridgefill_gdn_in_proj_device(const RadArgs* a, RadStream s) {
    RidgeFillInProj c;
    const int rc = ridgefill_in_proj_parse(a, &c);
    return rc != RAD_OK ? rc : launch_in_proj(c, rf::as_stream(s));
}

extern "C" int ridgefill_gemm_nt_bias_device(const RadArgs* a, RadStream s) {
    RidgeFillGemmBias g;
    const int rc = ridgefill_gemm_bias_parse(a, &g);
    return rc != RAD_OK ? rc : launch_gemm_bf16(g, rf::as_stream(s));
}

template <int NV>
int launch_quant_stage(const RidgeFillQuant& g, RadStream s) {
    constexpr int smem = (kQStageThreads / 32) * 2 * NV * 32 * 16;
    static int per_sm = 0;
    if (!per_sm) {
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(quant_stage_kernel<NV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return RAD_E_DEVICE;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quant_stage_kernel<NV>, kQStageThreads, smem) != cudaSuccess ||
            per_sm <= 0)
            return RAD_E_DEVICE;
    }
    const int64_t items = g.M * (g.K / g.group);
    const int64_t blocks = (items + kQStageThreads / 32 - 1) / (kQStageThreads / 32), cap = (int64_t)rf::sm_count() * per_sm;
    quant_stage_kernel<NV><<<(unsigned)(blocks < cap ? blocks : cap), kQStageThreads, smem, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}

extern "C" int ridgefill_quant_act_device(const RadArgs* a, RadStream s) {
    RidgeFillQuant g;
    const int rc = ridgefill_quant_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.M == 0) return RAD_OK;
    const bool pow2 = (g.group & (g.group - 1)) == 0;
    const int64_t warps = g.M * (g.K / g.group);
    const int64_t blocks = (warps + 7) / 8, cap = (int64_t)rf::sm_count() * 16;
    const unsigned grid = (unsigned)(blocks < cap ? blocks : cap);
    switch (g.group) {   /* a group of 256 NV columns, staged in shared memory */
        case 256: return launch_quant_stage<1>(g, s);
        case 512: return launch_quant_stage<2>(g, s);
        case 1024: return launch_quant_stage<4>(g, s);
        case 2048: return launch_quant_stage<8>(g, s);
        case 4096: quant_reg_kernel<16><<<grid, 256, 0, rf::as_stream(s)>>>(g); return rf::launch_status();
        default: break;
    }
    if (g.K % kQSeg == 0 && pow2 && g.group < 256) {   /* small groups: a CTA a 2,048-column segment */
        const int64_t iters = (g.M * (g.K / kQSeg) + kQRows - 1) / kQRows, cap = (int64_t)rf::sm_count() * 8;
        quant_seg_kernel<<<(unsigned)(iters < cap ? iters : cap), kQThreads, 0, rf::as_stream(s)>>>(g);
        return rf::launch_status();
    }
    quant_kernel<<<grid, 256, 0, rf::as_stream(s)>>>(g);
    return rf::launch_status();
}

/* The first device-side wait error any kernel of this library recorded (0: none), optionally
 * clearing it. Synchronises the current device: a diagnostic, never called on the launch path. */
extern "C" int ridgefill_device_error(int reset) {
    const int gemm = rf::read_device_error(reset), fill = rf::gdn_device_error(reset), team = rf::peer_device_error(reset);
    if (gemm < 0 || fill < 0 || team < 0) return -1;
    return gemm ? gemm : fill ? fill : team;
}
