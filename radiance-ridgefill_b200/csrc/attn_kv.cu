/* attn_kv.cu -- ridgefill_attn_kv_fill: the gated-attention block's K/V path in the lean fill on B200 (issue site
 * arch/qwen4exp_fill.h:104-114): k_norm over each k head, the rotary embedding of k, and the paged store of k and v
 * into the layer's cache, in one pass. The reference issues radiance's in-tree k_norm, rope_k and kv_store ops,
 * whose source is not part of the checkout; the arithmetic here is that unfused chain's, each stage rounded to
 * bf16 as its own op would write it: an RMS norm with the block's k_norm weight, the half-split rotation of the
 * first rope_dim elements (with the position planes of multi-section rope when the batch carries them), and a
 * row copy into the slot slot_mapping names.
 *
 * HBM-bound: every row's k and v are read once (2 Hkv D 2 bytes) and written once into the cache (the same again;
 * k_out adds half of it). A warp takes one row t: lane l holds elements 8l..8l+7 of a head (D = 256, one 16-byte
 * word), and every head's k and v loads of the row are issued before any arithmetic. The row's rope_dim/2 angles
 * are computed one a lane in f64 while those loads are in flight and handed to the lanes that rotate through the
 * warp's shared-memory slot.
 */
#include <cuda_bf16.h>

#include <cmath>

#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxPairs = 128;      /* rope_dim / 2 at head_dim 256 */
constexpr int kHeadsInFlight = 2;   /* kv heads whose k and v words a lane loads before computing */

/* The rotation's per-pair constants, computed on the host: theta^(-2j/R) in f64 and the position plane of pair j. */
struct RopeTable {
    double inv_freq[kMaxPairs];
    unsigned char plane[kMaxPairs];
};

__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
    const uint32_t w[4] = { v.x, v.y, v.z, v.w };
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        f[2 * e] = __uint_as_float(w[e] << 16);
        f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
    }
}

/* f32 -> bf16 -> f32 (round to nearest even by the hardware conversion). */
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *(const uint32_t*)&p;
}

__global__ void __launch_bounds__(kThreads) attn_kv_kernel(const RidgeFillAttnKv g, const RopeTable rt) {
    __shared__ double inv_freq[kMaxPairs];
    __shared__ unsigned char plane[kMaxPairs];
    __shared__ float2 cs[kWarps][kMaxPairs];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int half = (int)g.rope_dim / 2;
    for (int j = threadIdx.x; j < half; j += kThreads) {
        inv_freq[j] = rt.inv_freq[j];
        plane[j] = rt.plane[j];
    }
    float w[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
        w[e] = g.w_f32 ? ((const float*)g.w)[8 * lane + e] : rf::bf16_bits_to_f32(((const uint16_t*)g.w)[8 * lane + e]);
    __syncthreads();

    /* The rotation partner of this lane's eight elements: pair (j, j + half) lies in lanes j/8 and (j + half)/8. */
    const bool rotates = 8 * lane < 2 * half, first = 8 * lane < half;
    const int partner = rotates ? (first ? lane + half / 8 : lane - half / 8) : lane;
    const int j0 = first ? 8 * lane : 8 * lane - half;
    const int64_t stride = (int64_t)gridDim.x * kWarps;
    for (int64_t t = (int64_t)blockIdx.x * kWarps + warp; t < g.T; t += stride) {
        const int slot = g.slots[t];
        const bool store = slot >= 0 && (int64_t)slot < g.n_slots;
        int p = 0;
        if (lane < g.n_planes) p = g.pos[lane * g.pos_plane + t];
        const int pos0 = __shfl_sync(0xffffffffu, p, 0), pos1 = __shfl_sync(0xffffffffu, p, 1),
                  pos2 = __shfl_sync(0xffffffffu, p, 2);
        for (int h0 = 0; h0 < g.n_head_kv; h0 += kHeadsInFlight) {
            uint4 kw[kHeadsInFlight], vw[kHeadsInFlight];
#pragma unroll
            for (int i = 0; i < kHeadsInFlight; ++i)
                if (h0 + i < g.n_head_kv) {
                    kw[i] = __ldcs((const uint4*)(g.k + t * g.k_row + (h0 + i) * g.k_head + 8 * lane));
                    vw[i] = __ldcs((const uint4*)(g.v + t * g.v_row + (h0 + i) * g.v_head + 8 * lane));
                }
            if (h0 == 0) {   /* the row's angles while the loads are in flight */
                __syncwarp();   /* the previous row's reads of cs are done */
                for (int j = lane; j < half; j += 32) {
                    const int pl = plane[j];
                    const double a = (double)(pl == 0 ? pos0 : pl == 1 ? pos1 : pos2) * inv_freq[j];
                    double sv, cv;
                    sincos(a, &sv, &cv);
                    cs[warp][j] = make_float2((float)cv, (float)sv);
                }
                __syncwarp();
            }
#pragma unroll
            for (int i = 0; i < kHeadsInFlight; ++i) {
                if (h0 + i >= g.n_head_kv) break;
                const int64_t h = h0 + i;
                float x[8], kn[8], pr[8], out[8];
                unpack8(kw[i], x);
                float ss = 0.f;
#pragma unroll
                for (int e = 0; e < 8; ++e) ss = __fmaf_rn(x[e], x[e], ss);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
                const float r = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / 256.0f), g.eps)));
#pragma unroll
                for (int e = 0; e < 8; ++e) kn[e] = round_bf16(__fmul_rn(__fmul_rn(x[e], r), w[e]));
#pragma unroll
                for (int e = 0; e < 8; ++e) pr[e] = __shfl_sync(0xffffffffu, kn[e], partner);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    out[e] = kn[e];
                    if (rotates) {
                        const float2 c = cs[warp][j0 + e];
                        const float ps = __fmul_rn(pr[e], c.y);
                        out[e] = __fmaf_rn(kn[e], c.x, first ? -ps : ps);
                    }
                }
                const uint4 ko = make_uint4(bf16x2(out[0], out[1]), bf16x2(out[2], out[3]), bf16x2(out[4], out[5]),
                                            bf16x2(out[6], out[7]));
                if (g.k_out) *(uint4*)(g.k_out + t * g.ko_row + h * g.ko_head + 8 * lane) = ko;
                if (store) {
                    uint16_t* dst = g.cache + (int64_t)slot * g.c_slot + h * g.c_head + 8 * lane;
                    *(uint4*)dst = ko;
                    *(uint4*)(dst + g.c_kv) = vw[i];
                }
            }
        }
    }
}

}  // namespace

extern "C" int ridgefill_attn_kv_fill_device(const RadArgs* a, RadStream s) {
    RidgeFillAttnKv g;
    const int rc = ridgefill_attn_kv_parse(a, &g);
    if (rc != RAD_OK) return rc;
    if (g.T == 0) return RAD_OK;
    RopeTable rt{};
    const int half = (int)g.rope_dim / 2;
    for (int j = 0; j < half; ++j) {
        rt.inv_freq[j] = std::pow(g.theta, -2.0 * (double)j / (double)g.rope_dim);
        int pl = 0;
        if (g.n_planes == 3 && g.mode == RIDGEFILL_ROPE_MROPE)
            pl = j < g.sections[0] ? 0 : j < g.sections[0] + g.sections[1] ? 1 : 2;
        else if (g.n_planes == 3 && g.mode == RIDGEFILL_ROPE_IMROPE)
            pl = (j % 3 == 1 && j < 3 * g.sections[1]) ? 1 : (j % 3 == 2 && j < 3 * g.sections[2]) ? 2 : 0;
        rt.plane[j] = (unsigned char)pl;
    }
    static int per_sm = 0;   /* resident CTAs a SM */
    if (!per_sm && (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_kv_kernel, kThreads, 0) != cudaSuccess ||
                    per_sm <= 0))
        return RAD_E_DEVICE;
    const int64_t blocks = (g.T + kWarps - 1) / kWarps, cap = (int64_t)rf::sm_count() * per_sm;
    attn_kv_kernel<<<(unsigned)(blocks < cap ? blocks : cap), kThreads, 0, rf::as_stream(s)>>>(g, rt);
    return rf::launch_status();
}
