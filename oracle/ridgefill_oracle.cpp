/* ridgefill_oracle.cpp -- TEST INFRASTRUCTURE, not the product. The CPU restatement of the RidgeFill
 * ops that the CUDA rows are checked against, and the CPU baseline that bench.py times beside them.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU legs load it.
 *
 * Two parts:
 *  1. Host rows for the reference's seven ops, restating kernels/host_ref.cpp (operand checks :16-282,
 *     mask :284-330, rho :332-356, state_correct :358-386, state_read :388-407, select/drop :409-431,
 *     hazard :433-472) behind the same plugin exports (kernels/rows.cpp:382-399), so the reference's
 *     own harness (tests/kernel_test.cpp) can run against this library. The formulas are restated here
 *     rather than taken from the product header, so oracle and product are two implementations.
 *     PINNED: tests/kernel_test.cpp's host cases (known answers, rho_numpy.txt, rowsel_quick9.json)
 *     pass against this library, and tests compare it with the reference's host rows compiled from
 *     source (oracle/_ref).
 *  2. Plain-pointer oracles for the ops the reference does not contain (their arithmetic lives in
 *     radiance's libr4d and in-tree ops, absent): the activation quantiser, the int8 projector GEMM with
 *     its f32 block fold, the bf16 GEMM with bias / SiLU / residual, the gated delta rule, the DeltaNet
 *     input preparation (convolution, SiLU, L2 norm, gate) and the attention block's K/V cache write (RMS
 *     norm, rotary embedding, paged store). PARITY UNPINNED for all but the quantiser's
 *     rounding rule (no reference source, test or fixture exists for them; the gate is the reference's
 *     softplus rule, kernels/ridgefill.h:93-97); the quantiser's rounding rule is the reference's
 *     quantise_i8 (tools/ridgefill_projector.py:333-344) with an f32 scale.
 *
 * Built with -ffp-contract=off so `x + s*c` rounds twice, as the reference's host rows do
 * (kernels/CMakeLists.txt:48-51).
 */
#include "rad_plugin.h"
#include "ridgefill_schemas.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

/* ================================================================== formulas (restated) */

uint32_t lowbias32(uint32_t x) {   /* kernels/ridgefill.h:66-71 */
    x = (x ^ (x >> 16)) * 0x7feb352dU;
    x = (x ^ (x >> 15)) * 0x846ca68bU;
    return x ^ (x >> 16);
}

uint32_t position_key(long long seed, uint32_t pos) {   /* kernels/ridgefill.h:77-81 */
    const unsigned long long s = (unsigned long long)seed;
    const uint32_t mixed = lowbias32((uint32_t)s ^ lowbias32((uint32_t)(s >> 32)));
    return lowbias32(mixed ^ (pos * 0x9E3779B9U + 0x7F4A7C15U));
}

float clamp_ratio(float n, float d) {   /* kernels/ridgefill.h:86-91 */
    if (!(d > 0.0f)) return 1.0f;
    float r = n / d;
    if (!(r > 0.0f)) r = 0.0f;
    return r < 1.0f ? r : 1.0f;
}

float softplus2(float x) {   /* kernels/ridgefill.h:94-97, threshold 20 */
    if (x > 20.0f) return x;
    return x > 0.0f ? x + log1pf(expf(-x)) : log1pf(expf(x));
}

float bf16f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

uint16_t f2bf(float f) {   /* round to nearest even */
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

const int32_t* i32(const RadTensor* t) { return (const int32_t*)t->data; }
bool packed(const RadTensor* t) { return rad_tensor_is_contiguous(t); }

/* Extent of axes 2.. (one slot-head's worth of a LINEAR cache). */
int64_t tail_elems(const RadTensor* t) {
    int64_t n = 1;
    for (uint32_t i = 2; i < t->rank; ++i) n *= t->shape[i];
    return n;
}

/* Stride between N and D of an ND pool (its one trailing axis of extent 2), 0 if not a pair. */
int64_t nd_step(const RadTensor* t) {
    if (t->rank < 3 || tail_elems(t) != 2) return 0;
    for (uint32_t i = 2; i < t->rank; ++i)
        if (t->shape[i] == 2) return t->stride[i];
    return 0;
}

/* A slot index [n_seq] or [n_seq, pitch]; column 0 is the slot. */
int slot_index(const RadTensor* t, int64_t* rows, int64_t* pitch) {
    if (t->dtype != RAD_I32) return RAD_E_DTYPE;
    if (t->rank < 1 || t->rank > 2 || t->stride[t->rank - 1] != 1) return RAD_E_STRIDE;
    *rows = t->shape[0];
    *pitch = t->rank == 2 ? t->stride[0] : 1;
    return RAD_OK;
}

int bounds_operand(const RadTensor* t, int64_t need, const int32_t** out) {
    *out = nullptr;
    if (!t) return RAD_OK;
    if (t->dtype != RAD_I32) return RAD_E_DTYPE;
    if (!packed(t)) return RAD_E_STRIDE;
    if (rad_tensor_numel(t) < need) return RAD_E_SHAPE;
    *out = i32(t);
    return RAD_OK;
}

int mode_of(const char* s, std::initializer_list<const char*> names) {
    int i = 0;
    for (const char* n : names) {
        if (s && std::strcmp(s, n) == 0) return i;
        ++i;
    }
    return -1;
}

/* ================================================================== ridgefill_mask (host_ref.cpp:64-104, 284-330) */

enum { M_NONE, M_CLASS, M_RANDOM, M_ALL, M_STEP };

int mask_row(const RadArgs* a, RadStream) {
    const RadTensor *cu = rad_arg_in(a, 0), *tok = rad_arg_in(a, 1), *pos = rad_arg_in(a, 2), *score = rad_arg_in(a, 3);
    const RadTensor *mask = rad_arg_in(a, 4), *bounds = rad_arg_in(a, 5), *zeros = rad_arg_in(a, 6);
    const int mode = mode_of(rad_args_gets(a, "mode"), { "none", "class", "random", "all", "step" });
    const double share = rad_args_getf_or(a, "share", NAN);
    long long seed = 0;
    const bool ranked = mode == M_CLASS || mode == M_RANDOM;
    if (!cu || !tok || !pos || !mask || !bounds || (ranked && !score) || mode < 0 || !rad_args_geti(a, "seed", &seed) ||
        !(share >= 0.0 && share <= 1.0))
        return RAD_E_INVAL;
    for (const RadTensor* t : { cu, tok, pos, mask, bounds })
        if (t->dtype != RAD_I32) return RAD_E_DTYPE;
    if ((score && score->dtype != RAD_F32) || (zeros && zeros->dtype != RAD_I32)) return RAD_E_DTYPE;
    for (const RadTensor* t : { cu, tok, mask, bounds, score, zeros })
        if (t && !packed(t)) return RAD_E_STRIDE;
    const int64_t b = rad_tensor_numel(tok);
    if (pos->rank < 1 || pos->rank > 2 || pos->shape[pos->rank - 1] < b || rad_tensor_numel(cu) < 2 ||
        rad_tensor_numel(bounds) < 4)
        return RAD_E_SHAPE;
    const int64_t n = rad_tensor_numel(mask), pstride = pos->stride[pos->rank - 1];
    const int64_t s = i32(cu)[0], e = i32(cu)[1];
    if (s < 0 || s > e || e > n) return RAD_E_INVAL;
    const int64_t bulk = std::min(std::max(b, s), e);
    const int64_t from = mode == M_STEP && bulk > s ? 0 : s;
    int32_t* m = (int32_t*)mask->data;
    std::fill(m, m + n, 0);
    const int64_t vocab = score ? rad_tensor_numel(score) : 0;
    const float* table = score ? (const float*)score->data : nullptr;
    /* The window's rows and their keys. A matching row has a finite table score. */
    const int64_t w = bulk - from;
    std::vector<float> cls((size_t)std::max<int64_t>(w, 0), -INFINITY);
    std::vector<uint32_t> hsh((size_t)std::max<int64_t>(w, 0), 0);
    int64_t matches = 0;
    for (int64_t j = 0; j < w && ranked; ++j) {
        const int32_t id = i32(tok)[from + j];
        const float v = id >= 0 && id < vocab ? table[id] : -INFINITY;
        cls[(size_t)j] = std::isfinite(v) ? v : -INFINITY;
        hsh[(size_t)j] = position_key(seed, (uint32_t)i32(pos)[(from + j) * pstride]);
        matches += cls[(size_t)j] > -INFINITY;
    }
    const int64_t k = (int64_t)std::nearbyint(share * (double)matches);   /* half to even */
    /* The k rows ranked first are kept: order the candidates by the mode's key, ties by row. */
    std::vector<int64_t> order;
    for (int64_t j = 0; j < w; ++j)
        if ((mode == M_CLASS && cls[(size_t)j] > -INFINITY) || mode == M_RANDOM) order.push_back(j);
    if (mode == M_CLASS)
        std::stable_sort(order.begin(), order.end(), [&](int64_t x, int64_t y) { return cls[(size_t)x] > cls[(size_t)y]; });
    if (mode == M_RANDOM)
        std::stable_sort(order.begin(), order.end(), [&](int64_t x, int64_t y) { return hsh[(size_t)x] < hsh[(size_t)y]; });
    std::vector<char> kept((size_t)std::max<int64_t>(w, 0), mode == M_ALL ? 1 : 0);
    for (int64_t r = 0; r < (int64_t)order.size() && r < k; ++r) kept[(size_t)order[(size_t)r]] = 1;
    for (int64_t j = 0; j < w; ++j) m[from + j] = kept[(size_t)j] ? 0 : 1;
    int32_t* bo = (int32_t*)bounds->data;
    bo[0] = (int32_t)s; bo[1] = (int32_t)bulk; bo[2] = (int32_t)bulk; bo[3] = (int32_t)e;
    const int64_t nz = zeros ? rad_tensor_numel(zeros) : 0;
    for (int64_t i = 0; i < nz; ++i) ((int32_t*)zeros->data)[i] = 0;
    return RAD_OK;
}

/* ================================================================== ridgefill_rho_update (host_ref.cpp:106-145, 332-356) */

int rho_row(const RadArgs* a, RadStream) {
    const RadTensor *av = rad_arg_in(a, 0), *mask = rad_arg_in(a, 1), *alog = rad_arg_in(a, 2), *dtb = rad_arg_in(a, 3);
    const RadTensor *nd = rad_arg_in(a, 4), *sidx = rad_arg_in(a, 5);
    if (!av || !mask || !alog || !dtb || !nd || !sidx) return RAD_E_INVAL;
    if ((av->dtype != RAD_BF16 && av->dtype != RAD_F32) || mask->dtype != RAD_I32 || alog->dtype != RAD_F32 ||
        dtb->dtype != RAD_F32 || nd->dtype != RAD_F32)
        return RAD_E_DTYPE;
    int64_t n_seq = 0, pitch = 0;
    const int32_t* bounds = nullptr;
    int rc = slot_index(sidx, &n_seq, &pitch);
    if (rc == RAD_OK) rc = bounds_operand(rad_arg_in(a, 6), 1, &bounds);
    if (rc != RAD_OK) return rc;
    if (av->rank != 2 || !packed(mask) || !packed(alog) || !packed(dtb)) return RAD_E_STRIDE;
    long long heads = 0;
    if (!rad_args_geti(a, "n_head", &heads)) return RAD_E_INVAL;
    const int64_t n = av->shape[0], H = av->shape[1], inner = nd_step(nd);
    if (heads != H || rad_tensor_numel(mask) < n || rad_tensor_numel(alog) != heads || rad_tensor_numel(dtb) != heads ||
        nd->shape[1] != heads || inner == 0 || n_seq != 1)
        return RAD_E_SHAPE;
    const int32_t slot = i32(sidx)[0];
    if (slot < 0 || slot >= nd->shape[0]) return RAD_OK;
    const int64_t first = bounds ? std::min<int64_t>(std::max<int64_t>(bounds[0], 0), n) : 0;
    for (int64_t h = 0; h < H; ++h) {
        float* p = (float*)nd->data + slot * nd->stride[0] + h * nd->stride[1];
        float N = p[0], D = p[inner];
        const float rate = expf(((const float*)alog->data)[h]), bias = ((const float*)dtb->data)[h];
        for (int64_t t = first; t < n; ++t) {
            const int64_t at = t * av->stride[0] + h * av->stride[1];
            const float x = av->dtype == RAD_BF16 ? bf16f(((const uint16_t*)av->data)[at]) : ((const float*)av->data)[at];
            const float e = expf(-rate * softplus2(x + bias));
            D = e * D + 1.0f;
            N = e * N + (float)i32(mask)[t];
        }
        p[0] = N;
        p[inner] = D;
    }
    return RAD_OK;
}

/* ================================================================== ridgefill_state_correct (host_ref.cpp:147-197, 358-386) */

int correct_row(const RadArgs* a, RadStream) {
    const RadTensor *st = rad_arg_in(a, 0), *sidx = rad_arg_in(a, 1), *ap = rad_arg_in(a, 2), *aidx = rad_arg_in(a, 3);
    const RadTensor *c = rad_arg_in(a, 4), *nd = rad_arg_in(a, 5), *nidx = rad_arg_in(a, 6);
    if (!st || !sidx || !ap || !aidx || !c || (!nd) != (!nidx)) return RAD_E_INVAL;
    if (st->dtype != RAD_F32 || ap->dtype != RAD_F32 || c->dtype != RAD_F32 || (nd && nd->dtype != RAD_F32))
        return RAD_E_DTYPE;
    const int apply = mode_of(rad_args_gets(a, "mode"), { "undo", "apply" });
    const double alpha = rad_args_getf_or(a, "alpha", NAN);
    long long heads = 0, sd0 = 0, sd1 = 0;
    if (apply < 0 || !rad_args_geti(a, "n_head", &heads) || !rad_args_geti(a, "sd0", &sd0) ||
        !rad_args_geti(a, "sd1", &sd1) || (apply && !std::isfinite(alpha)))
        return RAD_E_INVAL;
    int64_t n_seq = 0, st_pitch = 0, ap_rows = 0, ap_pitch = 0, nd_rows = 0, nd_pitch = 0;
    const int32_t* bounds = nullptr;
    int rc = slot_index(sidx, &n_seq, &st_pitch);
    if (rc == RAD_OK) rc = slot_index(aidx, &ap_rows, &ap_pitch);
    if (rc == RAD_OK && nidx) rc = slot_index(nidx, &nd_rows, &nd_pitch);
    if (rc == RAD_OK) rc = bounds_operand(rad_arg_in(a, 7), 2, &bounds);
    if (rc != RAD_OK) return rc;
    if (ap_rows != n_seq || (nidx && nd_rows != n_seq)) return RAD_E_SHAPE;
    if (st->rank != 4 || st->shape[1] != heads || st->shape[2] != sd0 || st->shape[3] != sd1 || !packed(c) ||
        rad_tensor_numel(c) != heads * sd0 * sd1 || ap->rank < 2 || ap->shape[1] != heads || tail_elems(ap) != 1 ||
        (nd && (nd->shape[1] != heads || nd_step(nd) == 0)))
        return RAD_E_SHAPE;
    if (bounds && !(bounds[1] > bounds[0])) return RAD_OK;   /* no bulk row: nothing written */
    const float al = (float)alpha;
    const int64_t inner = nd ? nd_step(nd) : 0;
    for (int64_t s = 0; s < n_seq; ++s) {
        const int64_t ss = i32(sidx)[s * st_pitch], as = i32(aidx)[s * ap_pitch], ns = nd ? i32(nidx)[s * nd_pitch] : 0;
        if (ss < 0 || ss >= st->shape[0] || as < 0 || as >= ap->shape[0] || (nd && (ns < 0 || ns >= nd->shape[0])))
            continue;
        for (int64_t h = 0; h < heads; ++h) {
            float* applied = (float*)ap->data + as * ap->stride[0] + h * ap->stride[1];
            float scale = *applied;
            if (apply) {
                const float* q = nd ? (const float*)nd->data + ns * nd->stride[0] + h * nd->stride[1] : nullptr;
                scale = al * (q ? clamp_ratio(q[0], q[inner]) : 1.0f);
            }
            float* x = (float*)st->data + ss * st->stride[0] + h * st->stride[1];
            const float* cc = (const float*)c->data + h * sd0 * sd1;
            if (scale != 0.0f)
                for (int64_t i = 0; i < sd0; ++i)
                    for (int64_t j = 0; j < sd1; ++j) {
                        float& v = x[i * st->stride[2] + j * st->stride[3]];
                        const float d = scale * cc[i * sd1 + j];
                        v = apply ? v + d : v - d;
                    }
            *applied = apply ? scale : 0.0f;
        }
    }
    return RAD_OK;
}

/* ================================================================== ridgefill_state_read (host_ref.cpp:199-221, 388-407) */

int state_read_row(const RadArgs* a, RadStream) {
    const RadTensor *st = rad_arg_in(a, 0), *sidx = rad_arg_in(a, 1), *out = rad_arg_in(a, 2);
    long long heads = 0, sd0 = 0, sd1 = 0;
    if (!st || !sidx || !out || !rad_args_geti(a, "n_head", &heads) || !rad_args_geti(a, "sd0", &sd0) ||
        !rad_args_geti(a, "sd1", &sd1))
        return RAD_E_INVAL;
    if (st->dtype != RAD_F32 || out->dtype != RAD_F32) return RAD_E_DTYPE;
    int64_t n_seq = 0, pitch = 0;
    const int rc = slot_index(sidx, &n_seq, &pitch);
    if (rc != RAD_OK) return rc;
    if (!packed(out)) return RAD_E_STRIDE;
    if (st->rank != 4 || st->shape[1] != heads || st->shape[2] != sd0 || st->shape[3] != sd1 ||
        rad_tensor_numel(out) < n_seq * heads * sd0 * sd1)
        return RAD_E_SHAPE;
    float* o = (float*)out->data;
    for (int64_t s = 0; s < n_seq; ++s) {
        const int64_t slot = i32(sidx)[s * pitch];
        const bool inside = slot >= 0 && slot < st->shape[0];
        for (int64_t h = 0; h < heads; ++h)
            for (int64_t i = 0; i < sd0; ++i)
                for (int64_t j = 0; j < sd1; ++j)
                    *o++ = inside ? ((const float*)st->data)[slot * st->stride[0] + h * st->stride[1] +
                                                             i * st->stride[2] + j * st->stride[3]]
                                  : 0.0f;
    }
    return RAD_OK;
}

/* ================================================================== ridgefill_select / drop (host_ref.cpp:223-282, 409-431) */

struct Pair { const unsigned char* src; unsigned char* dst; int64_t sp, dp, width; };

int select_pair(const RadTensor* src, const RadTensor* dst, int64_t n, Pair* p) {
    *p = Pair{};
    if (!src && !dst) return RAD_OK;
    if (!src || !dst) return RAD_E_INVAL;
    const int bits = rad_dtype_bits(src->dtype);
    if (dst->dtype != src->dtype || bits <= 0 || bits % 8) return RAD_E_DTYPE;
    if (src->rank != 2 || dst->rank != 2 || src->shape[1] != dst->shape[1] || src->shape[0] < n || dst->shape[0] < n)
        return RAD_E_SHAPE;
    if (src->stride[1] != 1 || dst->stride[1] != 1) return RAD_E_STRIDE;
    const int64_t bytes = bits / 8;
    *p = Pair{ (const unsigned char*)src->data, (unsigned char*)dst->data, src->stride[0] * bytes,
               dst->stride[0] * bytes, src->shape[1] * bytes };
    return RAD_OK;
}

int select_row(const RadArgs* a, RadStream) {
    const RadTensor* mask = rad_arg_in(a, 0);
    if (!mask || !rad_arg_in(a, 1) || !rad_arg_in(a, 4)) return RAD_E_INVAL;
    if (mask->dtype != RAD_I32) return RAD_E_DTYPE;
    if (!packed(mask)) return RAD_E_STRIDE;
    const int64_t n = rad_tensor_numel(mask);
    Pair pairs[3];
    for (int k = 0; k < 3; ++k) {
        const int rc = select_pair(rad_arg_in(a, 1 + k), rad_arg_in(a, 4 + k), n, &pairs[k]);
        if (rc != RAD_OK) return rc;
    }
    for (int64_t i = 0; i < n; ++i) {
        if (i32(mask)[i] != 1) continue;
        for (const Pair& p : pairs)
            if (p.src) std::memmove(p.dst + i * p.dp, p.src + i * p.sp, (size_t)p.width);
    }
    return RAD_OK;
}

int drop_row(const RadArgs* a, RadStream) {
    const RadTensor *mask = rad_arg_in(a, 0), *ids = rad_arg_in(a, 1);
    long long top_k = -1;
    if (!mask || !ids || !rad_args_geti(a, "top_k", &top_k) || top_k < 0) return RAD_E_INVAL;
    if (mask->dtype != RAD_I32 || ids->dtype != RAD_I32) return RAD_E_DTYPE;
    if (!packed(mask) || (ids->rank == 2 && ids->stride[1] != 1)) return RAD_E_STRIDE;
    const int64_t n = rad_tensor_numel(mask);
    if (ids->rank != 2 || ids->shape[0] < n || ids->shape[1] < top_k) return RAD_E_SHAPE;
    for (int64_t i = 0; i < n; ++i)
        if (i32(mask)[i] == 1)
            for (int64_t j = 0; j < top_k; ++j) ((int32_t*)ids->data)[i * ids->stride[0] + j] = -1;
    return RAD_OK;
}

/* ================================================================== ridgefill_hazard (host_ref.cpp:435-472, ridgefill.h:232-249) */

int hazard_row(const RadArgs* a, RadStream) {
    const RadTensor *cu = rad_arg_in(a, 0), *pos = rad_arg_in(a, 1), *span = rad_arg_in(a, 3);
    const RadTensor *meta = rad_arg_in(a, 4), *idx = rad_arg_in(a, 5), *cnt = rad_arg_in(a, 6);
    if (!cu || !pos || !meta || !idx || !cnt) return RAD_E_INVAL;
    if (cu->dtype != RAD_I32 || pos->dtype != RAD_I32 || meta->dtype != RAD_F32 || cnt->dtype != RAD_F32)
        return RAD_E_DTYPE;
    if (!packed(cu) || !packed(cnt)) return RAD_E_STRIDE;
    int64_t rows = 0, pitch = 0;
    const int32_t* bounds = nullptr;
    int rc = slot_index(idx, &rows, &pitch);
    if (rc == RAD_OK) rc = bounds_operand(rad_arg_in(a, 2), 2, &bounds);
    if (rc != RAD_OK) return rc;
    if (rows < 1 || rad_tensor_numel(cu) < 2 || rad_tensor_numel(cnt) < 1 || pos->rank < 1 || pos->rank > 2 ||
        meta->rank < 2 || meta->shape[meta->rank - 1] != 2 || meta->stride[meta->rank - 1] != 1)
        return RAD_E_SHAPE;
    const int64_t s = i32(cu)[0], e = i32(cu)[1];
    if (s < 0 || s > e) return RAD_E_INVAL;
    const int32_t slot = i32(idx)[0];
    if (slot < 0 || slot >= meta->shape[0]) return RAD_OK;
    const int64_t ps = pos->stride[pos->rank - 1];
    float* m = (float*)meta->data + slot * meta->stride[0];
    float* count = (float*)cnt->data;
    const int64_t sp = span ? rad_tensor_numel(span) : 0;
    if (sp > 0 && e > s) {
        const int64_t P = i32(pos)[s * ps], before = sp - (e - s);
        const int64_t lo = std::max<int64_t>(P - before, (int64_t)m[1]), hi = std::min<int64_t>(P, (int64_t)m[0]);
        if (before > 0 && hi > lo) {
            count[0] += (float)(hi - lo);
            m[1] = (float)hi;
        }
    }
    if (bounds && bounds[1] > bounds[0]) m[0] = (float)(i32(pos)[(int64_t)(bounds[1] - 1) * ps] + 1);
    return RAD_OK;
}

/* ================================================================== the row table */

using namespace ridgefill_schema;

const RadConstraint kMaskModes[] = { RAD_CIN("mode", "none class random all step") };
const RadConstraint kCorrectModes[] = { RAD_CIN("mode", "undo apply") };

#define ORACLE_ROW(nm, op, cons, ncons, fn, shp)                                                                  \
    { nm, op, "ridgefill_oracle", "CPU restatement of the reference host row (test infrastructure)", "any",       \
      "as the schema", RAD_DOMAIN_HOST, 0, cons, ncons, nullptr, 0, nullptr, nullptr, nullptr, fn, nullptr,       \
      nullptr, nullptr, shp, nullptr, nullptr, nullptr, nullptr }

const RadKernelInfo kRows[] = {
    ORACLE_ROW("ridgefill_mask_oracle", "ridgefill_mask", kMaskModes, 1, mask_row, shape_mask),
    ORACLE_ROW("ridgefill_select_oracle", "ridgefill_select", nullptr, 0, select_row, shape_select),
    ORACLE_ROW("ridgefill_drop_rows_oracle", "ridgefill_drop_rows", nullptr, 0, drop_row, shape_drop),
    ORACLE_ROW("ridgefill_rho_update_oracle", "ridgefill_rho_update", nullptr, 0, rho_row, shape_rho),
    ORACLE_ROW("ridgefill_state_correct_oracle", "ridgefill_state_correct", kCorrectModes, 1, correct_row, shape_correct),
    ORACLE_ROW("ridgefill_state_read_oracle", "ridgefill_state_read", nullptr, 0, state_read_row, shape_state_read),
    ORACLE_ROW("ridgefill_hazard_oracle", "ridgefill_hazard", nullptr, 0, hazard_row, shape_hazard),
};

const RadPluginInfo kInfo = { RAD_PLUGIN_KERNEL, "ridgefill_oracle", "0.1.0",
                              "CPU restatement of the RidgeFill host rows (test infrastructure)", "host" };

}  // namespace

extern "C" {

uint32_t rad_plugin_abi_version(void) { return RAD_ABI_VERSION; }
const RadPluginInfo* rad_plugin_info(void) { return &kInfo; }
/* Only the reference's nine schemas: this library stands in for the reference's host rows. */
int rad_kernel_schema_count(void) { return kReferenceSchemas; }
const RadOpSchema* rad_kernel_schema_at(int i) { return i >= 0 && i < kReferenceSchemas ? &kSchemas[i] : nullptr; }
int rad_kernel_count(void) { return (int)(sizeof kRows / sizeof kRows[0]); }
const RadKernelInfo* rad_kernel_at(int i) { return i >= 0 && i < rad_kernel_count() ? &kRows[i] : nullptr; }
int rad_kernel_concurrent(int) { return 0; }

/* ================================================================== new-op oracles (plain pointers) */

/* Activation codes: per `group` columns of row m, s = absmax / 127 in f32 (1 when the group is all
 * zero, the value quant_act_i8g writes: tools/ridgefill_projector.py:341), q = round-half-even(x / s)
 * clamped to [-127, 127] (tools/ridgefill_projector.py:342). */
void oracle_quant_act_i8g(const uint16_t* x, int64_t ldx, int64_t M, int64_t K, int64_t group, int8_t* q,
                          int64_t ldq, float* s, int64_t lds) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m)
        for (int64_t g0 = 0; g0 < K; g0 += group) {
            float amax = 0.0f;
            for (int64_t k = g0; k < g0 + group; ++k) amax = std::max(amax, std::fabs(bf16f(x[m * ldx + k])));
            const float sc = amax == 0.0f ? 1.0f : amax / 127.0f;
            s[m * lds + g0 / group] = sc;
            for (int64_t k = g0; k < g0 + group; ++k) {
                const float r = std::nearbyint(bf16f(x[m * ldx + k]) / sc);
                q[m * ldq + k] = (int8_t)std::min(127.0f, std::max(-127.0f, r));
            }
        }
}

/* The weight's i8*bf16[1x128] encoding as tools/ridgefill_projector.py:333-344 writes it: scale =
 * bf16(absmax / 127) (1 for a zero group), code = round-half-even(w / scale) clamped to +-127. */
void oracle_quantise_weight_i8(const float* w, int64_t N, int64_t K, int8_t* codes, uint16_t* scale) {
    for (int64_t n = 0; n < N; ++n)
        for (int64_t g0 = 0; g0 < K; g0 += 128) {
            float amax = 0.0f;
            for (int64_t k = g0; k < g0 + 128; ++k) amax = std::max(amax, std::fabs(w[n * K + k]));
            uint16_t sb = f2bf(amax / 127.0f);
            if (amax == 0.0f) sb = f2bf(1.0f);
            scale[n * (K / 128) + g0 / 128] = sb;
            const float sc = bf16f(sb);
            for (int64_t k = g0; k < g0 + 128; ++k) {
                const float r = std::nearbyint(w[n * K + k] / sc);
                codes[n * K + k] = (int8_t)std::min(127.0f, std::max(-127.0f, r));
            }
        }
}

/* ridgefill_gemm_nt_q (+ bias): per block j of `group` columns, the exact int32 dot; then in block
 * order t = (float)dot * a_scale[m, j] (rounded), acc = fma(t, b_scale[j, n], acc) (one rounding);
 * y = bf16(acc), and with a bias y = bf16((float)y + bias[n]): the gemm_nt_q + add pair
 * (arch/ridgefill_layer.h:77-79). b_scale is the stored form f32 [K/group, N]. `acc_out` (optional)
 * receives every block's int32 dot as [M, N, K/group]. Rows [m0, m1) only, so a caller can sample. */
void oracle_gemm_nt_q(const int8_t* a, int64_t lda, const float* a_scale, int64_t ldas, const int8_t* b, int64_t ldb,
                      const float* b_scale, const uint16_t* bias, uint16_t* y, int64_t ldy, int32_t* acc_out,
                      int64_t M, int64_t N, int64_t K, int64_t group, int64_t m0, int64_t m1) {
    const int64_t blocks = K / group;
    (void)M;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t m = m0; m < m1; ++m)
        for (int64_t n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int64_t j = 0; j < blocks; ++j) {
                int32_t dot = 0;
                const int8_t* pa = a + m * lda + j * group;
                const int8_t* pb = b + n * ldb + j * group;
                for (int64_t k = 0; k < group; ++k) dot += (int32_t)pa[k] * (int32_t)pb[k];
                if (acc_out) acc_out[(m * N + n) * blocks + j] = dot;
                const float t = (float)dot * a_scale[m * ldas + j];
                acc = std::fma(t, b_scale[j * N + n], acc);
            }
            uint16_t out = f2bf(acc);
            if (bias) out = f2bf(bf16f(out) + bf16f(bias[n]));
            y[m * ldy + n] = out;
        }
}

/* ridgefill_gdn_conv_prep: the DeltaNet block's input preparation (issue site arch/qwen4exp_fill.h:41-50; the
 * op itself is radiance's and absent, so this is the published Gated DeltaNet input path restated, with the
 * reference's gate, kernels/ridgefill.h:93-97). x bf16 [T, C] (row pitch x_row), C = 2 Hk 128 + Hv 128 channels
 * q|k|v; per sequence i of cu (bounds clamped into [0, T]) and row t, channel c:
 *     u = bias[c] + w[c,0] x[t-3] + w[c,1] x[t-2] + w[c,2] x[t-1] + w[c,3] x[t]   (f32 fma in that order; rows
 *         before the sequence start from state[idx[i]] when ctx[i] > 0 and the slot is in the pool, else zero)
 *     y = u / (1 + exp(-u));  q, k heads: y / sqrt(sum_head y^2 + 1e-6);  bf16
 *     g[t,h] = -exp(A_log[h]) softplus(a[t,h] + dt_bias[h]);  beta[t,h] = 1 / (1 + exp(-b[t,h]))
 * then state[idx[i]] = the last three input rows of (history, rows). Outputs dense: q, k [T, Hk, 128],
 * v [T, Hv, 128], g, beta [T, Hv]; rows outside every sequence are left as they are. */
void oracle_gdn_conv_prep(const uint16_t* x, int64_t x_row, const uint16_t* w, const uint16_t* bias, const float* a_log,
                          const float* dt_bias, uint16_t* state, int64_t n_states, const int32_t* cu, int64_t n_seq,
                          const uint16_t* a, const uint16_t* b, const int32_t* idx, const int32_t* ctx, uint16_t* q,
                          uint16_t* k, uint16_t* v, float* g, float* beta, int64_t T, int64_t Hk, int64_t Hv) {
    const int64_t C = 2 * Hk * 128 + Hv * 128;
    std::vector<float> hist((size_t)(3 * C)), y((size_t)C);
    for (int64_t i = 0; i < n_seq; ++i) {
        const int64_t s0 = std::min(std::max((int64_t)cu[i], (int64_t)0), T);
        const int64_t e0 = std::min(std::max((int64_t)cu[i + 1], s0), T);
        const int64_t slot = idx[i];
        const bool in_pool = slot >= 0 && slot < n_states;
        const bool has = ctx && ctx[i] > 0 && in_pool;
        for (int64_t j = 0; j < 3 * C; ++j) hist[(size_t)j] = has ? bf16f(state[slot * 3 * C + j]) : 0.0f;
        auto at = [&](int64_t row, int64_t c) {   /* input row `row` (>= s0 - 3) of this sequence */
            return row >= s0 ? bf16f(x[row * x_row + c]) : hist[(size_t)((3 - (s0 - row)) * C + c)];
        };
        for (int64_t t = s0; t < e0; ++t) {
            for (int64_t c = 0; c < C; ++c) {
                float u = bias ? bf16f(bias[c]) : 0.0f;
                for (int j = 0; j < 4; ++j) u = std::fma(bf16f(w[c * 4 + j]), at(t - 3 + j, c), u);
                y[(size_t)c] = u / (1.0f + std::exp(-u));
            }
            for (int64_t hc = 0; hc < C / 128; ++hc) {
                float* yy = &y[(size_t)(hc * 128)];
                if (hc < 2 * Hk) {
                    float ss = 0.0f;
                    for (int e = 0; e < 128; ++e) ss += yy[e] * yy[e];
                    const float inv = 1.0f / std::sqrt(ss + 1e-6f);
                    for (int e = 0; e < 128; ++e) yy[e] *= inv;
                }
                uint16_t* out = hc < Hk ? q + (t * Hk + hc) * 128
                                        : hc < 2 * Hk ? k + (t * Hk + hc - Hk) * 128 : v + (t * Hv + hc - 2 * Hk) * 128;
                for (int e = 0; e < 128; ++e) out[e] = f2bf(yy[e]);
            }
            for (int64_t h = 0; h < Hv; ++h) {
                g[t * Hv + h] = -std::exp(a_log[h]) * softplus2(bf16f(a[t * Hv + h]) + dt_bias[h]);
                beta[t * Hv + h] = 1.0f / (1.0f + std::exp(-bf16f(b[t * Hv + h])));
            }
        }
        if (in_pool) {
            const int64_t L = e0 - s0;
            for (int j = 0; j < 3; ++j)
                for (int64_t c = 0; c < C; ++c)
                    state[slot * 3 * C + j * C + c] =
                        L + j < 3 ? f2bf(hist[(size_t)((L + j) * C + c)]) : x[(e0 - 3 + j) * x_row + c];
        }
    }
}

/* ridgefill_gemm_nt_bias (kernels/rows.cpp:155-160): y = res + act(a @ b^T + bias), bf16 a [M, K] and b [N, K],
 * bias bf16 or f32 [N], optional bf16 res [M, N]; rounded to bf16 after the biased product, after the
 * activation (act 1 = silu, x / (1 + e^-x)) and after the residual. The dot is summed in double (the exact
 * products of bf16 pairs), the bias added to the f32 sum. `z` (optional) receives the value before the
 * residual, for a tolerance that follows a residual's cancellation. Rows [m0, m1) only. */
void oracle_gemm_nt_bias(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, const void* bias,
                         int bias_f32, const uint16_t* res, int64_t ldr, uint16_t* y, int64_t ldy, uint16_t* z,
                         int64_t N, int64_t K, int act, int64_t m0, int64_t m1) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t m = m0; m < m1; ++m)
        for (int64_t n = 0; n < N; ++n) {
            double dot = 0.0;
            const uint16_t* pa = a + m * lda;
            const uint16_t* pb = b + n * ldb;
            for (int64_t k = 0; k < K; ++k) dot += (double)bf16f(pa[k]) * (double)bf16f(pb[k]);
            const float bv = bias_f32 ? ((const float*)bias)[n] : bf16f(((const uint16_t*)bias)[n]);
            uint16_t x = f2bf((float)dot + bv);
            if (act == 1) {
                const double v = bf16f(x);
                x = f2bf((float)(v / (1.0 + std::exp(-v))));
            }
            if (z) z[m * N + n] = x;
            if (res) x = f2bf(bf16f(x) + bf16f(res[m * ldr + n]));
            y[m * ldy + n] = x;
        }
}

/* ridgefill_attn_kv_fill: the gated-attention block's k_norm -> rope_k -> kv_store chain (issue site
 * arch/qwen4exp_fill.h:104-114), each stage rounded to bf16. k, v dense [T, Hkv, D] (D = 256), w [D] bf16 or f32,
 * pos [n_planes, T] (1 or 3 planes), slots [T], cache dense [2, n_slots, Hkv, D] (untouched where no row
 * stores), k_out dense [T, Hkv, D] or null. Per row and head:
 *   ss = the sum of squares in the order the device forms it: eight lane sums (fma, element order), then a
 *        butterfly over the 32 lane sums (offsets 16, 8, 4, 2, 1);
 *   kn = bf16((k r) w) with r = 1 / sqrt(ss / D + eps);
 *   for j < R/2: a = pos[plane(j)][t] * theta^(-2j/R) in f64, c, s = cos a, sin a rounded to f32,
 *        kr[j] = bf16(fma(kn[j], c, -(kn[j+R/2] s))), kr[j+R/2] = bf16(fma(kn[j+R/2], c, kn[j] s));
 *   cache[0, slot, h] = kr, cache[1, slot, h] = v for 0 <= slot < n_slots; k_out = kr.
 * plane(j): 0 unless three planes are given and mode is mrope (sections consecutive) or imrope (plane 1 at
 * j % 3 == 1, j < 3 s1; plane 2 at j % 3 == 2, j < 3 s2). */
void oracle_attn_kv_fill(const uint16_t* k, const uint16_t* v, const void* w, int w_f32, const int32_t* pos,
                         int n_planes, const int32_t* slots, uint16_t* cache, int64_t n_slots, uint16_t* k_out,
                         int64_t T, int64_t Hkv, int64_t R, double theta, float eps, int mode, const int32_t* sections) {
    const int64_t D = 256, half = R / 2;
    std::vector<double> inv_freq((size_t)half);
    std::vector<int> pl((size_t)half, 0);
    for (int64_t j = 0; j < half; ++j) {
        inv_freq[(size_t)j] = std::pow(theta, -2.0 * (double)j / (double)R);
        if (n_planes == 3 && mode == 1)
            pl[(size_t)j] = j < sections[0] ? 0 : j < sections[0] + sections[1] ? 1 : 2;
        else if (n_planes == 3 && mode == 2)
            pl[(size_t)j] = (j % 3 == 1 && j < 3 * sections[1]) ? 1 : (j % 3 == 2 && j < 3 * sections[2]) ? 2 : 0;
    }
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        float x[256], kn[256], kr[256], lane[32], tmp[32];
        std::vector<float> c((size_t)half), sn((size_t)half);
        for (int64_t j = 0; j < half; ++j) {
            const double ang = (double)pos[pl[(size_t)j] * T + t] * inv_freq[(size_t)j];
            c[(size_t)j] = (float)std::cos(ang);
            sn[(size_t)j] = (float)std::sin(ang);
        }
        for (int64_t h = 0; h < Hkv; ++h) {
            const uint16_t* kp = k + (t * Hkv + h) * D;
            for (int64_t i = 0; i < D; ++i) x[i] = bf16f(kp[i]);
            for (int l = 0; l < 32; ++l) {
                float acc = 0.0f;
                for (int e = 0; e < 8; ++e) acc = std::fma(x[8 * l + e], x[8 * l + e], acc);
                lane[l] = acc;
            }
            for (int off = 16; off > 0; off >>= 1) {
                for (int l = 0; l < 32; ++l) tmp[l] = lane[l] + lane[l ^ off];
                std::memcpy(lane, tmp, sizeof lane);
            }
            const float r = 1.0f / std::sqrt(lane[0] / 256.0f + eps);
            for (int64_t i = 0; i < D; ++i) {
                const float wi = w_f32 ? ((const float*)w)[i] : bf16f(((const uint16_t*)w)[i]);
                kn[i] = bf16f(f2bf((x[i] * r) * wi));
                kr[i] = kn[i];
            }
            for (int64_t j = 0; j < half; ++j) {
                const float a1 = kn[j], a2 = kn[j + half], cj = c[(size_t)j], sj = sn[(size_t)j];
                const float p2 = a2 * sj, p1 = a1 * sj;
                kr[j] = std::fma(a1, cj, -p2);
                kr[j + half] = std::fma(a2, cj, p1);
            }
            uint16_t out[256];
            for (int64_t i = 0; i < D; ++i) out[i] = f2bf(kr[i]);
            if (k_out) std::memcpy(k_out + (t * Hkv + h) * D, out, sizeof out);
            const int64_t slot = slots[t];
            if (slot >= 0 && slot < n_slots) {
                std::memcpy(cache + (slot * Hkv + h) * D, out, sizeof out);
                std::memcpy(cache + ((n_slots + slot) * Hkv + h) * D, v + (t * Hkv + h) * D, D * sizeof(uint16_t));
            }
        }
    }
}

}  // extern "C"

/* The gated delta rule, one row at a time (Yang, Kautz & Hatamizadeh, "Gated Delta Networks",
 * arXiv:2412.06464, eq. for S_t): per v-head h with k-head h / (Hv / Hk),
 *   S <- exp(g_t) S;  u = S k_t;  S <- S + beta_t (v_t - u) k_t^T;  o_t = scale * S q_t,
 * S [dv, dk] (state orientation [V, K]: arch/qwen4exp_adapter.h:59-60). Each sequence i covers rows
 * [cu[i], cu[i+1]) and carries state slot idx[i * idx_pitch] (outside [0, n_states): skipped).
 * `Real` is double for the reference value, float for the timed CPU baseline. q and o may be null
 * (state-only fill). Heads [h0, h1) only. */
template <typename Real>
void gdn_reference(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g, const float* beta,
                   float* state, const int32_t* idx, int64_t idx_pitch, int64_t n_states, const int32_t* cu,
                   int64_t n_seq, uint16_t* o, int64_t Hk, int64_t Hv, int64_t dk, int64_t dv, float scale,
                   int64_t h0, int64_t h1) {
    const int64_t group = Hv / Hk;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t h = h0; h < h1; ++h) {
        std::vector<Real> S((size_t)(dv * dk)), kt((size_t)dk), qt((size_t)dk), u((size_t)dv);
        for (int64_t sq = 0; sq < n_seq; ++sq) {
            const int64_t slot = idx[sq * idx_pitch];
            if (slot < 0 || slot >= n_states) continue;
            float* st = state + (slot * Hv + h) * dv * dk;
            for (int64_t e = 0; e < dv * dk; ++e) S[(size_t)e] = (Real)st[e];
            const int64_t hk = h / group;
            for (int64_t t = cu[sq]; t < cu[sq + 1]; ++t) {
                const Real decay = (Real)std::exp((Real)g[t * Hv + h]), b = (Real)beta[t * Hv + h];
                for (int64_t j = 0; j < dk; ++j) kt[(size_t)j] = (Real)bf16f(k[(t * Hk + hk) * dk + j]);
                for (int64_t i = 0; i < dv; ++i) {
                    Real acc = 0;
                    Real* row = &S[(size_t)(i * dk)];
                    for (int64_t j = 0; j < dk; ++j) {
                        row[j] *= decay;
                        acc += row[j] * kt[(size_t)j];
                    }
                    u[(size_t)i] = b * ((Real)bf16f(v[(t * Hv + h) * dv + i]) - acc);
                }
                for (int64_t i = 0; i < dv; ++i) {
                    Real* row = &S[(size_t)(i * dk)];
                    for (int64_t j = 0; j < dk; ++j) row[j] += u[(size_t)i] * kt[(size_t)j];
                }
                if (o && q) {
                    for (int64_t j = 0; j < dk; ++j) qt[(size_t)j] = (Real)bf16f(q[(t * Hk + hk) * dk + j]);
                    for (int64_t i = 0; i < dv; ++i) {
                        Real acc = 0;
                        for (int64_t j = 0; j < dk; ++j) acc += S[(size_t)(i * dk + j)] * qt[(size_t)j];
                        o[(t * Hv + h) * dv + i] = f2bf((float)(acc * (Real)scale));
                    }
                }
            }
            for (int64_t e = 0; e < dv * dk; ++e) st[e] = (float)S[(size_t)e];
        }
    }
}

extern "C" {

/* q, k [T, Hk, dk], v [T, Hv, dv], o [T, Hv, dv] bf16 packed; g, beta [T, Hv] f32; state
 * [n_states, Hv, dv, dk] f32 packed. */
void oracle_gdn_fill_f64(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g, const float* beta,
                         float* state, const int32_t* idx, int64_t idx_pitch, int64_t n_states, const int32_t* cu,
                         int64_t n_seq, uint16_t* o, int64_t Hk, int64_t Hv, int64_t dk, int64_t dv, float scale,
                         int64_t h0, int64_t h1) {
    gdn_reference<double>(q, k, v, g, beta, state, idx, idx_pitch, n_states, cu, n_seq, o, Hk, Hv, dk, dv, scale, h0, h1);
}

void oracle_gdn_fill_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g, const float* beta,
                         float* state, const int32_t* idx, int64_t idx_pitch, int64_t n_states, const int32_t* cu,
                         int64_t n_seq, uint16_t* o, int64_t Hk, int64_t Hv, int64_t dk, int64_t dv, float scale,
                         int64_t h0, int64_t h1) {
    gdn_reference<float>(q, k, v, g, beta, state, idx, idx_pitch, n_states, cu, n_seq, o, Hk, Hv, dk, dv, scale, h0, h1);
}

int oracle_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Sets the OpenMP thread count of the oracle's parallel loops (a launcher such as torchrun sets
 * OMP_NUM_THREADS=1 in every process it starts; the CPU baseline asks for the host's cores itself). */
void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

}  // extern "C"
