/* parse.cpp -- operand checks for every row of the B200 RidgeFill library: a RadArgs reduced to one of
 * the parsed structs of ridgefill.h, or a named refusal.
 *
 * The reference ops refuse exactly what the reference parse refuses, with the same code
 * (kernels/host_ref.cpp:16-282, 435-463); the new ops follow the same conventions. Nothing here
 * reads an operand's VALUES (they are device memory on a device row): values such as cu_last are
 * checked where the kernel reads them, with the reference's fail-safe.
 */
#include "ridgefill.h"

#include <cmath>
#include <cstring>

namespace {

bool dense(const RadTensor* t) { return rad_tensor_is_contiguous(t) != 0; }

int64_t per_slot_head(const RadTensor* t) {   /* extent of axes 2.. */
    int64_t n = 1;
    for (uint32_t i = 2; i < t->rank; ++i) n *= t->shape[i];
    return n;
}

/* The stride between N and D in an ND pool [.., 1, 2] or [.., 2, 1]; 0 if not such a pair
 * (kernels/host_ref.cpp:27-34). */
int64_t pair_stride(const RadTensor* t) {
    if (t->rank < 3 || per_slot_head(t) != 2) return 0;
    for (uint32_t i = 2; i < t->rank; ++i)
        if (t->shape[i] == 2) return t->stride[i];
    return 0;
}

int index_rows(const RadTensor* t, int64_t* rows, int64_t* pitch) {   /* host_ref.cpp:37-43 */
    if (t->dtype != RAD_I32) return RAD_E_DTYPE;
    if (t->rank < 1 || t->rank > 2 || t->stride[t->rank - 1] != 1) return RAD_E_STRIDE;
    *rows = t->shape[0];
    *pitch = t->rank == 2 ? t->stride[0] : 1;
    return RAD_OK;
}

int optional_bounds(const RadTensor* t, int64_t need, const int32_t** out) {   /* host_ref.cpp:46-54 */
    *out = nullptr;
    if (!t) return RAD_OK;
    if (t->dtype != RAD_I32) return RAD_E_DTYPE;
    if (!dense(t)) return RAD_E_STRIDE;
    if (rad_tensor_numel(t) < need) return RAD_E_SHAPE;
    *out = (const int32_t*)t->data;
    return RAD_OK;
}

int which(const char* s, const char* const* names, int n) {
    for (int i = 0; s && i < n; ++i)
        if (std::strcmp(s, names[i]) == 0) return i;
    return -1;
}

int copy_word(const RidgeFillCopy& p) {   /* host_ref.cpp:226-230 */
    const uint64_t all = (uint64_t)(uintptr_t)p.src | (uint64_t)(uintptr_t)p.dst | (uint64_t)p.src_pitch |
                         (uint64_t)p.dst_pitch | (uint64_t)p.row_bytes;
    return all % 16 == 0 ? 16 : (all % 4 == 0 ? 4 : 1);
}

int select_pair(const RadTensor* src, const RadTensor* dst, int64_t n, RidgeFillCopy* p) {   /* :234-251 */
    *p = RidgeFillCopy{};
    if (!src && !dst) return RAD_OK;
    if (!src || !dst) return RAD_E_INVAL;
    const int bits = rad_dtype_bits(src->dtype);
    if (dst->dtype != src->dtype || bits <= 0 || bits % 8 != 0) return RAD_E_DTYPE;
    if (src->rank != 2 || dst->rank != 2 || src->shape[1] != dst->shape[1] || src->shape[0] < n || dst->shape[0] < n)
        return RAD_E_SHAPE;
    if (src->stride[1] != 1 || dst->stride[1] != 1) return RAD_E_STRIDE;
    const int64_t bytes = bits / 8;
    p->src = (const unsigned char*)src->data;
    p->dst = (unsigned char*)dst->data;
    p->src_pitch = src->stride[0] * bytes;
    p->dst_pitch = dst->stride[0] * bytes;
    p->row_bytes = src->shape[1] * bytes;
    p->word = copy_word(*p);
    return RAD_OK;
}

}  // namespace

extern "C" int ridgefill_mask_parse(const RadArgs* a, RidgeFillMask* g) {   /* host_ref.cpp:64-104 */
    const RadTensor* cu = rad_arg_in(a, MK_CU);
    const RadTensor* tok = rad_arg_in(a, MK_TOKENS);
    const RadTensor* pos = rad_arg_in(a, MK_POS);
    const RadTensor* score = rad_arg_in(a, MK_SCORE);
    const RadTensor* mask = rad_arg_in(a, MK_MASK);
    const RadTensor* bounds = rad_arg_in(a, MK_BOUNDS);
    const RadTensor* zeros = rad_arg_in(a, MK_ZEROS);
    static const char* const modes[] = { "none", "class", "random", "all", "step" };
    *g = RidgeFillMask{};
    g->mode = which(rad_args_gets(a, "mode"), modes, 5);
    g->share = rad_args_getf_or(a, "share", NAN);
    long long seed = 0;
    const bool ranked = g->mode == RIDGEFILL_MODE_CLASS || g->mode == RIDGEFILL_MODE_RANDOM;
    if (!cu || !tok || !pos || !mask || !bounds || (ranked && !score) || g->mode < 0 ||
        !rad_args_geti(a, "seed", &seed) || !(g->share >= 0.0 && g->share <= 1.0))
        return RAD_E_INVAL;
    if (cu->dtype != RAD_I32 || tok->dtype != RAD_I32 || pos->dtype != RAD_I32 || mask->dtype != RAD_I32 ||
        bounds->dtype != RAD_I32 || (score && score->dtype != RAD_F32) || (zeros && zeros->dtype != RAD_I32))
        return RAD_E_DTYPE;
    if (!dense(cu) || !dense(tok) || !dense(mask) || !dense(bounds) || (score && !dense(score)) ||
        (zeros && !dense(zeros)))
        return RAD_E_STRIDE;
    g->b = rad_tensor_numel(tok);
    if (pos->rank < 1 || pos->rank > 2 || pos->shape[pos->rank - 1] < g->b || rad_tensor_numel(cu) < 2 ||
        rad_tensor_numel(bounds) < 4)
        return RAD_E_SHAPE;
    g->cu_last = (const int32_t*)cu->data;
    g->tokens = (const int32_t*)tok->data;
    g->positions = (const int32_t*)pos->data;
    g->pos_stride = pos->stride[pos->rank - 1];
    g->score = score ? (const float*)score->data : nullptr;
    g->vocab = score ? rad_tensor_numel(score) : 0;
    g->mask = (int32_t*)mask->data;
    g->n = rad_tensor_numel(mask);
    g->bounds = (int32_t*)bounds->data;
    g->zeros = zeros ? (int32_t*)zeros->data : nullptr;
    g->n_zeros = zeros ? rad_tensor_numel(zeros) : 0;
    g->seed = seed;
    return RAD_OK;
}

extern "C" int ridgefill_rho_parse(const RadArgs* a, RidgeFillRho* g) {   /* host_ref.cpp:106-145 */
    const RadTensor* av = rad_arg_in(a, RH_A);
    const RadTensor* mask = rad_arg_in(a, RH_MASK);
    const RadTensor* alog = rad_arg_in(a, RH_ALOG);
    const RadTensor* dtb = rad_arg_in(a, RH_DTBIAS);
    const RadTensor* nd = rad_arg_in(a, RH_ND);
    const RadTensor* sidx = rad_arg_in(a, RH_SIDX);
    *g = RidgeFillRho{};
    if (!av || !mask || !alog || !dtb || !nd || !sidx) return RAD_E_INVAL;
    if ((av->dtype != RAD_BF16 && av->dtype != RAD_F32) || mask->dtype != RAD_I32 || alog->dtype != RAD_F32 ||
        dtb->dtype != RAD_F32 || nd->dtype != RAD_F32)
        return RAD_E_DTYPE;
    int64_t n_seq = 0, pitch = 0;
    int rc = index_rows(sidx, &n_seq, &pitch);
    if (rc == RAD_OK) rc = optional_bounds(rad_arg_in(a, RH_BOUNDS), 1, &g->bounds);
    if (rc != RAD_OK) return rc;
    if (av->rank != 2 || !dense(mask) || !dense(alog) || !dense(dtb)) return RAD_E_STRIDE;
    long long heads = 0;
    if (!rad_args_geti(a, "n_head", &heads)) return RAD_E_INVAL;
    g->n = av->shape[0];
    g->n_head = av->shape[1];
    g->nd_inner = pair_stride(nd);
    if (heads != g->n_head || rad_tensor_numel(mask) < g->n || rad_tensor_numel(alog) != heads ||
        rad_tensor_numel(dtb) != heads || nd->shape[1] != heads || g->nd_inner == 0 || n_seq != 1)
        return RAD_E_SHAPE;
    g->a = av->data;
    g->a_pitch = av->stride[0];
    g->a_col = av->stride[1];
    g->a_bf16 = av->dtype == RAD_BF16;
    g->mask = (const int32_t*)mask->data;
    g->a_log = (const float*)alog->data;
    g->dt_bias = (const float*)dtb->data;
    g->nd = (float*)nd->data;
    g->nd_slot = nd->stride[0];
    g->nd_head = nd->stride[1];
    g->n_states = nd->shape[0];
    g->state_idx = (const int32_t*)sidx->data;
    return RAD_OK;
}

extern "C" int ridgefill_correct_parse(const RadArgs* a, RidgeFillCorrect* g) {   /* host_ref.cpp:147-197 */
    const RadTensor* st = rad_arg_in(a, SC_STATE);
    const RadTensor* sidx = rad_arg_in(a, SC_STATE_IDX);
    const RadTensor* ap = rad_arg_in(a, SC_APPLIED);
    const RadTensor* aidx = rad_arg_in(a, SC_APPLIED_IDX);
    const RadTensor* c = rad_arg_in(a, SC_C);
    const RadTensor* nd = rad_arg_in(a, SC_ND);
    const RadTensor* nidx = rad_arg_in(a, SC_ND_IDX);
    *g = RidgeFillCorrect{};
    if (!st || !sidx || !ap || !aidx || !c || !nd != !nidx) return RAD_E_INVAL;
    if (st->dtype != RAD_F32 || ap->dtype != RAD_F32 || c->dtype != RAD_F32 || (nd && nd->dtype != RAD_F32))
        return RAD_E_DTYPE;
    static const char* const modes[] = { "undo", "apply" };
    long long heads = 0, sd0 = 0, sd1 = 0;
    g->apply = which(rad_args_gets(a, "mode"), modes, 2);
    const double alpha = rad_args_getf_or(a, "alpha", NAN);
    if (g->apply < 0 || !rad_args_geti(a, "n_head", &heads) || !rad_args_geti(a, "sd0", &sd0) ||
        !rad_args_geti(a, "sd1", &sd1) || (g->apply && !std::isfinite(alpha)))
        return RAD_E_INVAL;
    int64_t ap_rows = 0, nd_rows = 0;
    int rc = index_rows(sidx, &g->n_seq, &g->st_pitch);
    if (rc == RAD_OK) rc = index_rows(aidx, &ap_rows, &g->ap_pitch);
    if (rc == RAD_OK && nidx) rc = index_rows(nidx, &nd_rows, &g->nd_pitch);
    if (rc == RAD_OK) rc = optional_bounds(rad_arg_in(a, SC_BOUNDS), 2, &g->bounds);
    if (rc != RAD_OK) return rc;
    if (ap_rows != g->n_seq || (nidx && nd_rows != g->n_seq)) return RAD_E_SHAPE;
    if (st->rank != 4 || st->shape[1] != heads || st->shape[2] != sd0 || st->shape[3] != sd1 || !dense(c) ||
        rad_tensor_numel(c) != heads * sd0 * sd1 || ap->rank < 2 || ap->shape[1] != heads || per_slot_head(ap) != 1 ||
        (nd && (nd->shape[1] != heads || pair_stride(nd) == 0)))
        return RAD_E_SHAPE;
    g->state = (float*)st->data;
    g->st_slot = st->stride[0];
    g->st_head = st->stride[1];
    g->st_row = st->stride[2];
    g->st_col = st->stride[3];
    g->applied = (float*)ap->data;
    g->ap_slot = ap->stride[0];
    g->ap_head = ap->stride[1];
    g->c = (const float*)c->data;
    g->c_head = sd0 * sd1;   /* C is read packed [heads, sd0, sd1] whatever its rank (host_ref.cpp:181-183) */
    g->c_row = sd1;
    g->nd = nd ? (const float*)nd->data : nullptr;
    g->nd_slot = nd ? nd->stride[0] : 0;
    g->nd_head = nd ? nd->stride[1] : 0;
    g->nd_inner = nd ? pair_stride(nd) : 0;
    g->st_idx = (const int32_t*)sidx->data;
    g->ap_idx = (const int32_t*)aidx->data;
    g->nd_idx = nidx ? (const int32_t*)nidx->data : nullptr;
    g->st_states = st->shape[0];
    g->ap_states = ap->shape[0];
    g->nd_states = nd ? nd->shape[0] : 0;
    g->n_head = heads;
    g->sd0 = sd0;
    g->sd1 = sd1;
    g->alpha = (float)alpha;
    return RAD_OK;
}

extern "C" int ridgefill_state_read_parse(const RadArgs* a, RidgeFillStateRead* g) {   /* host_ref.cpp:199-221 */
    const RadTensor* st = rad_arg_in(a, SR_STATE);
    const RadTensor* sidx = rad_arg_in(a, SR_STATE_IDX);
    const RadTensor* out = rad_arg_in(a, SR_OUT);
    long long heads = 0, sd0 = 0, sd1 = 0;
    *g = RidgeFillStateRead{};
    if (!st || !sidx || !out || !rad_args_geti(a, "n_head", &heads) || !rad_args_geti(a, "sd0", &sd0) ||
        !rad_args_geti(a, "sd1", &sd1))
        return RAD_E_INVAL;
    if (st->dtype != RAD_F32 || out->dtype != RAD_F32) return RAD_E_DTYPE;
    const int rc = index_rows(sidx, &g->n_seq, &g->idx_pitch);
    if (rc != RAD_OK) return rc;
    if (!dense(out)) return RAD_E_STRIDE;
    if (st->rank != 4 || st->shape[1] != heads || st->shape[2] != sd0 || st->shape[3] != sd1 ||
        rad_tensor_numel(out) < g->n_seq * heads * sd0 * sd1)
        return RAD_E_SHAPE;
    g->state = (const float*)st->data;
    g->st_slot = st->stride[0];
    g->st_head = st->stride[1];
    g->st_row = st->stride[2];
    g->st_col = st->stride[3];
    g->n_states = st->shape[0];
    g->idx = (const int32_t*)sidx->data;
    g->out = (float*)out->data;
    g->n_head = heads;
    g->sd0 = sd0;
    g->sd1 = sd1;
    return RAD_OK;
}

extern "C" int ridgefill_select_parse(const RadArgs* a, RidgeFillSelect* g) {   /* host_ref.cpp:253-266 */
    const RadTensor* mask = rad_arg_in(a, SL_MASK);
    *g = RidgeFillSelect{};
    if (!mask || !rad_arg_in(a, SL_X_SRC) || !rad_arg_in(a, SL_X)) return RAD_E_INVAL;
    if (mask->dtype != RAD_I32) return RAD_E_DTYPE;
    if (!dense(mask)) return RAD_E_STRIDE;
    g->mask = (const int32_t*)mask->data;
    g->n = rad_tensor_numel(mask);
    for (int k = 0; k < RIDGEFILL_SELECT_PAIRS; ++k) {
        const int rc = select_pair(rad_arg_in(a, SL_X_SRC + k), rad_arg_in(a, SL_X + k), g->n, &g->pair[k]);
        if (rc != RAD_OK) return rc;
    }
    return RAD_OK;
}

extern "C" int ridgefill_drop_parse(const RadArgs* a, RidgeFillDrop* g) {   /* host_ref.cpp:268-282 */
    const RadTensor* mask = rad_arg_in(a, DR_MASK);
    const RadTensor* ids = rad_arg_in(a, DR_IDS);
    long long top_k = -1;
    *g = RidgeFillDrop{};
    if (!mask || !ids || !rad_args_geti(a, "top_k", &top_k) || top_k < 0) return RAD_E_INVAL;
    if (mask->dtype != RAD_I32 || ids->dtype != RAD_I32) return RAD_E_DTYPE;
    if (!dense(mask) || (ids->rank == 2 && ids->stride[1] != 1)) return RAD_E_STRIDE;
    g->n = rad_tensor_numel(mask);
    if (ids->rank != 2 || ids->shape[0] < g->n || ids->shape[1] < top_k) return RAD_E_SHAPE;
    g->mask = (const int32_t*)mask->data;
    g->ids = (int32_t*)ids->data;
    g->pitch = ids->stride[0];
    g->top_k = top_k;
    return RAD_OK;
}

extern "C" int ridgefill_hazard_parse(const RadArgs* a, RidgeFillHazard* g) {   /* host_ref.cpp:435-463 */
    const RadTensor* cu = rad_arg_in(a, HZ_CU);
    const RadTensor* pos = rad_arg_in(a, HZ_POS);
    const RadTensor* span = rad_arg_in(a, HZ_SPAN);
    const RadTensor* meta = rad_arg_in(a, HZ_META);
    const RadTensor* idx = rad_arg_in(a, HZ_META_IDX);
    const RadTensor* cnt = rad_arg_in(a, HZ_COUNT);
    *g = RidgeFillHazard{};
    if (!cu || !pos || !meta || !idx || !cnt) return RAD_E_INVAL;
    if (cu->dtype != RAD_I32 || pos->dtype != RAD_I32 || meta->dtype != RAD_F32 || cnt->dtype != RAD_F32)
        return RAD_E_DTYPE;
    if (!dense(cu) || !dense(cnt)) return RAD_E_STRIDE;
    int64_t rows = 0, pitch = 0;
    int rc = index_rows(idx, &rows, &pitch);
    if (rc == RAD_OK) rc = optional_bounds(rad_arg_in(a, HZ_BOUNDS), 2, &g->bounds);
    if (rc != RAD_OK) return rc;
    if (rows < 1 || rad_tensor_numel(cu) < 2 || rad_tensor_numel(cnt) < 1 || pos->rank < 1 || pos->rank > 2 ||
        meta->rank < 2 || meta->shape[meta->rank - 1] != 2 || meta->stride[meta->rank - 1] != 1)
        return RAD_E_SHAPE;
    g->cu_last = (const int32_t*)cu->data;
    g->positions = (const int32_t*)pos->data;
    g->pos_stride = pos->stride[pos->rank - 1];
    g->span = span ? rad_tensor_numel(span) : 0;
    g->meta = (float*)meta->data;
    g->meta_slot = meta->stride[0];
    g->meta_states = meta->shape[0];
    g->meta_idx = (const int32_t*)idx->data;
    g->count = (float*)cnt->data;
    return RAD_OK;
}

/* ridgefill_gemm_nt_q (with_bias 0: operands a, a_scale, b, b_scale, y, a_sum, b_ref) and
 * ridgefill_gemm_nt_q_bias (with_bias 1: a, a_scale, b, b_scale, bias, y, acc). a_scale is required (an
 * i8a8 product has activation scales); a_sum and b_ref (zero-point terms of other dtypes) must be
 * absent. K must be a multiple of 128 and of `group`; `group` divides K (128, or K itself for
 * BASELINE's per-row / per-column scaling); rows of a and codes of b start 16-byte aligned (the TMA
 * reads them in 128-byte rows). */
extern "C" int ridgefill_gemm_q_parse(const RadArgs* a, int with_bias, RidgeFillGemmQ* g) {
    *g = RidgeFillGemmQ{};
    const RadTensor* A = rad_arg_in(a, GQ_A);
    const RadTensor* AS = rad_arg_in(a, GQ_A_SCALE);
    const RadTensor* B = rad_arg_in(a, GQ_B);
    const RadTensor* BS = rad_arg_in(a, GQ_B_SCALE);
    const RadTensor* bias = with_bias ? rad_arg_in(a, GB_BIAS) : nullptr;
    const RadTensor* Y = rad_arg_in(a, with_bias ? (int)GB_Y : (int)GQ_Y);
    const RadTensor* acc = with_bias ? rad_arg_in(a, GB_ACC) : nullptr;
    long long M = 0, N = 0, K = 0, group = 0;
    const char* dt = rad_args_gets(a, "dtype");
    if (!A || !AS || !B || !BS || !Y || !rad_args_geti(a, "N", &N) || !rad_args_geti(a, "K", &K) ||
        !rad_args_geti(a, "group", &group) || !dt || std::strcmp(dt, "i8a8") != 0)
        return RAD_E_INVAL;
    if (!with_bias && (rad_arg_in(a, GQ_A_SUM) || rad_arg_in(a, GQ_B_REF))) return RAD_E_UNSUPPORTED;
    if (A->dtype != RAD_I8 || AS->dtype != RAD_F32 || B->dtype != RAD_I8 || BS->dtype != RAD_F32 ||
        Y->dtype != RAD_BF16 || (bias && bias->dtype != RAD_BF16) || (acc && acc->dtype != RAD_I32))
        return RAD_E_DTYPE;
    if (A->rank != 2 || B->rank != 2 || Y->rank != 2) return RAD_E_SHAPE;
    M = A->shape[0];
    if (group <= 0 || K <= 0 || K % group != 0 || K % 128 != 0 || group % 128 != 0 || N <= 0 || N % 16 != 0)
        return RAD_E_SHAPE;
    const int64_t blocks = K / group;
    if (A->shape[1] != K || B->shape[0] != N || B->shape[1] != K || Y->shape[0] != M || Y->shape[1] != N ||
        rad_tensor_numel(AS) != M * blocks || rad_tensor_numel(BS) != blocks * N || (bias && rad_tensor_numel(bias) != N) ||
        (acc && rad_tensor_numel(acc) != M * N * blocks))
        return RAD_E_SHAPE;
    if (A->stride[1] != 1 || B->stride[1] != 1 || Y->stride[1] != 1 || !dense(BS) || (bias && !dense(bias)) ||
        (acc && !dense(acc)))
        return RAD_E_STRIDE;
    if (AS->rank == 2 ? (AS->stride[1] != 1) : !dense(AS)) return RAD_E_STRIDE;
    /* TMA: 16-byte aligned bases and row pitches. */
    if (((uintptr_t)A->data | (uintptr_t)B->data) % 16 || A->stride[0] % 16 || B->stride[0] % 16 ||
        ((uintptr_t)Y->data % 16) || (Y->stride[0] * 2) % 16 || (uintptr_t)BS->data % 16 ||
        (bias && (uintptr_t)bias->data % 16))
        return RAD_E_STRIDE;
    g->a = (const int8_t*)A->data;
    g->lda = A->stride[0];
    g->a_scale = (const float*)AS->data;
    g->ldas = AS->rank == 2 ? AS->stride[0] : blocks;
    g->b = (const int8_t*)B->data;
    g->ldb = B->stride[0];
    g->b_scale = (const float*)BS->data;
    g->bias = bias ? (const uint16_t*)bias->data : nullptr;
    g->y = (uint16_t*)Y->data;
    g->ldy = Y->stride[0];
    g->acc = acc ? (int32_t*)acc->data : nullptr;
    g->M = M;
    g->N = N;
    g->K = K;
    g->group = group;
    long long max_ctas = 0;   /* optional: a caller sharing the GPU with another stream's kernels bounds the grid */
    if (rad_args_geti(a, "max_ctas", &max_ctas) && max_ctas < 0) return RAD_E_INVAL;
    g->max_ctas = max_ctas;
    return RAD_OK;
}

/* ridgefill_gemm_nt_bias: see include/ridgefill.h. */
extern "C" int ridgefill_gemm_bias_parse(const RadArgs* a, RidgeFillGemmBias* g) {
    *g = RidgeFillGemmBias{};
    const RadTensor* A = rad_arg_in(a, GN_A);
    const RadTensor* B = rad_arg_in(a, GN_B);
    const RadTensor* bias = rad_arg_in(a, GN_BIAS);
    const RadTensor* R = rad_arg_in(a, GN_RES);
    const RadTensor* Y = rad_arg_in(a, GN_Y);
    long long N = 0, K = 0;
    const char* dt = rad_args_gets(a, "dtype");
    if (!A || !B || !bias || !Y || !rad_args_geti(a, "N", &N) || !rad_args_geti(a, "K", &K) || !dt) return RAD_E_INVAL;
    if (std::strcmp(dt, "bf16") != 0) return RAD_E_UNSUPPORTED;
    const char* act = rad_args_gets(a, "act");
    int act_code = RIDGEFILL_ACT_NONE;
    if (act && std::strcmp(act, "none") != 0) {
        if (std::strcmp(act, "silu") == 0) act_code = RIDGEFILL_ACT_SILU;
        else return RAD_E_UNSUPPORTED;
    }
    if (A->dtype != RAD_BF16 || B->dtype != RAD_BF16 || (bias->dtype != RAD_BF16 && bias->dtype != RAD_F32) ||
        (R && R->dtype != RAD_BF16) || Y->dtype != RAD_BF16)
        return RAD_E_DTYPE;
    if (A->rank != 2 || B->rank != 2 || Y->rank != 2 || (R && R->rank != 2)) return RAD_E_SHAPE;
    const int64_t M = A->shape[0];
    if (K <= 0 || N <= 0 || K % 8 != 0 || N % 8 != 0) return RAD_E_SHAPE;   /* 16-byte row pitches */
    if (A->shape[1] != K || B->shape[0] != N || B->shape[1] != K || Y->shape[0] != M || Y->shape[1] != N ||
        rad_tensor_numel(bias) != N || (R && (R->shape[0] != M || R->shape[1] != N)))
        return RAD_E_SHAPE;
    if (A->stride[1] != 1 || B->stride[1] != 1 || Y->stride[1] != 1 || !dense(bias) || (R && R->stride[1] != 1))
        return RAD_E_STRIDE;
    /* TMA tiles of a, b and y, 16-byte vector reads of the bias and the residual. */
    if (((uintptr_t)A->data | (uintptr_t)B->data | (uintptr_t)Y->data | (uintptr_t)bias->data) % 16 ||
        (A->stride[0] * 2) % 16 || (B->stride[0] * 2) % 16 || (Y->stride[0] * 2) % 16 ||
        (R && ((uintptr_t)R->data % 16 || (R->stride[0] * 2) % 16)))
        return RAD_E_STRIDE;
    g->a = (const uint16_t*)A->data;
    g->lda = A->stride[0];
    g->b = (const uint16_t*)B->data;
    g->ldb = B->stride[0];
    g->bias = bias->data;
    g->bias_f32 = bias->dtype == RAD_F32;
    g->res = R ? (const uint16_t*)R->data : nullptr;
    g->ldr = R ? R->stride[0] : 0;
    g->y = (uint16_t*)Y->data;
    g->ldy = Y->stride[0];
    g->M = M;
    g->N = N;
    g->K = K;
    g->act = act_code;
    return RAD_OK;
}

/* ridgefill_gdn_conv_prep: x bf16 [T, C] (C = 2 Hk dk + Hv dv, rows 16-byte aligned), w bf16 [C, 4] dense,
 * bias bf16 [C] or absent (16-byte aligned), A_log and dt_bias f32 [Hv], state bf16 [slots, 3, C] (a dense [3, C] per slot),
 * cu_seqlens i32 [n_seq + 1], a and b bf16 [T, Hv] (any row pitch, last stride 1), idx i32 [n_seq] or [n_seq, >= 1],
 * ctx_lens i32 [n_seq] or absent, q and k bf16 [T, Hk, dk], v bf16 [T, Hv, dv] (each head dense, rows and
 * heads 16-byte aligned), g and beta f32 [T, Hv]. Head dims 128, width 4. */
extern "C" int ridgefill_conv_prep_parse(const RadArgs* a, RidgeFillConvPrep* g) {
    *g = RidgeFillConvPrep{};
    const RadTensor* X = rad_arg_in(a, CP_X);
    const RadTensor* W = rad_arg_in(a, CP_W);
    const RadTensor* B0 = rad_arg_in(a, CP_BIAS);
    const RadTensor* AL = rad_arg_in(a, CP_A_LOG);
    const RadTensor* DT = rad_arg_in(a, CP_DT_BIAS);
    const RadTensor* ST = rad_arg_in(a, CP_STATE);
    const RadTensor* CU = rad_arg_in(a, CP_CU);
    const RadTensor* A = rad_arg_in(a, CP_A);
    const RadTensor* Bg = rad_arg_in(a, CP_B);
    const RadTensor* I = rad_arg_in(a, CP_IDX);
    const RadTensor* CX = rad_arg_in(a, CP_CTX);
    const RadTensor* Q = rad_arg_in(a, CP_Q);
    const RadTensor* K = rad_arg_in(a, CP_K);
    const RadTensor* V = rad_arg_in(a, CP_V);
    const RadTensor* G = rad_arg_in(a, CP_G);
    const RadTensor* BE = rad_arg_in(a, CP_BETA);
    long long T = 0, hk = 0, hv = 0, dk = 0, dv = 0, width = 0;
    if (!X || !W || !AL || !DT || !ST || !CU || !A || !Bg || !I || !Q || !K || !V || !G || !BE) return RAD_E_INVAL;
    if (!rad_args_geti(a, "M", &T) || !rad_args_geti(a, "n_head_k", &hk) || !rad_args_geti(a, "n_head_v", &hv) ||
        !rad_args_geti(a, "head_k", &dk) || !rad_args_geti(a, "head_v", &dv) || !rad_args_geti(a, "conv", &width))
        return RAD_E_INVAL;
    if (dk != 128 || dv != 128 || width != 4) return RAD_E_UNSUPPORTED;
    if (hk <= 0 || hv <= 0 || T < 0) return RAD_E_SHAPE;
    const int64_t C = 2 * hk * dk + hv * dv;
    if (X->dtype != RAD_BF16 || W->dtype != RAD_BF16 || (B0 && B0->dtype != RAD_BF16) || AL->dtype != RAD_F32 ||
        DT->dtype != RAD_F32 || ST->dtype != RAD_BF16 || CU->dtype != RAD_I32 || A->dtype != RAD_BF16 ||
        Bg->dtype != RAD_BF16 || I->dtype != RAD_I32 || (CX && CX->dtype != RAD_I32) || Q->dtype != RAD_BF16 ||
        K->dtype != RAD_BF16 || V->dtype != RAD_BF16 || G->dtype != RAD_F32 || BE->dtype != RAD_F32)
        return RAD_E_DTYPE;
    if (X->rank != 2 || X->shape[0] != T || X->shape[1] != C || X->stride[1] != 1) return X->rank == 2 && X->stride[1] != 1 ? RAD_E_STRIDE : RAD_E_SHAPE;
    if (W->rank != 2 || W->shape[0] != C || W->shape[1] != 4 || !dense(W)) return RAD_E_SHAPE;
    if (B0 && (rad_tensor_numel(B0) != C || !dense(B0))) return RAD_E_SHAPE;
    if (B0 && (uintptr_t)B0->data % 16) return RAD_E_STRIDE;
    if (rad_tensor_numel(AL) != hv || rad_tensor_numel(DT) != hv || !dense(AL) || !dense(DT)) return RAD_E_SHAPE;
    if (ST->rank != 3 || ST->shape[1] != 3 || ST->shape[2] != C || ST->stride[2] != 1 || ST->stride[1] != C) return RAD_E_SHAPE;
    if (CU->rank != 1 || CU->shape[0] < 1 || CU->stride[0] != 1) return RAD_E_SHAPE;
    const int64_t n_seq = CU->shape[0] - 1;
    if (I->rank == 1 ? (I->shape[0] < n_seq || I->stride[0] != 1) : (I->rank != 2 || I->shape[0] < n_seq || I->shape[1] < 1))
        return RAD_E_SHAPE;
    if (CX && (CX->rank != 1 || CX->shape[0] < n_seq || CX->stride[0] != 1)) return RAD_E_SHAPE;
    const RadTensor* per_head[4] = { A, Bg, G, BE };
    for (const RadTensor* t : per_head)
        if (t->rank != 2 || t->shape[0] != T || t->shape[1] != hv || t->stride[1] != 1) return RAD_E_SHAPE;
    if (Q->rank != 3 || Q->shape[0] != T || Q->shape[1] != hk || Q->shape[2] != dk || Q->stride[2] != 1) return RAD_E_SHAPE;
    if (K->rank != 3 || K->shape[0] != T || K->shape[1] != hk || K->shape[2] != dk || K->stride[2] != 1) return RAD_E_SHAPE;
    if (V->rank != 3 || V->shape[0] != T || V->shape[1] != hv || V->shape[2] != dv || V->stride[2] != 1) return RAD_E_SHAPE;
    /* 16-byte loads of x, w, the bias and the state, 16-byte stores of q, k, v (eight channels a lane). */
    if (((uintptr_t)X->data | (uintptr_t)Q->data | (uintptr_t)K->data | (uintptr_t)V->data | (uintptr_t)W->data |
         (uintptr_t)ST->data) % 16 ||
        (X->stride[0] * 2) % 16 || (Q->stride[0] * 2) % 16 || (Q->stride[1] * 2) % 16 || (K->stride[0] * 2) % 16 ||
        (K->stride[1] * 2) % 16 || (V->stride[0] * 2) % 16 || (V->stride[1] * 2) % 16 || (ST->stride[0] * 2) % 16)
        return RAD_E_STRIDE;
    g->x = (const uint16_t*)X->data;
    g->x_row = X->stride[0];
    g->w = (const uint16_t*)W->data;
    g->bias = B0 ? (const uint16_t*)B0->data : nullptr;
    g->a_log = (const float*)AL->data;
    g->dt_bias = (const float*)DT->data;
    g->state = (uint16_t*)ST->data;
    g->st_slot = ST->stride[0];
    g->n_states = ST->shape[0];
    g->cu = (const int32_t*)CU->data;
    g->n_seq = n_seq;
    g->a = (const uint16_t*)A->data;
    g->a_row = A->stride[0];
    g->b = (const uint16_t*)Bg->data;
    g->b_row = Bg->stride[0];
    g->idx = (const int32_t*)I->data;
    g->idx_pitch = I->rank == 1 ? 1 : I->stride[0];
    g->ctx = CX ? (const int32_t*)CX->data : nullptr;
    g->q = (uint16_t*)Q->data;
    g->q_row = Q->stride[0];
    g->q_head = Q->stride[1];
    g->k = (uint16_t*)K->data;
    g->k_row = K->stride[0];
    g->k_head = K->stride[1];
    g->v = (uint16_t*)V->data;
    g->v_row = V->stride[0];
    g->v_head = V->stride[1];
    g->g = (float*)G->data;
    g->g_row = G->stride[0];
    g->beta = (float*)BE->data;
    g->beta_row = BE->stride[0];
    g->T = T;
    g->n_head_k = hk;
    g->n_head_v = hv;
    g->dk = dk;
    g->dv = dv;
    g->width = width;
    return RAD_OK;
}

/* "s0,s1,s2" (optionally in brackets, spaces allowed): three non-negative counts; false otherwise. */
static bool parse_sections(const char* s, int (&out)[3]) {
    if (!s) return false;
    int n = 0;
    long long cur = -1;
    for (const char* c = s;; ++c) {
        if (*c >= '0' && *c <= '9') {
            cur = (cur < 0 ? 0 : cur) * 10 + (*c - '0');
            if (cur > 1 << 20) return false;
        } else if (*c == ',' || *c == ']' || *c == '\0') {
            if (cur < 0 || n >= 3) return false;
            out[n++] = (int)cur;
            cur = -1;
            if (*c != ',') {
                for (const char* d = *c ? c + 1 : c; *d; ++d)
                    if (*d != ' ') return false;
                return n == 3;
            }
        } else if (!(*c == ' ' || (*c == '[' && n == 0 && cur < 0))) {
            return false;
        }
    }
}

/* ridgefill_attn_kv_fill: k, v bf16 [T, Hkv, 256] (last stride 1, rows and heads 16-byte aligned), k_norm bf16 or
 * f32 [256] dense, positions i32 [T] or [3, T] (last stride 1), slot_mapping i32 [T] dense, cache bf16
 * [2, slots, Hkv, 256] (last stride 1, its other strides and base 16-byte aligned), k_out bf16 [T, Hkv, 256] or
 * absent (it may be k itself). rope_dim a multiple of 16 in [16, 256]; rope_theta > 1; eps >= 0 (1e-6 when
 * absent); rope_mode absent / "neox", "mrope" or "imrope", the last two with rope_sections "s0,s1,s2" summing
 * to rope_dim / 2. */
extern "C" int ridgefill_attn_kv_parse(const RadArgs* a, RidgeFillAttnKv* g) {
    *g = RidgeFillAttnKv{};
    const RadTensor* K = rad_arg_in(a, AK_K);
    const RadTensor* V = rad_arg_in(a, AK_V);
    const RadTensor* W = rad_arg_in(a, AK_W);
    const RadTensor* P = rad_arg_in(a, AK_POS);
    const RadTensor* S = rad_arg_in(a, AK_SLOTS);
    const RadTensor* C = rad_arg_in(a, AK_CACHE);
    const RadTensor* KO = rad_arg_in(a, AK_K_OUT);
    long long T = 0, hkv = 0, D = 0, R = 0;
    if (!K || !V || !W || !P || !S || !C) return RAD_E_INVAL;
    if (!rad_args_geti(a, "M", &T) || !rad_args_geti(a, "n_head_kv", &hkv) || !rad_args_geti(a, "head_dim", &D) ||
        !rad_args_geti(a, "rope_dim", &R))
        return RAD_E_INVAL;
    const double theta = rad_args_getf_or(a, "rope_theta", NAN), eps = rad_args_getf_or(a, "eps", 1e-6);
    if (!(theta > 1.0) || !std::isfinite(theta) || !(eps >= 0.0) || !std::isfinite(eps)) return RAD_E_INVAL;
    static const char* const modes[] = { "neox", "mrope", "imrope" };
    const char* m = rad_args_gets(a, "rope_mode");
    const int mode = m ? which(m, modes, 3) : RIDGEFILL_ROPE_NEOX;
    if (mode < 0) return RAD_E_INVAL;
    int sec[3] = { 0, 0, 0 };
    if (mode != RIDGEFILL_ROPE_NEOX && (!parse_sections(rad_args_gets(a, "rope_sections"), sec) ||
                                        (long long)sec[0] + sec[1] + sec[2] != R / 2))
        return RAD_E_INVAL;
    if (D != 256 || R < 16 || R > D || R % 16) return RAD_E_UNSUPPORTED;
    if (hkv <= 0 || T < 0) return RAD_E_SHAPE;
    if (K->dtype != RAD_BF16 || V->dtype != RAD_BF16 || (W->dtype != RAD_BF16 && W->dtype != RAD_F32) ||
        P->dtype != RAD_I32 || S->dtype != RAD_I32 || C->dtype != RAD_BF16 || (KO && KO->dtype != RAD_BF16))
        return RAD_E_DTYPE;
    const RadTensor* rows[3] = { K, V, KO };
    for (const RadTensor* t : rows)
        if (t && (t->rank != 3 || t->shape[0] != T || t->shape[1] != hkv || t->shape[2] != D || t->stride[2] != 1))
            return RAD_E_SHAPE;
    if (rad_tensor_numel(W) != D || !dense(W)) return RAD_E_SHAPE;
    if (P->rank == 1 ? (P->shape[0] != T || P->stride[0] != 1)
                     : (P->rank != 2 || P->shape[0] != 3 || P->shape[1] != T || P->stride[1] != 1))
        return RAD_E_SHAPE;
    if (rad_tensor_numel(S) != T || !dense(S)) return RAD_E_SHAPE;
    if (C->rank != 4 || C->shape[0] != 2 || C->shape[2] != hkv || C->shape[3] != D || C->stride[3] != 1) return RAD_E_SHAPE;
    /* 16-byte loads and stores: eight elements a lane. */
    uint64_t align = (uint64_t)(uintptr_t)K->data | (uint64_t)(uintptr_t)V->data | (uint64_t)(uintptr_t)C->data |
                     (uint64_t)(K->stride[0] * 2) | (uint64_t)(K->stride[1] * 2) | (uint64_t)(V->stride[0] * 2) |
                     (uint64_t)(V->stride[1] * 2) | (uint64_t)(C->stride[0] * 2) | (uint64_t)(C->stride[1] * 2) |
                     (uint64_t)(C->stride[2] * 2);
    if (KO) align |= (uint64_t)(uintptr_t)KO->data | (uint64_t)(KO->stride[0] * 2) | (uint64_t)(KO->stride[1] * 2);
    if (align % 16) return RAD_E_STRIDE;
    g->k = (const uint16_t*)K->data;
    g->k_row = K->stride[0];
    g->k_head = K->stride[1];
    g->v = (const uint16_t*)V->data;
    g->v_row = V->stride[0];
    g->v_head = V->stride[1];
    g->w = W->data;
    g->w_f32 = W->dtype == RAD_F32;
    g->pos = (const int32_t*)P->data;
    g->n_planes = P->rank == 1 ? 1 : 3;
    g->pos_plane = P->rank == 1 ? 0 : P->stride[0];
    g->slots = (const int32_t*)S->data;
    g->cache = (uint16_t*)C->data;
    g->c_kv = C->stride[0];
    g->c_slot = C->stride[1];
    g->c_head = C->stride[2];
    g->n_slots = C->shape[1];
    g->k_out = KO ? (uint16_t*)KO->data : nullptr;
    g->ko_row = KO ? KO->stride[0] : 0;
    g->ko_head = KO ? KO->stride[1] : 0;
    g->T = T;
    g->n_head_kv = hkv;
    g->head_dim = D;
    g->rope_dim = R;
    g->theta = theta;
    g->eps = (float)eps;
    g->mode = mode;
    for (int i = 0; i < 3; ++i) g->sections[i] = sec[i];
    return RAD_OK;
}

/* ridgefill_quant_act_i8g: x bf16 [M, n] (row pitch free, last stride 1), q i8 [M, n], s f32 [M, n/group]. */
extern "C" int ridgefill_quant_parse(const RadArgs* a, RidgeFillQuant* g) {
    *g = RidgeFillQuant{};
    const RadTensor* X = rad_arg_in(a, QA_X);
    const RadTensor* Q = rad_arg_in(a, QA_Q);
    const RadTensor* S = rad_arg_in(a, QA_S);
    long long n = 0, group = 0;
    if (!X || !Q || !S || !rad_args_geti(a, "n", &n) || !rad_args_geti(a, "group", &group)) return RAD_E_INVAL;
    if (X->dtype != RAD_BF16 || Q->dtype != RAD_I8 || S->dtype != RAD_F32) return RAD_E_DTYPE;
    if (X->rank != 2 || Q->rank != 2 || S->rank != 2) return RAD_E_SHAPE;
    if (group <= 0 || n % group != 0 || group % 8 != 0) return RAD_E_SHAPE;
    const int64_t M = X->shape[0];
    if (X->shape[1] != n || Q->shape[0] != M || Q->shape[1] != n || S->shape[0] != M || S->shape[1] != n / group)
        return RAD_E_SHAPE;
    if (X->stride[1] != 1 || Q->stride[1] != 1 || S->stride[1] != 1) return RAD_E_STRIDE;
    /* 16-byte vector loads of x, 8-byte stores of q. */
    if ((uintptr_t)X->data % 16 || (X->stride[0] * 2) % 16 || (uintptr_t)Q->data % 8 || Q->stride[0] % 8)
        return RAD_E_STRIDE;
    g->x = (const uint16_t*)X->data;
    g->ldx = X->stride[0];
    g->q = (int8_t*)Q->data;
    g->ldq = Q->stride[0];
    g->s = (float*)S->data;
    g->lds = S->stride[0];
    g->M = M;
    g->K = n;
    g->group = group;
    return RAD_OK;
}

/* ridgefill_gdn_fill: q (optional, with o), k [T, Hk, dk], v [T, Hv, dv] bf16, g and beta f32 [T, Hv],
 * state f32 [slots, Hv, dv, dk] (slot and head strides free, the [dv, dk] plane packed), state_idx
 * [n_seq] or [n_seq, pitch], cu_seqlens i32 [n_seq + 1], o bf16 [T, Hv, dv]. Head dims 128 and
 * chunk 64 are what the device row serves; Hv a multiple of Hk. */
extern "C" int ridgefill_gdn_parse(const RadArgs* a, RidgeFillGdn* g) {
    *g = RidgeFillGdn{};
    const RadTensor* Q = rad_arg_in(a, GD_Q);
    const RadTensor* Kt = rad_arg_in(a, GD_K);
    const RadTensor* V = rad_arg_in(a, GD_V);
    const RadTensor* G = rad_arg_in(a, GD_G);
    const RadTensor* Bt = rad_arg_in(a, GD_BETA);
    const RadTensor* St = rad_arg_in(a, GD_STATE);
    const RadTensor* Si = rad_arg_in(a, GD_STATE_IDX);
    const RadTensor* Cu = rad_arg_in(a, GD_CU);
    const RadTensor* O = rad_arg_in(a, GD_O);
    long long hk = 0, hv = 0, dk = 0, dv = 0, chunk = 0;
    if (!Kt || !V || !G || !Bt || !St || !Si || !Cu || (!Q) != (!O) || !rad_args_geti(a, "n_head_k", &hk) ||
        !rad_args_geti(a, "n_head_v", &hv) || !rad_args_geti(a, "head_k", &dk) || !rad_args_geti(a, "head_v", &dv) ||
        !rad_args_geti(a, "chunk", &chunk))
        return RAD_E_INVAL;
    if (Kt->dtype != RAD_BF16 || V->dtype != RAD_BF16 || (Q && Q->dtype != RAD_BF16) || (O && O->dtype != RAD_BF16) ||
        G->dtype != RAD_F32 || Bt->dtype != RAD_F32 || St->dtype != RAD_F32 || Cu->dtype != RAD_I32)
        return RAD_E_DTYPE;
    int64_t n_seq = 0, pitch = 0;
    const int rc = index_rows(Si, &n_seq, &pitch);
    if (rc != RAD_OK) return rc;
    if (hk <= 0 || hv <= 0 || hv % hk != 0 || dk != 128 || dv != 128 || chunk != 64) return RAD_E_UNSUPPORTED;
    if (Kt->rank != 3 || V->rank != 3 || G->rank != 2 || Bt->rank != 2 || St->rank != 4 ||
        (Q && Q->rank != 3) || (O && O->rank != 3))
        return RAD_E_SHAPE;
    const int64_t T = Kt->shape[0];
    if (Kt->shape[1] != hk || Kt->shape[2] != dk || V->shape[0] != T || V->shape[1] != hv || V->shape[2] != dv ||
        G->shape[0] != T || G->shape[1] != hv || Bt->shape[0] != T || Bt->shape[1] != hv || St->shape[1] != hv ||
        St->shape[2] != dv || St->shape[3] != dk || rad_tensor_numel(Cu) != n_seq + 1 ||
        (Q && (Q->shape[0] != T || Q->shape[1] != hk || Q->shape[2] != dk)) ||
        (O && (O->shape[0] != T || O->shape[1] != hv || O->shape[2] != dv)))
        return RAD_E_SHAPE;
    if (Kt->stride[2] != 1 || V->stride[2] != 1 || G->stride[1] != 1 || Bt->stride[1] != 1 || !dense(Cu) ||
        St->stride[3] != 1 || St->stride[2] != dk || (Q && Q->stride[2] != 1) || (O && O->stride[2] != 1))
        return RAD_E_STRIDE;
    /* 16-byte vector loads of k, v, q rows and of the state plane. */
    if ((uintptr_t)Kt->data % 16 || (uintptr_t)V->data % 16 || (Kt->stride[0] | Kt->stride[1]) % 8 ||
        (V->stride[0] | V->stride[1]) % 8 || (uintptr_t)St->data % 16 || (St->stride[0] | St->stride[1]) % 4 ||
        (Q && ((uintptr_t)Q->data % 16 || (Q->stride[0] | Q->stride[1]) % 8)) ||
        (O && ((uintptr_t)O->data % 16 || (O->stride[0] | O->stride[1]) % 8)))
        return RAD_E_STRIDE;
    g->q = Q ? (const uint16_t*)Q->data : nullptr;
    g->q_row = Q ? Q->stride[0] : 0;
    g->q_head = Q ? Q->stride[1] : 0;
    g->k = (const uint16_t*)Kt->data;
    g->k_row = Kt->stride[0];
    g->k_head = Kt->stride[1];
    g->v = (const uint16_t*)V->data;
    g->v_row = V->stride[0];
    g->v_head = V->stride[1];
    g->g = (const float*)G->data;
    g->g_row = G->stride[0];
    g->beta = (const float*)Bt->data;
    g->b_row = Bt->stride[0];
    g->state = (float*)St->data;
    g->st_slot = St->stride[0];
    g->st_head = St->stride[1];
    g->n_states = St->shape[0];
    g->state_idx = (const int32_t*)Si->data;
    g->idx_pitch = pitch;
    g->cu = (const int32_t*)Cu->data;
    g->n_seq = n_seq;
    g->o = O ? (uint16_t*)O->data : nullptr;
    g->o_row = O ? O->stride[0] : 0;
    g->o_head = O ? O->stride[1] : 0;
    g->T = T;
    g->n_head_k = hk;
    g->n_head_v = hv;
    g->dk = dk;
    g->dv = dv;
    g->chunk = chunk;
    g->scale = (float)rad_args_getf_or(a, "scale", 1.0 / std::sqrt((double)dk));
    return RAD_OK;
}
