/* parse.cpp -- operand checks for every row of the B200 RidgeFill library: a RadArgs reduced to one of
 * the parsed structs of ridgefill.h, or a named refusal.
 *
 * Each parse is written as the list of what its operands and parameters must be, in the order in which
 * their refusals take precedence, on a `Gate` (below): the first requirement that fails fixes the code,
 * and every later one is skipped. After the gate, an op's shape relations (one predicate) and then the
 * parsed struct's fields. The reference ops refuse what the reference plugin refuses, with the same code
 * and the same code winning when an operand set breaks several rules (kernels/host_ref.cpp:16-282,
 * 435-463; the new ops follow the same conventions). Nothing here reads an operand's VALUES (they are
 * device memory on a device row): values such as cu_last are checked where the kernel reads them, with
 * the reference's fail-safe.
 */
#include "ridgefill.h"

#include <cmath>
#include <cstring>
#include <initializer_list>
#include <type_traits>

namespace {

bool packed(const RadTensor* t) { return rad_tensor_is_contiguous(t) != 0; }

/* The position of `s` in `names`, -1 when it names none (or is null). */
int name_index(const char* s, const char* const* names, int n) {
    if (!s) return -1;
    for (int i = 0; i < n; ++i)
        if (!std::strcmp(s, names[i])) return i;
    return -1;
}

/* Elements one (slot, head) of a [slots, heads, ...] pool holds: the product of the axes after the second. */
int64_t cell_elems(const RadTensor* t) {
    int64_t n = 1;
    for (uint32_t ax = 2; ax < t->rank; ++ax) n *= t->shape[ax];
    return n;
}

/* An N|D pair pool [slots, heads, 1, 2] or [slots, heads, 2, 1]: the element distance from N to D, which
 * is the stride of the cell's axis of extent 2; 0 when the cell is not such a pair. */
int64_t pair_gap(const RadTensor* t) {
    if (t->rank < 3 || cell_elems(t) != 2) return 0;
    for (uint32_t ax = 2; ax < t->rank; ++ax)
        if (t->shape[ax] == 2) return t->stride[ax];
    return 0;
}

/* A slot index operand, [n_seq] or [n_seq, pitch]: the sequence count and the row pitch. */
struct SlotRows {
    int64_t rows = 0, pitch = 0;
};

/* The refusal of one parse. Every requirement is a no-op once one has failed, so a parse is a chain of
 * requirements; conditions that look inside an operand are callables, evaluated only while the operands
 * they read are known to be given. */
class Gate {
   public:
    explicit Gate(const RadArgs* a) : a_(a) {}

    int code() const { return rc_; }
    bool open() const { return rc_ == RAD_OK; }
    const RadTensor* at(int pos) const { return rad_arg_in(a_, pos); }

    /* RAD_E_INVAL unless every listed operand is given. */
    Gate& given(std::initializer_list<int> pos) {
        for (int p : pos)
            if (!at(p)) return fail(RAD_E_INVAL);
        return *this;
    }
    /* RAD_E_INVAL unless the two operands are both given or both absent. */
    Gate& paired(int p, int q) { return (!at(p)) != (!at(q)) ? fail(RAD_E_INVAL) : *this; }
    /* `code` unless `ok` (a bool, or a callable returning one, called only while the gate is open). */
    template <class F>
    Gate& holds(int code, F&& ok) {
        if (open() && !test(ok)) rc_ = code;
        return *this;
    }
    /* RAD_E_INVAL unless integer parameter `key` is given; its value into *out. */
    Gate& integer(const char* key, long long* out) {
        if (open() && !rad_args_geti(a_, key, out)) rc_ = RAD_E_INVAL;
        return *this;
    }
    /* RAD_E_DTYPE unless each listed operand is absent or of type `dt`. */
    Gate& typed(uint32_t dt, std::initializer_list<int> pos) {
        for (int p : pos)
            if (at(p) && at(p)->dtype != dt) return fail(RAD_E_DTYPE);
        return *this;
    }
    /* RAD_E_STRIDE unless each listed operand is absent or packed. */
    Gate& compact(std::initializer_list<int> pos) {
        for (int p : pos)
            if (at(p) && !packed(at(p))) return fail(RAD_E_STRIDE);
        return *this;
    }
    /* A slot index operand: i32 (else RAD_E_DTYPE), rank 1 or 2 with a unit last stride (else
     * RAD_E_STRIDE). An absent optional index passes. */
    Gate& slots(int pos, SlotRows* out) {
        const RadTensor* t = open() ? at(pos) : nullptr;
        if (!t) return *this;
        if (t->dtype != RAD_I32) return fail(RAD_E_DTYPE);
        if (t->rank != 1 && t->rank != 2) return fail(RAD_E_STRIDE);
        if (t->stride[t->rank - 1] != 1) return fail(RAD_E_STRIDE);
        out->rows = t->shape[0];
        out->pitch = t->rank == 1 ? 1 : t->stride[0];
        return *this;
    }
    /* An optional ridgefill_mask `bounds` operand read by another op: absent, or i32 (RAD_E_DTYPE),
     * packed (RAD_E_STRIDE) and of at least `need` elements (RAD_E_SHAPE). */
    Gate& limits(int pos, int64_t need, const int32_t** out) {
        *out = nullptr;
        const RadTensor* t = open() ? at(pos) : nullptr;
        if (!t) return *this;
        if (t->dtype != RAD_I32) return fail(RAD_E_DTYPE);
        if (!packed(t)) return fail(RAD_E_STRIDE);
        if (rad_tensor_numel(t) < need) return fail(RAD_E_SHAPE);
        *out = (const int32_t*)t->data;
        return *this;
    }

   private:
    Gate& fail(int code) {
        if (open()) rc_ = code;
        return *this;
    }
    template <class F>
    static bool test(F& f) {
        if constexpr (std::is_invocable_v<F&>) return f();
        else return static_cast<bool>(f);
    }

    const RadArgs* a_;
    int rc_ = RAD_OK;
};

/* A state pool [slots, heads, sd0, sd1] at its own strides. */
struct Pool4 {
    int64_t slot, head, row, col, slots;
};
Pool4 pool4(const RadTensor* t) { return { t->stride[0], t->stride[1], t->stride[2], t->stride[3], t->shape[0] }; }

/* The widest word every address, pitch and row width of a select pair is a multiple of: 16, 4 or 1
 * bytes (the device row moves a row in such words). */
int copy_unit(const RidgeFillCopy& c) {
    const uint64_t bits = (uint64_t)(uintptr_t)c.src | (uint64_t)(uintptr_t)c.dst | (uint64_t)c.src_pitch |
                          (uint64_t)c.dst_pitch | (uint64_t)c.row_bytes;
    const uint64_t low = bits & (~bits + 1);   /* the lowest set bit; 0 when every term is 0 */
    if (low == 0 || low >= 16) return 16;
    return low >= 4 ? 4 : 1;
}

/* Select pair k (source `from`, destination `to`): absent together, or one whole-byte dtype, rank 2 with
 * the same row width and at least n rows each, unit last strides. */
int select_pair(const RadArgs* a, int from, int to, int64_t n, RidgeFillCopy* c) {
    *c = RidgeFillCopy{};
    Gate gate(a);
    gate.paired(from, to);
    const RadTensor* s = gate.at(from);
    const RadTensor* d = gate.at(to);
    if (!gate.open() || !s) return gate.code();
    const int bits = rad_dtype_bits(s->dtype);
    gate.holds(RAD_E_DTYPE, d->dtype == s->dtype && bits > 0 && bits % 8 == 0)
        .holds(RAD_E_SHAPE, s->rank == 2 && d->rank == 2 && s->shape[1] == d->shape[1] && s->shape[0] >= n &&
                                d->shape[0] >= n)
        .holds(RAD_E_STRIDE, [&] { return s->stride[1] == 1 && d->stride[1] == 1; });
    if (!gate.open()) return gate.code();
    const int64_t elem = bits / 8;
    c->src = (const unsigned char*)s->data;
    c->dst = (unsigned char*)d->data;
    c->src_pitch = elem * s->stride[0];
    c->dst_pitch = elem * d->stride[0];
    c->row_bytes = elem * s->shape[1];
    c->word = copy_unit(*c);
    return RAD_OK;
}

}  // namespace

/* ridgefill_mask: cu_last, token ids, positions ([b], or [c, b] whose row 0 is the index), the class score
 * table (needed by the class and random modes only), the mask, its bounds and the optional zeroed rows. */
extern "C" int ridgefill_mask_parse(const RadArgs* a, RidgeFillMask* g) {
    static const char* const kModes[] = { "none", "class", "random", "all", "step" };
    *g = RidgeFillMask{};
    g->mode = name_index(rad_args_gets(a, "mode"), kModes, 5);
    g->share = rad_args_getf_or(a, "share", NAN);
    const bool ranked = g->mode == RIDGEFILL_MODE_CLASS || g->mode == RIDGEFILL_MODE_RANDOM;
    long long seed = 0;
    Gate gate(a);
    gate.given({ MK_CU, MK_TOKENS, MK_POS, MK_MASK, MK_BOUNDS })
        .holds(RAD_E_INVAL, !ranked || gate.at(MK_SCORE))
        .holds(RAD_E_INVAL, g->mode >= 0)
        .integer("seed", &seed)
        .holds(RAD_E_INVAL, g->share >= 0.0 && g->share <= 1.0)
        .typed(RAD_I32, { MK_CU, MK_TOKENS, MK_POS, MK_MASK, MK_BOUNDS })
        .typed(RAD_F32, { MK_SCORE })
        .typed(RAD_I32, { MK_ZEROS })
        .compact({ MK_CU, MK_TOKENS, MK_MASK, MK_BOUNDS, MK_SCORE, MK_ZEROS });
    if (!gate.open()) return gate.code();
    const RadTensor* pos = gate.at(MK_POS);
    const RadTensor* score = gate.at(MK_SCORE);
    const RadTensor* zeros = gate.at(MK_ZEROS);
    const int64_t b = rad_tensor_numel(gate.at(MK_TOKENS));
    const bool fits = (pos->rank == 1 || pos->rank == 2) && pos->shape[pos->rank - 1] >= b &&
                      rad_tensor_numel(gate.at(MK_CU)) >= 2 && rad_tensor_numel(gate.at(MK_BOUNDS)) >= 4;
    if (!fits) return RAD_E_SHAPE;
    g->cu_last = (const int32_t*)gate.at(MK_CU)->data;
    g->tokens = (const int32_t*)gate.at(MK_TOKENS)->data;
    g->b = b;
    g->positions = (const int32_t*)pos->data;
    g->pos_stride = pos->stride[pos->rank - 1];
    if (score) {
        g->score = (const float*)score->data;
        g->vocab = rad_tensor_numel(score);
    }
    g->mask = (int32_t*)gate.at(MK_MASK)->data;
    g->n = rad_tensor_numel(gate.at(MK_MASK));
    g->bounds = (int32_t*)gate.at(MK_BOUNDS)->data;
    if (zeros) {
        g->zeros = (int32_t*)zeros->data;
        g->n_zeros = rad_tensor_numel(zeros);
    }
    g->seed = seed;
    return RAD_OK;
}

/* ridgefill_rho_update: a [n, heads] at any strides (bf16 or f32), the mask, A_log and dt_bias per head, the
 * N|D pair pool, one sequence's slot index, optional bounds. */
extern "C" int ridgefill_rho_parse(const RadArgs* a, RidgeFillRho* g) {
    *g = RidgeFillRho{};
    SlotRows idx;
    long long heads = 0;
    Gate gate(a);
    gate.given({ RH_A, RH_MASK, RH_ALOG, RH_DTBIAS, RH_ND, RH_SIDX })
        .holds(RAD_E_DTYPE, [&] { return gate.at(RH_A)->dtype == RAD_BF16 || gate.at(RH_A)->dtype == RAD_F32; })
        .typed(RAD_I32, { RH_MASK })
        .typed(RAD_F32, { RH_ALOG, RH_DTBIAS, RH_ND })
        .slots(RH_SIDX, &idx)
        .limits(RH_BOUNDS, 1, &g->bounds)
        .holds(RAD_E_STRIDE, [&] { return gate.at(RH_A)->rank == 2; })
        .compact({ RH_MASK, RH_ALOG, RH_DTBIAS })
        .integer("n_head", &heads);
    if (!gate.open()) return gate.code();
    const RadTensor* av = gate.at(RH_A);
    const RadTensor* nd = gate.at(RH_ND);
    const int64_t gap = pair_gap(nd);
    const bool fits = av->shape[1] == heads && rad_tensor_numel(gate.at(RH_MASK)) >= av->shape[0] &&
                      rad_tensor_numel(gate.at(RH_ALOG)) == heads && rad_tensor_numel(gate.at(RH_DTBIAS)) == heads &&
                      nd->shape[1] == heads && gap != 0 && idx.rows == 1;   /* one sequence a call */
    if (!fits) return RAD_E_SHAPE;
    g->a = av->data;
    g->a_pitch = av->stride[0];
    g->a_col = av->stride[1];
    g->a_bf16 = av->dtype == RAD_BF16;
    g->mask = (const int32_t*)gate.at(RH_MASK)->data;
    g->a_log = (const float*)gate.at(RH_ALOG)->data;
    g->dt_bias = (const float*)gate.at(RH_DTBIAS)->data;
    g->nd = (float*)nd->data;
    g->nd_slot = nd->stride[0];
    g->nd_head = nd->stride[1];
    g->nd_inner = gap;
    g->n_states = nd->shape[0];
    g->state_idx = (const int32_t*)gate.at(RH_SIDX)->data;
    g->n = av->shape[0];
    g->n_head = av->shape[1];
    return RAD_OK;
}

/* ridgefill_state_correct: the state pool [slots, heads, sd0, sd1] at any strides, the applied-scale pool
 * [slots, heads, 1...], C packed as [heads, sd0, sd1] whatever its rank, the optional N|D pool with its
 * index, three slot indices of equal rows, optional bounds. */
extern "C" int ridgefill_correct_parse(const RadArgs* a, RidgeFillCorrect* g) {
    static const char* const kModes[] = { "undo", "apply" };
    *g = RidgeFillCorrect{};
    long long heads = 0, sd0 = 0, sd1 = 0;
    SlotRows st_rows, ap_rows, nd_rows;
    g->apply = name_index(rad_args_gets(a, "mode"), kModes, 2);
    const double alpha = rad_args_getf_or(a, "alpha", NAN);
    Gate gate(a);
    gate.given({ SC_STATE, SC_STATE_IDX, SC_APPLIED, SC_APPLIED_IDX, SC_C })
        .paired(SC_ND, SC_ND_IDX)
        .typed(RAD_F32, { SC_STATE, SC_APPLIED, SC_C, SC_ND })
        .holds(RAD_E_INVAL, g->apply >= 0)
        .integer("n_head", &heads)
        .integer("sd0", &sd0)
        .integer("sd1", &sd1)
        .holds(RAD_E_INVAL, g->apply == 0 || std::isfinite(alpha))
        .slots(SC_STATE_IDX, &st_rows)
        .slots(SC_APPLIED_IDX, &ap_rows)
        .slots(SC_ND_IDX, &nd_rows)
        .limits(SC_BOUNDS, 2, &g->bounds)
        .holds(RAD_E_SHAPE, [&] { return ap_rows.rows == st_rows.rows && (!gate.at(SC_ND_IDX) || nd_rows.rows == st_rows.rows); });
    if (!gate.open()) return gate.code();
    const RadTensor* st = gate.at(SC_STATE);
    const RadTensor* ap = gate.at(SC_APPLIED);
    const RadTensor* c = gate.at(SC_C);
    const RadTensor* nd = gate.at(SC_ND);
    const bool state_ok = st->rank == 4 && st->shape[1] == heads && st->shape[2] == sd0 && st->shape[3] == sd1;
    const bool c_ok = packed(c) && rad_tensor_numel(c) == heads * sd0 * sd1;
    const bool applied_ok = ap->rank >= 2 && ap->shape[1] == heads && cell_elems(ap) == 1;
    const bool nd_ok = !nd || (nd->shape[1] == heads && pair_gap(nd) != 0);
    if (!(state_ok && c_ok && applied_ok && nd_ok)) return RAD_E_SHAPE;
    const Pool4 sp = pool4(st);
    g->state = (float*)st->data;
    g->st_slot = sp.slot;
    g->st_head = sp.head;
    g->st_row = sp.row;
    g->st_col = sp.col;
    g->st_states = sp.slots;
    g->applied = (float*)ap->data;
    g->ap_slot = ap->stride[0];
    g->ap_head = ap->stride[1];
    g->ap_states = ap->shape[0];
    g->c = (const float*)c->data;
    g->c_head = sd0 * sd1;   /* C is read packed: its element count, not its rank, is the contract */
    g->c_row = sd1;
    if (nd) {
        g->nd = (const float*)nd->data;
        g->nd_slot = nd->stride[0];
        g->nd_head = nd->stride[1];
        g->nd_inner = pair_gap(nd);
        g->nd_states = nd->shape[0];
        g->nd_idx = (const int32_t*)gate.at(SC_ND_IDX)->data;
        g->nd_pitch = nd_rows.pitch;
    }
    g->st_idx = (const int32_t*)gate.at(SC_STATE_IDX)->data;
    g->st_pitch = st_rows.pitch;
    g->ap_idx = (const int32_t*)gate.at(SC_APPLIED_IDX)->data;
    g->ap_pitch = ap_rows.pitch;
    g->n_seq = st_rows.rows;
    g->n_head = heads;
    g->sd0 = sd0;
    g->sd1 = sd1;
    g->alpha = (float)alpha;
    return RAD_OK;
}

/* ridgefill_state_read: the state pool, a slot index, and a packed f32 output of at least
 * n_seq * heads * sd0 * sd1 elements, written from its first element. */
extern "C" int ridgefill_state_read_parse(const RadArgs* a, RidgeFillStateRead* g) {
    *g = RidgeFillStateRead{};
    long long heads = 0, sd0 = 0, sd1 = 0;
    SlotRows rows;
    Gate gate(a);
    gate.given({ SR_STATE, SR_STATE_IDX, SR_OUT })
        .integer("n_head", &heads)
        .integer("sd0", &sd0)
        .integer("sd1", &sd1)
        .typed(RAD_F32, { SR_STATE, SR_OUT })
        .slots(SR_STATE_IDX, &rows)
        .compact({ SR_OUT });
    if (!gate.open()) return gate.code();
    const RadTensor* st = gate.at(SR_STATE);
    const RadTensor* out = gate.at(SR_OUT);
    if (!(st->rank == 4 && st->shape[1] == heads && st->shape[2] == sd0 && st->shape[3] == sd1 &&
          rad_tensor_numel(out) >= rows.rows * heads * sd0 * sd1))
        return RAD_E_SHAPE;
    const Pool4 sp = pool4(st);
    g->state = (const float*)st->data;
    g->st_slot = sp.slot;
    g->st_head = sp.head;
    g->st_row = sp.row;
    g->st_col = sp.col;
    g->n_states = sp.slots;
    g->idx = (const int32_t*)gate.at(SR_STATE_IDX)->data;
    g->idx_pitch = rows.pitch;
    g->out = (float*)out->data;
    g->n_seq = rows.rows;
    g->n_head = heads;
    g->sd0 = sd0;
    g->sd1 = sd1;
    return RAD_OK;
}

/* ridgefill_select: the mask, then the x pair (required) and the q and s pairs (each optional as a pair). */
extern "C" int ridgefill_select_parse(const RadArgs* a, RidgeFillSelect* g) {
    *g = RidgeFillSelect{};
    Gate gate(a);
    gate.given({ SL_MASK, SL_X_SRC, SL_X }).typed(RAD_I32, { SL_MASK }).compact({ SL_MASK });
    if (!gate.open()) return gate.code();
    g->mask = (const int32_t*)gate.at(SL_MASK)->data;
    g->n = rad_tensor_numel(gate.at(SL_MASK));
    for (int k = 0; k < RIDGEFILL_SELECT_PAIRS; ++k)
        if (const int rc = select_pair(a, SL_X_SRC + k, SL_X + k, g->n, &g->pair[k])) return rc;
    return RAD_OK;
}

/* ridgefill_drop_rows: the mask and the routing ids [>= n, >= top_k] with a unit last stride. */
extern "C" int ridgefill_drop_parse(const RadArgs* a, RidgeFillDrop* g) {
    *g = RidgeFillDrop{};
    long long top_k = -1;
    Gate gate(a);
    gate.given({ DR_MASK, DR_IDS })
        .integer("top_k", &top_k)
        .holds(RAD_E_INVAL, [&] { return top_k >= 0; })
        .typed(RAD_I32, { DR_MASK, DR_IDS })
        .compact({ DR_MASK })
        .holds(RAD_E_STRIDE, [&] { return gate.at(DR_IDS)->rank != 2 || gate.at(DR_IDS)->stride[1] == 1; });
    if (!gate.open()) return gate.code();
    const RadTensor* ids = gate.at(DR_IDS);
    const int64_t n = rad_tensor_numel(gate.at(DR_MASK));
    if (!(ids->rank == 2 && ids->shape[0] >= n && ids->shape[1] >= top_k)) return RAD_E_SHAPE;
    g->mask = (const int32_t*)gate.at(DR_MASK)->data;
    g->n = n;
    g->ids = (int32_t*)ids->data;
    g->pitch = ids->stride[0];
    g->top_k = top_k;
    return RAD_OK;
}

/* ridgefill_hazard: cu_last, positions ([n] or [c, n]), optional bounds, the optional span (its extent is
 * all that is read), the meta pool [slots, ..., 2] with a unit last stride, its slot index, the count. */
extern "C" int ridgefill_hazard_parse(const RadArgs* a, RidgeFillHazard* g) {
    *g = RidgeFillHazard{};
    SlotRows rows;
    Gate gate(a);
    gate.given({ HZ_CU, HZ_POS, HZ_META, HZ_META_IDX, HZ_COUNT })
        .typed(RAD_I32, { HZ_CU, HZ_POS })
        .typed(RAD_F32, { HZ_META, HZ_COUNT })
        .compact({ HZ_CU, HZ_COUNT })
        .slots(HZ_META_IDX, &rows)
        .limits(HZ_BOUNDS, 2, &g->bounds);
    if (!gate.open()) return gate.code();
    const RadTensor* pos = gate.at(HZ_POS);
    const RadTensor* meta = gate.at(HZ_META);
    const RadTensor* span = gate.at(HZ_SPAN);
    const bool fits = rows.rows >= 1 && rad_tensor_numel(gate.at(HZ_CU)) >= 2 && rad_tensor_numel(gate.at(HZ_COUNT)) >= 1 &&
                      (pos->rank == 1 || pos->rank == 2) && meta->rank >= 2 && meta->shape[meta->rank - 1] == 2 &&
                      meta->stride[meta->rank - 1] == 1;
    if (!fits) return RAD_E_SHAPE;
    g->cu_last = (const int32_t*)gate.at(HZ_CU)->data;
    g->positions = (const int32_t*)pos->data;
    g->pos_stride = pos->stride[pos->rank - 1];
    g->span = span ? rad_tensor_numel(span) : 0;
    g->meta = (float*)meta->data;
    g->meta_slot = meta->stride[0];
    g->meta_states = meta->shape[0];
    g->meta_idx = (const int32_t*)gate.at(HZ_META_IDX)->data;
    g->count = (float*)gate.at(HZ_COUNT)->data;
    return RAD_OK;
}

/* ridgefill_gemm_nt_q (with_bias 0: operands a, a_scale, b, b_scale, y, a_sum, b_ref) and
 * ridgefill_gemm_nt_q_bias (with_bias 1: a, a_scale, b, b_scale, bias, y, acc). a_scale is required (an
 * i8a8 product has activation scales); a_sum and b_ref (zero-point terms of other dtypes) must be
 * absent. K must be a multiple of 128 and of `group`; `group` divides K (128, or K itself for
 * the late pass's per-row / per-column scaling); rows of a and codes of b start 16-byte aligned (the TMA
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
    const RadTensor* rows = with_bias ? rad_arg_in(a, GB_ROWS) : nullptr;
    long long M = 0, N = 0, K = 0, group = 0;
    const char* dt = rad_args_gets(a, "dtype");
    if (!A || !AS || !B || !BS || !Y || !rad_args_geti(a, "N", &N) || !rad_args_geti(a, "K", &K) ||
        !rad_args_geti(a, "group", &group) || !dt || std::strcmp(dt, "i8a8") != 0)
        return RAD_E_INVAL;
    if (!with_bias && (rad_arg_in(a, GQ_A_SUM) || rad_arg_in(a, GQ_B_REF))) return RAD_E_UNSUPPORTED;
    if (acc && rows) return RAD_E_UNSUPPORTED;   /* the debug sums and the row selection are separate forms */
    if (A->dtype != RAD_I8 || AS->dtype != RAD_F32 || B->dtype != RAD_I8 || BS->dtype != RAD_F32 ||
        Y->dtype != RAD_BF16 || (bias && bias->dtype != RAD_BF16) || (acc && acc->dtype != RAD_I32) ||
        (rows && rows->dtype != RAD_I32))
        return RAD_E_DTYPE;
    if (A->rank != 2 || B->rank != 2 || Y->rank != 2) return RAD_E_SHAPE;
    M = A->shape[0];
    if (group <= 0 || K <= 0 || K % group != 0 || K % 128 != 0 || group % 128 != 0 || N <= 0 || N % 16 != 0)
        return RAD_E_SHAPE;
    const int64_t blocks = K / group;
    if (A->shape[1] != K || B->shape[0] != N || B->shape[1] != K || Y->shape[0] != M || Y->shape[1] != N ||
        rad_tensor_numel(AS) != M * blocks || rad_tensor_numel(BS) != blocks * N || (bias && rad_tensor_numel(bias) != N) ||
        (acc && rad_tensor_numel(acc) != M * N * blocks) || (rows && rad_tensor_numel(rows) < M))
        return RAD_E_SHAPE;
    if (A->stride[1] != 1 || B->stride[1] != 1 || Y->stride[1] != 1 || !packed(BS) || (bias && !packed(bias)) ||
        (acc && !packed(acc)) || (rows && !packed(rows)))
        return RAD_E_STRIDE;
    if (AS->rank == 2 ? (AS->stride[1] != 1) : !packed(AS)) return RAD_E_STRIDE;
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
    g->rows = rows ? (const int32_t*)rows->data : nullptr;
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
    if (A->stride[1] != 1 || B->stride[1] != 1 || Y->stride[1] != 1 || !packed(bias) || (R && R->stride[1] != 1))
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
 * ctx_lens i32 [n_seq] or absent, q (or absent: its columns are then not computed) and k bf16 [T, Hk, dk], v bf16
 * [T, Hv, dv] (each head dense, rows and heads 16-byte aligned), g and beta f32 [T, Hv]. Head dims 128, width 4. */
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
    if (!X || !W || !AL || !DT || !ST || !CU || !A || !Bg || !I || !K || !V || !G || !BE) return RAD_E_INVAL;   /* q optional */
    if (!rad_args_geti(a, "M", &T) || !rad_args_geti(a, "n_head_k", &hk) || !rad_args_geti(a, "n_head_v", &hv) ||
        !rad_args_geti(a, "head_k", &dk) || !rad_args_geti(a, "head_v", &dv) || !rad_args_geti(a, "conv", &width))
        return RAD_E_INVAL;
    if (dk != 128 || dv != 128 || width != 4) return RAD_E_UNSUPPORTED;
    if (hk <= 0 || hv <= 0 || T < 0) return RAD_E_SHAPE;
    const int64_t C = 2 * hk * dk + hv * dv;
    if (X->dtype != RAD_BF16 || W->dtype != RAD_BF16 || (B0 && B0->dtype != RAD_BF16) || AL->dtype != RAD_F32 ||
        DT->dtype != RAD_F32 || ST->dtype != RAD_BF16 || CU->dtype != RAD_I32 || A->dtype != RAD_BF16 ||
        Bg->dtype != RAD_BF16 || I->dtype != RAD_I32 || (CX && CX->dtype != RAD_I32) || (Q && Q->dtype != RAD_BF16) ||
        K->dtype != RAD_BF16 || V->dtype != RAD_BF16 || G->dtype != RAD_F32 || BE->dtype != RAD_F32)
        return RAD_E_DTYPE;
    if (X->rank != 2 || X->shape[0] != T || X->shape[1] != C || X->stride[1] != 1) return X->rank == 2 && X->stride[1] != 1 ? RAD_E_STRIDE : RAD_E_SHAPE;
    if (W->rank != 2 || W->shape[0] != C || W->shape[1] != 4 || !packed(W)) return RAD_E_SHAPE;
    if (B0 && (rad_tensor_numel(B0) != C || !packed(B0))) return RAD_E_SHAPE;
    if (B0 && (uintptr_t)B0->data % 16) return RAD_E_STRIDE;
    if (rad_tensor_numel(AL) != hv || rad_tensor_numel(DT) != hv || !packed(AL) || !packed(DT)) return RAD_E_SHAPE;
    if (ST->rank != 3 || ST->shape[1] != 3 || ST->shape[2] != C || ST->stride[2] != 1 || ST->stride[1] != C) return RAD_E_SHAPE;
    if (CU->rank != 1 || CU->shape[0] < 1 || CU->stride[0] != 1) return RAD_E_SHAPE;
    const int64_t n_seq = CU->shape[0] - 1;
    if (I->rank == 1 ? (I->shape[0] < n_seq || I->stride[0] != 1) : (I->rank != 2 || I->shape[0] < n_seq || I->shape[1] < 1))
        return RAD_E_SHAPE;
    if (CX && (CX->rank != 1 || CX->shape[0] < n_seq || CX->stride[0] != 1)) return RAD_E_SHAPE;
    const RadTensor* per_head[4] = { A, Bg, G, BE };
    for (const RadTensor* t : per_head)
        if (t->rank != 2 || t->shape[0] != T || t->shape[1] != hv || t->stride[1] != 1) return RAD_E_SHAPE;
    if (Q && (Q->rank != 3 || Q->shape[0] != T || Q->shape[1] != hk || Q->shape[2] != dk || Q->stride[2] != 1)) return RAD_E_SHAPE;
    if (K->rank != 3 || K->shape[0] != T || K->shape[1] != hk || K->shape[2] != dk || K->stride[2] != 1) return RAD_E_SHAPE;
    if (V->rank != 3 || V->shape[0] != T || V->shape[1] != hv || V->shape[2] != dv || V->stride[2] != 1) return RAD_E_SHAPE;
    /* 16-byte loads of x, w, the bias and the state, 16-byte stores of q, k, v (eight channels a lane). */
    if (((uintptr_t)X->data | (Q ? (uintptr_t)Q->data : 0) | (uintptr_t)K->data | (uintptr_t)V->data | (uintptr_t)W->data |
         (uintptr_t)ST->data) % 16 ||
        (X->stride[0] * 2) % 16 || (Q && ((Q->stride[0] * 2) % 16 || (Q->stride[1] * 2) % 16)) || (K->stride[0] * 2) % 16 ||
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
    g->q = Q ? (uint16_t*)Q->data : nullptr;
    g->q_row = Q ? Q->stride[0] : 0;
    g->q_head = Q ? Q->stride[1] : 0;
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
    long long columns = 1;   /* optional: 0 computes only the gates and the conv state (ridgefill_gdn_in_proj wrote k, v) */
    if (rad_args_geti(a, "columns", &columns) && columns != 0 && columns != 1) return RAD_E_INVAL;
    g->columns = (int)columns;
    return RAD_OK;
}

/* ridgefill_gdn_in_proj: a i8 [T, K] (rows 16-byte aligned), a_scale f32 [T, 1], b i8 [N, K] the k|v rows of the
 * in-projection, b_scale f32 [1, N] (per-column scaling: group = K), w bf16 [N, 4] dense, bias bf16 [N] or absent,
 * conv state bf16 [slots, 3, N] (any slot and row pitch, last stride 1: the k|v channels of the pool), cu_seqlens
 * i32 [n_seq + 1], conv_idx i32 [n_seq] or [n_seq, >= 1], ctx_lens i32 [n_seq] or absent, k bf16 [T, Hk, 128],
 * v bf16 [T, Hv, 128] (rows and heads 16-byte aligned), tail bf16 [T, N] (rows 16-byte aligned). N = (Hk + Hv) 128. */
extern "C" int ridgefill_in_proj_parse(const RadArgs* a, RidgeFillInProj* g) {
    *g = RidgeFillInProj{};
    const RadTensor* A = rad_arg_in(a, IP_A);
    const RadTensor* AS = rad_arg_in(a, IP_A_SCALE);
    const RadTensor* B = rad_arg_in(a, IP_B);
    const RadTensor* BS = rad_arg_in(a, IP_B_SCALE);
    const RadTensor* W = rad_arg_in(a, IP_W);
    const RadTensor* B0 = rad_arg_in(a, IP_BIAS);
    const RadTensor* ST = rad_arg_in(a, IP_STATE);
    const RadTensor* CU = rad_arg_in(a, IP_CU);
    const RadTensor* I = rad_arg_in(a, IP_IDX);
    const RadTensor* CX = rad_arg_in(a, IP_CTX);
    const RadTensor* K = rad_arg_in(a, IP_K);
    const RadTensor* V = rad_arg_in(a, IP_V);
    const RadTensor* TL = rad_arg_in(a, IP_TAIL);
    long long T = 0, N = 0, Kd = 0, hk = 0, hv = 0, group = 0;
    const char* dt = rad_args_gets(a, "dtype");
    if (!A || !AS || !B || !BS || !W || !ST || !CU || !I || !K || !V || !TL || !dt || !rad_args_geti(a, "M", &T) ||
        !rad_args_geti(a, "N", &N) || !rad_args_geti(a, "K", &Kd) || !rad_args_geti(a, "n_head_k", &hk) ||
        !rad_args_geti(a, "n_head_v", &hv) || !rad_args_geti(a, "group", &group))
        return RAD_E_INVAL;
    if (std::strcmp(dt, "i8a8") != 0) return RAD_E_UNSUPPORTED;
    if (group != Kd) return RAD_E_UNSUPPORTED;   /* per-row activation, per-column weight scaling */
    if (A->dtype != RAD_I8 || AS->dtype != RAD_F32 || B->dtype != RAD_I8 || BS->dtype != RAD_F32 || W->dtype != RAD_BF16 ||
        (B0 && B0->dtype != RAD_BF16) || ST->dtype != RAD_BF16 || CU->dtype != RAD_I32 || I->dtype != RAD_I32 ||
        (CX && CX->dtype != RAD_I32) || K->dtype != RAD_BF16 || V->dtype != RAD_BF16 || TL->dtype != RAD_BF16)
        return RAD_E_DTYPE;
    if (T < 0 || hk <= 0 || hv <= 0 || N != (hk + hv) * 128 || Kd <= 0 || Kd % 128 != 0) return RAD_E_SHAPE;
    if (A->rank != 2 || A->shape[0] != T || A->shape[1] != Kd || B->rank != 2 || B->shape[0] != N || B->shape[1] != Kd ||
        rad_tensor_numel(AS) != T || rad_tensor_numel(BS) != N || W->rank != 2 || W->shape[0] != N || W->shape[1] != 4 ||
        (B0 && rad_tensor_numel(B0) != N) || ST->rank != 3 || ST->shape[1] != 3 || ST->shape[2] != N || TL->rank != 2 ||
        TL->shape[0] != T || TL->shape[1] != N)
        return RAD_E_SHAPE;
    if (CU->rank != 1 || CU->shape[0] < 1 || CU->stride[0] != 1) return RAD_E_SHAPE;
    const int64_t n_seq = CU->shape[0] - 1;
    if (I->rank == 1 ? (I->shape[0] < n_seq || I->stride[0] != 1) : (I->rank != 2 || I->shape[0] < n_seq || I->shape[1] < 1))
        return RAD_E_SHAPE;
    if (CX && (CX->rank != 1 || CX->shape[0] < n_seq || CX->stride[0] != 1)) return RAD_E_SHAPE;
    if (K->rank != 3 || K->shape[0] != T || K->shape[1] != hk || K->shape[2] != 128 || K->stride[2] != 1 ||
        V->rank != 3 || V->shape[0] != T || V->shape[1] != hv || V->shape[2] != 128 || V->stride[2] != 1)
        return RAD_E_SHAPE;
    if (A->stride[1] != 1 || B->stride[1] != 1 || !packed(AS) || !packed(BS) || !packed(W) || (B0 && !packed(B0)) ||
        ST->stride[2] != 1 || TL->stride[1] != 1)
        return RAD_E_STRIDE;
    /* TMA reads of a and b (16-byte bases and pitches); 16-byte loads and stores of b_scale, taps, state, k, v, tail */
    if (((uintptr_t)A->data | (uintptr_t)B->data | (uintptr_t)W->data | (uintptr_t)ST->data | (uintptr_t)K->data |
         (uintptr_t)V->data | (uintptr_t)TL->data | (uintptr_t)BS->data | (B0 ? (uintptr_t)B0->data : 0)) % 16 ||
        A->stride[0] % 16 || B->stride[0] % 16 || (ST->stride[0] * 2) % 16 || (ST->stride[1] * 2) % 16 ||
        (K->stride[0] * 2) % 16 || (K->stride[1] * 2) % 16 || (V->stride[0] * 2) % 16 || (V->stride[1] * 2) % 16 ||
        (TL->stride[0] * 2) % 16)
        return RAD_E_STRIDE;
    RidgeFillGemmQ& q = g->gemm;
    q.a = (const int8_t*)A->data;
    q.lda = A->stride[0];
    q.a_scale = (const float*)AS->data;
    q.ldas = 1;
    q.b = (const int8_t*)B->data;
    q.ldb = B->stride[0];
    q.b_scale = (const float*)BS->data;
    q.y = (uint16_t*)TL->data;
    q.ldy = TL->stride[0];
    q.M = T;
    q.N = N;
    q.K = Kd;
    q.group = Kd;
    g->w = (const uint16_t*)W->data;
    g->bias = B0 ? (const uint16_t*)B0->data : nullptr;
    g->state = (const uint16_t*)ST->data;
    g->st_slot = ST->stride[0];
    g->st_row = ST->stride[1];
    g->n_states = ST->shape[0];
    g->cu = (const int32_t*)CU->data;
    g->n_seq = n_seq;
    g->idx = (const int32_t*)I->data;
    g->idx_pitch = I->rank == 1 ? 1 : I->stride[0];
    g->ctx = CX ? (const int32_t*)CX->data : nullptr;
    g->k = (uint16_t*)K->data;
    g->k_row = K->stride[0];
    g->k_head = K->stride[1];
    g->v = (uint16_t*)V->data;
    g->v_row = V->stride[0];
    g->v_head = V->stride[1];
    g->n_k = hk * 128;
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
    const int mode = m ? name_index(m, modes, 3) : RIDGEFILL_ROPE_NEOX;
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
    if (rad_tensor_numel(W) != D || !packed(W)) return RAD_E_SHAPE;
    if (P->rank == 1 ? (P->shape[0] != T || P->stride[0] != 1)
                     : (P->rank != 2 || P->shape[0] != 3 || P->shape[1] != T || P->stride[1] != 1))
        return RAD_E_SHAPE;
    if (rad_tensor_numel(S) != T || !packed(S)) return RAD_E_SHAPE;
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
    SlotRows rows;
    Gate gate(a);
    gate.slots(GD_STATE_IDX, &rows);
    if (!gate.open()) return gate.code();
    const int64_t n_seq = rows.rows, pitch = rows.pitch;
    /* head dims 128 (the chunked tensor-core fill) or at most 64 each (the per-row fill), dk whole 16-byte rows */
    const bool wide = dk == 128 && dv == 128, small = dk >= 8 && dk <= 64 && dk % 8 == 0 && dv >= 1 && dv <= 64;
    if (hk <= 0 || hv <= 0 || hv % hk != 0 || !(wide || small) || chunk != 64) return RAD_E_UNSUPPORTED;
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
    if (Kt->stride[2] != 1 || V->stride[2] != 1 || G->stride[1] != 1 || Bt->stride[1] != 1 || !packed(Cu) ||
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
