/* ridgefill.h -- the C ABI of the B200 RidgeFill kernel library: operand positions, the formulas that
 * define each op's answer, the parsed-operand structs the CUDA kernels take by value, and the
 * extern "C" entry points.
 *
 * Interface it replaces: the reference's kernels/ridgefill.h (operand enums :50-57, shared formulas
 * :62-104, parsed structs :112-272, entry points :278-310). The op names, operand order, parameter
 * keys, refusal codes and the fail-safe rules are the reference's; the structs are this library's
 * own (they never cross the ABI: a row receives a RadArgs and parses it here).
 *
 * The formulas below are compiled for host and device alike (RIDGEFILL_HD), so the parse and the
 * kernels of one op read one definition.
 */
#ifndef RIDGEFILL_B200_H
#define RIDGEFILL_B200_H

#include "rad_abi.h"
#include "rad_plugin.h"

#include <math.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define RIDGEFILL_HD __host__ __device__ __forceinline__
#else
#define RIDGEFILL_HD static inline
#endif

/* ------------------------------------------------------------------ limits
 * RIDGEFILL_MASK_MAX_ROWS: the window's keys live in one CTA's shared memory (4 bytes a row); the
 * reference's device row stopped at 8,192 rows (kernels/ridgefill.h:32), this one at 49,152. The
 * host-side refusal is b > this (RAD_E_SHAPE), as the reference refuses b > 8,192
 * (kernels/mask.hip:82). */
enum { RIDGEFILL_MASK_MAX_ROWS = 49152, RIDGEFILL_SELECT_PAIRS = 3 };

/* Above this, softplus(x) is x to every bit f32 holds (kernels/ridgefill.h:37). */
#define RIDGEFILL_SOFTPLUS_THRESHOLD 20.0f

/* ridgefill_mask's `mode` (kernels/ridgefill.h:42). */
enum { RIDGEFILL_MODE_NONE = 0, RIDGEFILL_MODE_CLASS = 1, RIDGEFILL_MODE_RANDOM = 2, RIDGEFILL_MODE_ALL = 3,
       RIDGEFILL_MODE_STEP = 4 };

/* ------------------------------------------------------------------ operand positions (schema order)
 * The reference ops (kernels/ridgefill.h:51-57) and this library's new ones. */
enum { MK_CU = 0, MK_TOKENS, MK_POS, MK_SCORE, MK_MASK, MK_BOUNDS, MK_ZEROS };
enum { RH_A = 0, RH_MASK, RH_ALOG, RH_DTBIAS, RH_ND, RH_SIDX, RH_BOUNDS };
enum { SC_STATE = 0, SC_STATE_IDX, SC_APPLIED, SC_APPLIED_IDX, SC_C, SC_ND, SC_ND_IDX, SC_BOUNDS };
enum { SR_STATE = 0, SR_STATE_IDX, SR_OUT };
enum { SL_MASK = 0, SL_X_SRC, SL_Q_SRC, SL_S_SRC, SL_X, SL_Q, SL_S };
enum { DR_MASK = 0, DR_IDS };
enum { HZ_CU = 0, HZ_POS, HZ_BOUNDS, HZ_SPAN, HZ_META, HZ_META_IDX, HZ_COUNT };
/* ridgefill_gemm_nt_q (kernels/rows.cpp:74-76): a, a_scale, b, b_scale, y, a_sum, b_ref. */
enum { GQ_A = 0, GQ_A_SCALE, GQ_B, GQ_B_SCALE, GQ_Y, GQ_A_SUM, GQ_B_REF };
/* ridgefill_gemm_nt_q_bias (new): gemm_nt_q's operands, then the bias, an int32 debug output and the row
 * selection (ridgefill_select's mask: only rows whose entry is 1 are written). */
enum { GB_A = 0, GB_A_SCALE, GB_B, GB_B_SCALE, GB_BIAS, GB_Y, GB_ACC, GB_ROWS };
/* ridgefill_gemm_nt_bias (kernels/rows.cpp:67-70, oGemm): a, b, bias, res (optional), y. */
enum { GN_A = 0, GN_B, GN_BIAS, GN_RES, GN_Y };
/* ridgefill_quant_act_i8g (new; libr4d's quant_act_i8g operands, arch/ridgefill_layer.h:74-76). */
enum { QA_X = 0, QA_Q, QA_S };
/* ridgefill_gdn_fill (new; the chunk scan's operands, arch/qwen4exp_fill.h:55-60, without kkt:
 * the intra-chunk transform is computed inside the op). */
enum { GD_Q = 0, GD_K, GD_V, GD_G, GD_BETA, GD_STATE, GD_STATE_IDX, GD_CU, GD_O };
/* ridgefill_gdn_conv_prep (new; the operands of the DeltaNet block's conv_prep issue, arch/qwen4exp_fill.h:44-50,
 * with the gate written per row rather than in its in-chunk cumulative form). */
enum { CP_X = 0, CP_W, CP_BIAS, CP_A_LOG, CP_DT_BIAS, CP_STATE, CP_CU, CP_A, CP_B, CP_IDX, CP_CTX, CP_Q, CP_K, CP_V,
       CP_G, CP_BETA };
/* ridgefill_gdn_in_proj (new; the DeltaNet block's int8 in-projection of its k|v channels, arch/qwen4exp_fill.h:
 * 36-40, with conv_prep's convolution, SiLU and k norm in the projection's epilogue). */
enum { IP_A = 0, IP_A_SCALE, IP_B, IP_B_SCALE, IP_W, IP_BIAS, IP_STATE, IP_CU, IP_IDX, IP_CTX, IP_K, IP_V, IP_TAIL };
/* ridgefill_attn_kv_fill (new; the gated-attention block's K/V path in the lean fill, arch/qwen4exp_fill.h:104-114:
 * the k_norm, rope_k and kv_store issues after the k and v projections, as one op). */
enum { AK_K = 0, AK_V, AK_W, AK_POS, AK_SLOTS, AK_CACHE, AK_K_OUT };

/* ------------------------------------------------------------------ the shared formulas */

/* Wellons' lowbias32 finaliser (kernels/ridgefill.h:66-71). */
RIDGEFILL_HD uint32_t ridgefill_mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352dU;
    x ^= x >> 15;
    x *= 0x846ca68bU;
    x ^= x >> 16;
    return x;
}

/* The random selector's rank key of absolute position `position` under `seed`
 * (kernels/ridgefill.h:77-81): both seed halves folded through mix32, then the position's golden-ratio
 * step mixed in. */
RIDGEFILL_HD uint32_t ridgefill_row_hash(long long seed, uint32_t position) {
    const unsigned long long s = (unsigned long long)seed;
    const uint32_t folded = ridgefill_mix32((uint32_t)s ^ ridgefill_mix32((uint32_t)(s >> 32)));
    return ridgefill_mix32(folded ^ (position * 0x9E3779B9U + 0x7F4A7C15U));
}

/* rho = clamp(N / D, 0, 1), 1 while D is not positive; a NaN ratio lands on 0
 * (kernels/ridgefill.h:86-91). */
RIDGEFILL_HD float ridgefill_rho(float n, float d) {
    if (!(d > 0.0f)) return 1.0f;
    const float r = n / d;
    if (!(r > 0.0f)) return 0.0f;
    return r < 1.0f ? r : 1.0f;
}

/* Two-sided softplus with the threshold above (kernels/ridgefill.h:94-97). */
RIDGEFILL_HD float ridgefill_softplus(float x) {
    if (x > RIDGEFILL_SOFTPLUS_THRESHOLD) return x;
    return x > 0.0f ? x + log1pf(expf(-x)) : log1pf(expf(x));
}

RIDGEFILL_HD float ridgefill_bf16_to_f32(uint16_t h) {
    const uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* ridgefill_mask's window (kernels/ridgefill.h:130-139): s, e from cu_last, b the bulk end, n the mask's
 * extent; w = {start, bulk end b', end}. False when cu_last is out of order; the window is then empty
 * inside the clamped [s, e] (the device fail-safe). */
RIDGEFILL_HD int ridgefill_mask_window(int64_t s, int64_t e, int64_t b, int64_t n, int64_t* w) {
    const int valid = s >= 0 && s <= e && e <= n;
    const int64_t end = e < 0 ? 0 : (e > n ? n : e);
    const int64_t start = s < 0 ? 0 : (s > end ? end : s);
    const int64_t bulk = b < start ? start : (b > end ? end : b);
    w[0] = start;
    w[1] = valid ? bulk : start;
    w[2] = end;
    return valid;
}

/* Where the 1s may start: row 0 in step mode with a non-empty window, else the window start
 * (kernels/ridgefill.h:46-48). */
RIDGEFILL_HD int64_t ridgefill_mask_from(int mode, const int64_t* w) {
    return mode == RIDGEFILL_MODE_STEP && w[1] > w[0] ? 0 : w[0];
}

/* ------------------------------------------------------------------ parsed operands
 * Plain scalars and pointers only: each is a kernel argument passed by value. */

typedef struct RidgeFillMask {
    const int32_t* cu_last;                       /* [2] {s, e}, device memory */
    const int32_t* tokens;   int64_t b;           /* [b] ids of rows [0, b) */
    const int32_t* positions; int64_t pos_stride;
    const float*   score;    int64_t vocab;       /* null in none / all mode when absent */
    int32_t*       mask;     int64_t n;
    int32_t*       bounds;                        /* [4] {s, b', b', e} */
    int32_t*       zeros;    int64_t n_zeros;
    double         share;
    long long      seed;
    int            mode;
} RidgeFillMask;

/* Row i's class score: -inf for an id outside the table or a non-finite score
 * (kernels/ridgefill.h:143-147). */
RIDGEFILL_HD float ridgefill_mask_score(const RidgeFillMask* g, int64_t i) {
    const int32_t id = g->tokens[i];
    const float s = id >= 0 && id < g->vocab ? g->score[id] : -INFINITY;
    return s > -INFINITY && s < INFINITY ? s : -INFINITY;
}

typedef struct RidgeFillRho {
    const void*    a;        int64_t a_pitch, a_col; int a_bf16;
    const int32_t* mask;
    const float*   a_log;
    const float*   dt_bias;
    float*         nd;       int64_t nd_slot, nd_head, nd_inner, n_states;
    const int32_t* state_idx;
    const int32_t* bounds;                        /* [>=1] or null */
    int64_t        n, n_head;
} RidgeFillRho;

/* First row of the recurrence: bounds[0] clamped into [0, n], 0 without bounds
 * (kernels/ridgefill.h:163-167). */
RIDGEFILL_HD int64_t ridgefill_rho_first_row(const RidgeFillRho* g) {
    if (!g->bounds) return 0;
    const int64_t s = g->bounds[0];
    return s < 0 ? 0 : (s > g->n ? g->n : s);
}

typedef struct RidgeFillCorrect {
    float*         state;    int64_t st_slot, st_head, st_row, st_col;
    float*         applied;  int64_t ap_slot, ap_head;
    const float*   c;        int64_t c_head, c_row;
    const float*   nd;       int64_t nd_slot, nd_head, nd_inner;
    const int32_t* st_idx;   const int32_t* ap_idx;  const int32_t* nd_idx;
    int64_t        st_pitch, ap_pitch, nd_pitch;
    int64_t        st_states, ap_states, nd_states;
    int64_t        n_seq, n_head, sd0, sd1;
    const int32_t* bounds;                        /* [>=2] or null */
    float          alpha;
    int            apply;                         /* 1 apply, 0 undo */
} RidgeFillCorrect;

/* False when the step's last sequence had no bulk row: the op then writes nothing
 * (kernels/ridgefill.h:188-190). */
RIDGEFILL_HD int ridgefill_correct_has_bulk(const RidgeFillCorrect* g) {
    return !g->bounds || g->bounds[1] > g->bounds[0];
}

/* Sequence s's slot in each pool; false when any is outside its pool (kernels/ridgefill.h:194-201). */
RIDGEFILL_HD int ridgefill_correct_slots(const RidgeFillCorrect* g, int64_t s, int64_t* st, int64_t* ap,
                                         int64_t* nd) {
    *st = g->st_idx[s * g->st_pitch];
    *ap = g->ap_idx[s * g->ap_pitch];
    *nd = g->nd ? g->nd_idx[s * g->nd_pitch] : 0;
    return *st >= 0 && *st < g->st_states && *ap >= 0 && *ap < g->ap_states &&
           (!g->nd || (*nd >= 0 && *nd < g->nd_states));
}

typedef struct RidgeFillStateRead {
    const float*   state;    int64_t st_slot, st_head, st_row, st_col, n_states;
    const int32_t* idx;      int64_t idx_pitch;
    float*         out;
    int64_t        n_seq, n_head, sd0, sd1;
} RidgeFillStateRead;

typedef struct RidgeFillHazard {
    const int32_t* cu_last;
    const int32_t* positions; int64_t pos_stride;
    const int32_t* bounds;
    int64_t        span;
    float*         meta;     int64_t meta_slot, meta_states;
    const int32_t* meta_idx;
    float*         count;
} RidgeFillHazard;

/* The branch hazard rule on the step's last sequence (the reference's rule, kernels/ridgefill.h:232-249).
 * The slot's record holds rec[0] = one past the last position an approximate pass covered and rec[1] = how
 * far hazards have been counted. The sequence's exact tail spans `span` positions, of which the q rows of
 * this pass are the last: the `span - q` before them, positions [first - (span - q), first), came from the
 * prefix cache. Those of them below rec[0] and not yet counted (at or above rec[1]) were approximated by
 * whoever wrote the cached state: they are added to the count once, and rec[1] moves past them. Then a pass
 * with bulk rows records its last bulk position + 1 in rec[0]. */
RIDGEFILL_HD void ridgefill_hazard_step(const RidgeFillHazard* g) {
    const int32_t slot = g->meta_idx[0];
    if (slot < 0 || slot >= g->meta_states) return;
    float* rec = g->meta + slot * g->meta_slot;
    const int64_t q = (int64_t)g->cu_last[1] - (int64_t)g->cu_last[0];
    const int64_t cached = g->span - q;
    if (g->span > 0 && q > 0 && cached > 0) {
        const int64_t first = g->positions[(int64_t)g->cu_last[0] * g->pos_stride];
        const int64_t covered = (int64_t)rec[0], counted = (int64_t)rec[1];
        const int64_t from = counted > first - cached ? counted : first - cached;   /* window start, past the counted */
        const int64_t to = covered < first ? covered : first;                       /* window end, within the covered */
        if (to > from) {
            g->count[0] += (float)(to - from);
            rec[1] = (float)to;
        }
    }
    if (g->bounds && g->bounds[0] < g->bounds[1]) {
        const int64_t last_bulk = (int64_t)g->bounds[1] - 1;
        rec[0] = (float)(g->positions[last_bulk * g->pos_stride] + 1);
    }
}

/* One ridgefill_select (source, destination) pair in bytes; `word` is 16, 4 or 1 (the widest unit every
 * address, pitch and width is a multiple of), 0 when the pair is absent (kernels/ridgefill.h:254-259). */
typedef struct RidgeFillCopy {
    const unsigned char* src;
    unsigned char*       dst;
    int64_t              src_pitch, dst_pitch, row_bytes;
    int                  word;
} RidgeFillCopy;

typedef struct RidgeFillSelect {
    const int32_t* mask;     int64_t n;
    RidgeFillCopy  pair[RIDGEFILL_SELECT_PAIRS];
} RidgeFillSelect;

typedef struct RidgeFillDrop {
    const int32_t* mask;     int64_t n;
    int32_t*       ids;      int64_t pitch, top_k;
} RidgeFillDrop;

/* ridgefill_gemm_nt_q / _bias: y[m, n] = sum over K blocks of a_scale[m, j] * b_scale[n, j] * (int32 dot of
 * the block), folded in f32 in block order, rounded once to bf16; with a bias, rounded again after
 * adding it (the gemm_nt_q + add pair of arch/ridgefill_layer.h:77-79, bit for bit). */
typedef struct RidgeFillGemmQ {
    const int8_t*  a;        int64_t lda;         /* [M, K] codes, row pitch lda (bytes) */
    const float*   a_scale;  int64_t ldas;        /* [M, K/group] f32 */
    const int8_t*  b;        int64_t ldb;         /* [N, K] codes (stored form == canonical) */
    const float*   b_scale;                       /* stored form: f32 [K/group, N] */
    const uint16_t* bias;                         /* [N] bf16 or null */
    uint16_t*      y;        int64_t ldy;         /* [M, N] bf16 */
    int32_t*       acc;                           /* optional [M, N, K/group] int32 block sums (debug) */
    const int32_t* rows;                          /* optional [M]: write row m only where rows[m] == 1 */
    int64_t        M, N, K, group;
    int64_t        max_ctas;                      /* at most this many CTAs (SMs), 0: the whole GPU */
} RidgeFillGemmQ;

/* ridgefill_quant_act_i8g: x bf16 [M, K] -> q i8 [M, K], s f32 [M, K/group]: per group of `group` columns,
 * s = absmax / 127 (1 for an all-zero group), q = round-half-even(x / s) clamped to [-127, 127]. */
typedef struct RidgeFillQuant {
    const uint16_t* x;       int64_t ldx;
    int8_t*        q;        int64_t ldq;
    float*         s;        int64_t lds;
    int64_t        M, K, group;
} RidgeFillQuant;

/* ridgefill_gdn_fill: the gated delta rule over each sequence of cu_seqlens, state [slot, Hv, V, K] f32
 * carried in place; per v-head h (k-head h / (Hv / Hk)) and row t:
 *   S <- exp(g[t, h]) * S;  S <- S + beta[t, h] * (v_t - S k_t) k_t^T;  o_t = scale * S q_t.
 * q, k [T, Hk, dk] bf16; v [T, Hv, dv] bf16; g (log decay) and beta f32 [T, Hv]; o [T, Hv, dv] bf16 or
 * absent (state-only fill). */
typedef struct RidgeFillGdn {
    const uint16_t* q;       int64_t q_row, q_head;
    const uint16_t* k;       int64_t k_row, k_head;
    const uint16_t* v;       int64_t v_row, v_head;
    const float*   g;        int64_t g_row;
    const float*   beta;     int64_t b_row;
    float*         state;    int64_t st_slot, st_head, n_states;
    const int32_t* state_idx; int64_t idx_pitch;
    const int32_t* cu;       int64_t n_seq;
    uint16_t*      o;        int64_t o_row, o_head;
    int64_t        T, n_head_k, n_head_v, dk, dv, chunk;
    float          scale;
} RidgeFillGdn;

/* ridgefill_gdn_conv_prep: the DeltaNet block's input preparation over each sequence [cu[i], cu[i+1]).
 * x bf16 [T, C] holds the projected q|k|v channels (C = 2 Hk dk + Hv dv, that order); per channel c and row t a
 * causal depthwise convolution of width 4 over the sequence's rows, the rows before its start taken from the
 * conv state (ctx_lens[i] > 0) or zero:
 *     u = bias[c] + w[c,0] x[t-3,c] + w[c,1] x[t-2,c] + w[c,2] x[t-1,c] + w[c,3] x[t,c]   (f32, in that order)
 *     y = u / (1 + exp(-u))                                                               (SiLU)
 * q and k heads are L2-normalised, y / sqrt(sum_head y^2 + 1e-6); q, k, v rounded to bf16. Per v-head h:
 *     g[t,h] = -exp(A_log[h]) * softplus(a[t,h] + dt_bias[h]),  beta[t,h] = 1 / (1 + exp(-b[t,h])).
 * The conv state [slots, 3, C] bf16 of each sequence's slot idx[i] is then the last three input rows of
 * (state, rows) (a slot outside the pool: zero history, nothing written). Rows outside every sequence are not
 * written. q is optional: without it the q columns are not computed (a state-only fill reads no q), and x's q
 * columns are read only in each sequence's last three rows, for the conv state. */
typedef struct RidgeFillConvPrep {
    const uint16_t* x;       int64_t x_row;
    const uint16_t* w;                          /* [C, 4] bf16, dense */
    const uint16_t* bias;                       /* [C] bf16 or null */
    const float*   a_log;    const float* dt_bias;
    uint16_t*      state;    int64_t st_slot, n_states;
    const int32_t* cu;       int64_t n_seq;
    const uint16_t* a;       int64_t a_row;
    const uint16_t* b;       int64_t b_row;
    const int32_t* idx;      int64_t idx_pitch;
    const int32_t* ctx;                         /* [n_seq] or null (every sequence starts fresh) */
    uint16_t*      q;        int64_t q_row, q_head;
    uint16_t*      k;        int64_t k_row, k_head;
    uint16_t*      v;        int64_t v_row, v_head;
    float*         g;        int64_t g_row;
    float*         beta;     int64_t beta_row;
    int64_t        T, n_head_k, n_head_v, dk, dv, width;
    int            columns;                     /* 0: gates and conv state only (the columns come from in_proj) */
} RidgeFillConvPrep;

/* ridgefill_gdn_in_proj: x = bf16(a_scale[t] b_scale[n] sum_k a[t,k] b[n,k]) over the k|v channels n of the
 * DeltaNet block's input (N = (Hk + Hv) 128: k heads first), then per channel the causal width-4 convolution over
 * each sequence (the rows before its start from the conv state when ctx > 0, else zero), SiLU, the L2 norm of each
 * k head (eps 1e-6), k and v rounded to bf16 -- conv_prep's arithmetic on the projection's rows, which never leave
 * the SM except each sequence's last three, written to `tail` (what the conv-state update reads). */
typedef struct RidgeFillInProj {
    RidgeFillGemmQ gemm;                        /* a, a_scale, b, b_scale; y = tail; group = K */
    const uint16_t* w;                          /* [N, 4] bf16 taps */
    const uint16_t* bias;                       /* [N] bf16 or null */
    const uint16_t* state;   int64_t st_slot, st_row, n_states;   /* history row t of slot s: state + s st_slot + t st_row */
    const int32_t* cu;       int64_t n_seq;
    const int32_t* idx;      int64_t idx_pitch;
    const int32_t* ctx;                         /* [n_seq] or null */
    uint16_t*      k;        int64_t k_row, k_head;
    uint16_t*      v;        int64_t v_row, v_head;
    int64_t        n_k;                         /* columns [0, n_k) are k channels (Hk 128) */
} RidgeFillInProj;

/* ridgefill_attn_kv_fill: the attention block's cache write for a prefill of T rows. Per row t and kv-head h
 * (D = head_dim = 256, R = rope_dim, lane l = elements 8l..8l+7):
 *   k_norm  ss = sum of k^2 (f32; each lane's 8 squares by fma in element order, then a butterfly over the 32
 *           lane sums), r = 1 / sqrt(ss / D + eps), kn[i] = bf16((k[i] r) w[i]);
 *   rope_k  for j < R/2: a = pos[p(j)][t] * theta^(-2j/R) (f64), c = f32(cos a), s = f32(sin a),
 *           kr[j] = bf16(fma(kn[j], c, -(kn[j+R/2] s))), kr[j+R/2] = bf16(fma(kn[j+R/2], c, kn[j] s));
 *           kr[i] = kn[i] for i >= R. p(j) is the position plane of rotary pair j: 0 for plain rope (or a
 *           one-plane positions operand); for mrope sections (s0, s1, s2) plane 0 on [0, s0), 1 on
 *           [s0, s0+s1), 2 after; for imrope plane 1 where j % 3 == 1 and j < 3 s1, 2 where j % 3 == 2 and
 *           j < 3 s2, 0 elsewhere;
 *   kv_store cache[0, slot, h] = kr, cache[1, slot, h] = v[t, h] for slot = slot_mapping[t] when
 *           0 <= slot < slots (other rows store nothing); k_out[t, h] = kr when k_out is present. */
enum { RIDGEFILL_ROPE_NEOX = 0, RIDGEFILL_ROPE_MROPE = 1, RIDGEFILL_ROPE_IMROPE = 2 };
typedef struct RidgeFillAttnKv {
    const uint16_t* k;       int64_t k_row, k_head;        /* [T, Hkv, D] */
    const uint16_t* v;       int64_t v_row, v_head;        /* [T, Hkv, D] */
    const void*    w;        int w_f32;                    /* [D] bf16 (w_f32 0) or f32 */
    const int32_t* pos;      int64_t pos_plane; int n_planes;   /* [T] or [3, T] */
    const int32_t* slots;                                  /* [T] */
    uint16_t*      cache;    int64_t c_kv, c_slot, c_head, n_slots;   /* [2, slots, Hkv, D] */
    uint16_t*      k_out;    int64_t ko_row, ko_head;      /* [T, Hkv, D] or null */
    int64_t        T, n_head_kv, head_dim, rope_dim;
    double         theta;
    float          eps;
    int            mode;
    int            sections[3];
} RidgeFillAttnKv;

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ entry points
 * Parses shared by every row of an op: RAD_OK or a named refusal (kernels/ridgefill.h:278-285). */
int ridgefill_mask_parse(const RadArgs* a, RidgeFillMask* out);
int ridgefill_rho_parse(const RadArgs* a, RidgeFillRho* out);
int ridgefill_correct_parse(const RadArgs* a, RidgeFillCorrect* out);
int ridgefill_state_read_parse(const RadArgs* a, RidgeFillStateRead* out);
int ridgefill_select_parse(const RadArgs* a, RidgeFillSelect* out);
int ridgefill_drop_parse(const RadArgs* a, RidgeFillDrop* out);
int ridgefill_hazard_parse(const RadArgs* a, RidgeFillHazard* out);
int ridgefill_gemm_q_parse(const RadArgs* a, int with_bias, RidgeFillGemmQ* out);

/* ridgefill_gemm_nt_bias, the bf16 projector and the final map (schema kernels/rows.cpp:67-70,155-160; issue
 * arch/ridgefill_declare.h:236-240, arch/ridgefill_final.h:40-44): y = res + act(a @ b^T + bias), rounded to
 * bf16 after the biased product (accumulated in f32, the bias added in f32), after the activation and after
 * the residual. a bf16 [M, K], b bf16 [N, K], bias bf16 or f32 [N], res bf16 [M, N] optional, y bf16 [M, N];
 * dtype "bf16"; act absent / "none" or "silu" (x * sigmoid(x)); K a multiple of 64; rows 16-byte aligned. */
enum { RIDGEFILL_ACT_NONE = 0, RIDGEFILL_ACT_SILU = 1 };
typedef struct RidgeFillGemmBias {
    const uint16_t* a;       int64_t lda;         /* [M, K] */
    const uint16_t* b;       int64_t ldb;         /* [N, K] */
    const void*    bias;     int bias_f32;        /* [N] bf16 (bias_f32 0) or f32 */
    const uint16_t* res;     int64_t ldr;         /* [M, N] or null */
    uint16_t*      y;        int64_t ldy;         /* [M, N] */
    int64_t        M, N, K;
    int            act;
} RidgeFillGemmBias;
int ridgefill_gemm_bias_parse(const RadArgs* a, RidgeFillGemmBias* out);
int ridgefill_quant_parse(const RadArgs* a, RidgeFillQuant* out);
int ridgefill_gdn_parse(const RadArgs* a, RidgeFillGdn* out);
int ridgefill_conv_prep_parse(const RadArgs* a, RidgeFillConvPrep* out);
int ridgefill_in_proj_parse(const RadArgs* a, RidgeFillInProj* out);
int ridgefill_attn_kv_parse(const RadArgs* a, RidgeFillAttnKv* out);

/* The device rows (kernels/ridgefill.h:304-310 and the new ops): async launches on `s` (a
 * cudaStream_t); no allocation, no synchronisation. */
int ridgefill_mask_device(const RadArgs* a, RadStream s);
int ridgefill_rho_device(const RadArgs* a, RadStream s);
int ridgefill_correct_device(const RadArgs* a, RadStream s);
int ridgefill_state_read_device(const RadArgs* a, RadStream s);
int ridgefill_select_device(const RadArgs* a, RadStream s);
int ridgefill_drop_device(const RadArgs* a, RadStream s);
int ridgefill_hazard_device(const RadArgs* a, RadStream s);
int ridgefill_gemm_nt_q_device(const RadArgs* a, RadStream s);
int ridgefill_gemm_nt_q_bias_device(const RadArgs* a, RadStream s);
int ridgefill_gemm_nt_bias_device(const RadArgs* a, RadStream s);
int ridgefill_quant_act_device(const RadArgs* a, RadStream s);
int ridgefill_gdn_fill_device(const RadArgs* a, RadStream s);
int ridgefill_gdn_conv_prep_device(const RadArgs* a, RadStream s);
int ridgefill_gdn_in_proj_device(const RadArgs* a, RadStream s);
int ridgefill_attn_kv_fill_device(const RadArgs* a, RadStream s);

/* The first error code a tensor-core kernel of this library recorded after giving up on a bounded
 * wait (0: none), optionally cleared. Synchronises the current device: a diagnostic, never called on
 * a launch path. -1 when the device could not be read. */
int ridgefill_device_error(int reset);

/* Failure-detection self-test (no counterpart in the reference): launches, on stream `s`, one kernel that runs
 * the two waits the library's kernels block on against a barrier phase and a flag that nothing completes: an
 * mbarrier wait (every tensor-core hand-over) and the DeltaNet chain's wait for a slot flag (`*flag`, device
 * memory, must be 0 and stay 0). Each gives up after its limit (2 s), records its code for
 * ridgefill_device_error and writes 0 into status[0] / status[1] (device memory; 1 would mean it completed).
 * The kernel then returns: no trap, no fault, the context stays usable. RAD_E_INVAL on null pointers. */
int ridgefill_wait_selftest(int* flag, int* status, RadStream s);

/* ridgefill_gdn_fill without a workspace operand (no counterpart in the reference): for callers that
 * cannot allocate device memory where they launch the fill -- an FFI host with no device allocator of
 * its own, or an engine step whose memory is fixed before the pass and which may not cudaMalloc inside
 * it. Same operands as the row; RadArgs::scratch is ignored and a 64 MiB workspace compiled into the
 * library is used instead (held on every GPU that loads the library until exit). RAD_E_SHAPE when the
 * call needs more than 64 MiB: a one-sequence 2,048-row call fits at up to 40 value heads for the state
 * alone, at up to 19 with the output o. The first call on a device resolves the workspace's address there
 * (again after the device's context changes, e.g. after cudaDeviceReset): make it before any stream
 * capture. Calls share the workspace: calls that overlap on the GPU race. Allocates and frees nothing. A state-only
 * call of at least 64 chains (value heads x sequences) takes the per-head form, which uses no workspace. */
int ridgefill_gdn_fill_noalloc(const RadArgs* a, RadStream s);

/* ridgefill_gdn_fill's scratch hook: device bytes the row needs in RadArgs::scratch. */
int64_t ridgefill_gdn_fill_scratch(const RadArgs* a);

/* ridgefill_gemm_nt_q's stored-form hooks for operand 2 (codes) and 3 (scale) of encoding
 * i8*bf16[1x128] (the hooks arch/ridgefill_int8.h:87-130 calls). */
int ridgefill_gemm_q_layout(const RadParam* p, int n_p, int operand, const RadEncoding* enc, const int* sel,
                            const RadTensor* geom, int n_geom, RadLayout* out);
int ridgefill_gemm_q_relayout(const RadParam* p, int n_p, int operand, const RadEncoding* enc, const int* sel,
                              const RadTensor* src, int n_src, void* dst, int64_t dst_bytes);
int ridgefill_gemm_q_unrelayout(const RadParam* p, int n_p, int operand, const RadEncoding* enc, const int* sel,
                                const RadTensor* src, int n_src, void* dst, int64_t dst_bytes);

#ifdef __cplusplus
}
#endif

#endif /* RIDGEFILL_B200_H */
