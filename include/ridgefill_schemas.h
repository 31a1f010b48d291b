/* ridgefill_schemas.h -- the op schemas and cold-call operand descriptions of the RidgeFill kernel
 * library (C++ only).
 *
 * The first nine schemas are the reference plugin's (kernels/rows.cpp:44-168): same op names, the same
 * parameters and the same operand order, so an issue site written for the reference
 * (arch/ridgefill_layer.h, arch/qwen4exp_blocks.h) binds unchanged. The remaining schemas are the ops
 * this library adds: the fused-bias int8 projector, the activation quantiser and the chunked Gated
 * DeltaNet fill. The descriptions (opd_shape) give a tool the operands to call a row cold, as the
 * reference's do (kernels/rows.cpp:170-301).
 */
#ifndef RIDGEFILL_SCHEMAS_H
#define RIDGEFILL_SCHEMAS_H

#include "rad_plugin.h"

#include <cstring>
#include <initializer_list>

namespace ridgefill_schema {

#define RF_P_INT(k) { (k), RAD_P_INT, RAD_REQUIRED, RAD_PROLE_NONE }
#define RF_P_STR(k) { (k), RAD_P_STR, RAD_REQUIRED, RAD_PROLE_NONE }
#define RF_P_F64(k) { (k), RAD_P_F64, RAD_REQUIRED, RAD_PROLE_NONE }
#define RF_P_OPT(k, t) { (k), (t), RAD_OPTIONAL, RAD_PROLE_NONE }
#define RF_IN(n) { (n), RAD_OPD_IN, 0 }
#define RF_IN_OPT(n) { (n), RAD_OPD_IN, 1 }
#define RF_OUT(n) { (n), RAD_OPD_OUT, 0 }
#define RF_OUT_OPT(n) { (n), RAD_OPD_OUT, 1 }
#define RF_INOUT(n) { (n), RAD_OPD_INOUT, 0 }
#define RF_INOUT_OPT(n) { (n), RAD_OPD_INOUT, 1 }
#define RF_WGT(n) { (n), RAD_OPD_WEIGHT, 0 }
#define RF_ARR(a) (a), (int)(sizeof(a) / sizeof((a)[0]))

static const RadParamSpec pMask[] = { RF_P_INT("M"), RF_P_F64("share"), RF_P_INT("seed"), RF_P_STR("mode") };
static const RadOperandSpec oMask[] = { RF_IN("cu_last"), RF_IN("token_ids"), RF_IN("positions"), RF_IN_OPT("score"),
                                        RF_OUT("mask"), RF_OUT("bounds"), RF_OUT_OPT("zeros") };
static const RadParamSpec pSelect[] = { RF_P_INT("M") };
static const RadOperandSpec oSelect[] = { RF_IN("mask"), RF_IN("x_src"), RF_IN_OPT("q_src"), RF_IN_OPT("s_src"),
                                          RF_INOUT("x"), RF_INOUT_OPT("q"), RF_INOUT_OPT("s") };
static const RadParamSpec pDrop[] = { RF_P_INT("M"), RF_P_INT("top_k") };
static const RadOperandSpec oDrop[] = { RF_IN("mask"), RF_INOUT("ids") };
static const RadParamSpec pRho[] = { RF_P_INT("M"), RF_P_INT("n_head") };
static const RadOperandSpec oRho[] = { RF_IN("a"), RF_IN("mask"), RF_WGT("A_log"), RF_WGT("dt_bias"),
                                       RF_INOUT("ND"), RF_IN("state_idx"), RF_IN_OPT("bounds") };
static const RadParamSpec pCorrect[] = { RF_P_INT("M"), RF_P_STR("mode"), RF_P_F64("alpha"), RF_P_INT("n_head"),
                                         RF_P_INT("sd0"), RF_P_INT("sd1") };
static const RadOperandSpec oCorrect[] = { RF_INOUT("state"), RF_IN("state_idx"), RF_INOUT("applied"),
                                           RF_IN("applied_idx"), RF_IN("C"), RF_IN_OPT("ND"), RF_IN_OPT("nd_idx"),
                                           RF_IN_OPT("bounds") };
static const RadParamSpec pStateRead[] = { RF_P_INT("M"), RF_P_INT("n_head"), RF_P_INT("sd0"), RF_P_INT("sd1") };
static const RadOperandSpec oStateRead[] = { RF_IN("state"), RF_IN("state_idx"), RF_OUT("out") };
static const RadParamSpec pHazard[] = { RF_P_INT("M") };
static const RadOperandSpec oHazard[] = { RF_IN("cu_last"), RF_IN("positions"), RF_IN_OPT("bounds"),
                                          RF_IN_OPT("span"), RF_INOUT("meta"), RF_IN("meta_idx"), RF_INOUT("count") };
static const RadParamSpec pGemm[] = { RF_P_INT("M"), RF_P_INT("N"), RF_P_INT("K"), RF_P_STR("dtype"),
                                      RF_P_OPT("act", RAD_P_STR) };
static const RadOperandSpec oGemm[] = { RF_IN("a"), RF_IN("b"), RF_IN("bias"), RF_IN_OPT("res"), RF_OUT("y") };
static const RadParamSpec pGemmQ[] = { RF_P_INT("M"), RF_P_INT("N"), RF_P_INT("K"), RF_P_INT("group"),
                                       RF_P_STR("dtype") };
static const RadOperandSpec oGemmQ[] = { RF_IN("a"), RF_IN_OPT("a_scale"), RF_IN("b"), RF_IN("b_scale"), RF_OUT("y"),
                                         RF_IN_OPT("a_sum"), RF_IN_OPT("b_ref") };
/* new ops */
static const RadParamSpec pGemmQBias[] = { RF_P_INT("M"), RF_P_INT("N"), RF_P_INT("K"), RF_P_INT("group"),
                                           RF_P_STR("dtype"), RF_P_OPT("max_ctas", RAD_P_INT) };
static const RadOperandSpec oGemmQBias[] = { RF_IN("a"), RF_IN("a_scale"), RF_IN("b"), RF_IN("b_scale"),
                                             RF_IN_OPT("bias"), RF_OUT("y"), RF_OUT_OPT("acc"), RF_IN_OPT("rows") };
static const RadParamSpec pQuant[] = { RF_P_INT("M"), RF_P_INT("n"), RF_P_INT("group"), RF_P_STR("dtype") };
static const RadOperandSpec oQuant[] = { RF_IN("x"), RF_OUT("q"), RF_OUT("s") };
static const RadParamSpec pGdn[] = { RF_P_INT("M"), RF_P_INT("n_head_k"), RF_P_INT("n_head_v"), RF_P_INT("head_k"),
                                     RF_P_INT("head_v"), RF_P_INT("chunk"), RF_P_OPT("scale", RAD_P_F64) };
static const RadOperandSpec oGdn[] = { RF_IN_OPT("q"), RF_IN("k"), RF_IN("v"), RF_IN("g"), RF_IN("beta"),
                                       RF_INOUT("state"), RF_IN("state_idx"), RF_IN("cu_seqlens"), RF_OUT_OPT("o") };
static const RadParamSpec pConv[] = { RF_P_INT("M"), RF_P_INT("n_head_k"), RF_P_INT("n_head_v"), RF_P_INT("head_k"),
                                      RF_P_INT("head_v"), RF_P_INT("conv"), RF_P_OPT("columns", RAD_P_INT) };
static const RadOperandSpec oConv[] = { RF_IN("x"), RF_IN("w_conv"), RF_IN_OPT("conv_bias"), RF_IN("A_log"),
                                        RF_IN("dt_bias"), RF_INOUT("conv_state"), RF_IN("cu_seqlens"), RF_IN("a"),
                                        RF_IN("b"), RF_IN("conv_idx"), RF_IN_OPT("ctx_lens"), RF_OUT_OPT("q"), RF_OUT("k"),
                                        RF_OUT("v"), RF_OUT("g"), RF_OUT("beta") };
static const RadParamSpec pInProj[] = { RF_P_INT("M"), RF_P_INT("N"), RF_P_INT("K"), RF_P_INT("n_head_k"),
                                        RF_P_INT("n_head_v"), RF_P_INT("group"), RF_P_STR("dtype") };
static const RadOperandSpec oInProj[] = { RF_IN("a"), RF_IN("a_scale"), RF_IN("b"), RF_IN("b_scale"), RF_IN("w_conv"),
                                          RF_IN_OPT("conv_bias"), RF_IN("conv_state"), RF_IN("cu_seqlens"),
                                          RF_IN("conv_idx"), RF_IN_OPT("ctx_lens"), RF_OUT("k"), RF_OUT("v"),
                                          RF_OUT("tail") };
static const RadParamSpec pAttnKv[] = { RF_P_INT("M"), RF_P_INT("n_head_kv"), RF_P_INT("head_dim"), RF_P_INT("rope_dim"),
                                        RF_P_F64("rope_theta"), RF_P_OPT("eps", RAD_P_F64),
                                        RF_P_OPT("rope_mode", RAD_P_STR), RF_P_OPT("rope_sections", RAD_P_STR) };
static const RadOperandSpec oAttnKv[] = { RF_IN("k"), RF_IN("v"), RF_IN("k_norm"), RF_IN("positions"),
                                          RF_IN("slot_mapping"), RF_INOUT("kv_cache"), RF_OUT_OPT("k_out") };

/* The reference's nine schemas come first, in its order (kernels/rows.cpp:84-168). */
enum { kReferenceSchemas = 9 };

static const RadOpSchema kSchemas[] = {
{ "ridgefill_mask", RF_ARR(pMask), RF_ARR(oMask),
  "Which rows of the step's last sequence stay exact. cu_last [2] = {s, e} (read on the device); b = token_ids' "
  "extent; b' = min(max(b, s), e); window W = [s, b'). mask [n] is written on every row, 0 outside W. Inside W: "
  "none 1, all 0, step 1 on [0, b') when W is not empty; class: a row matches when score[token_ids[i]] is finite, "
  "k = rint(share * matches) half to even, a matching row is kept (0) when fewer than k matching rows rank before "
  "it by (score descending, row ascending); random: the same k over all rows of W ranked by "
  "row_hash(seed, positions[i]) ascending, ties by row. bounds [4] = {s, b', b', e}. Optional zeros written 0. "
  "Host row refuses s < 0, s > e, e > n; the device row takes the window empty instead." },
{ "ridgefill_select", RF_ARR(pSelect), RF_ARR(oSelect),
  "For every row i < n (mask's extent) with mask[i] == 1, row i of each present destination (x, q, s) is "
  "overwritten by its source row, byte for byte; nothing else is written. Pairs present or absent together; "
  "rank 2, last stride 1, one dtype of whole bytes and one row width per pair." },
{ "ridgefill_drop_rows", RF_ARR(pDrop), RF_ARR(oDrop),
  "For every row i < n with mask[i] == 1, ids[i, 0 .. top_k) = -1; nothing else is written." },
{ "ridgefill_rho_update", RF_ARR(pRho), RF_ARR(oRho),
  "Per head h over rows t of a [n, n_head] (own strides): e = exp(-exp(A_log[h]) * softplus(a[t,h] + dt_bias[h])); "
  "D = e*D + 1; N = e*N + mask[t]; (N, D) carried in the ND slot state_idx[0] (outside the pool: nothing). "
  "Optional bounds: rows [clamp(bounds[0], 0, n), n) only." },
{ "ridgefill_state_correct", RF_ARR(pCorrect), RF_ARR(oCorrect),
  "Per (sequence, head), each pool through its own slot index (a sequence with any slot outside its pool is "
  "skipped): undo: state -= applied * C, applied = 0; apply: s = alpha * (ND ? clamp(N/D, 0, 1) : 1), "
  "state += s * C, applied = s; nothing added when the scale is 0. Optional bounds: bounds[1] <= bounds[0] "
  "writes nothing." },
{ "ridgefill_state_read", RF_ARR(pStateRead), RF_ARR(oStateRead),
  "out[s, h, i, j] = state[slot_s, h, i, j], densely from out's first element; a slot outside the pool reads "
  "zeros." },
{ "ridgefill_hazard", RF_ARR(pHazard), RF_ARR(oHazard),
  "Prefix-cache branch hazard count on the step's last sequence (the rule of ridgefill_hazard_step); the host "
  "row refuses s < 0 or s > e, the device row counts nothing instead." },
{ "ridgefill_gemm_nt_bias", RF_ARR(pGemm), RF_ARR(oGemm),
  "y = res + act(a @ b^T + bias) in bf16 with the weight b [N, K] and bias [N] as IN operands." },
{ "ridgefill_gemm_nt_q", RF_ARR(pGemmQ), RF_ARR(oGemmQ),
  "y[m, n] = sum_j a_scale[m, j] * b_scale[n, j] * sum_{k in block j} a[m, k] * b[n, k], bf16; int32 within "
  "each `group`-column block, f32 fold in block order, one rounding. a i8 [M, K], a_scale f32 [M, K/group]; "
  "b and b_scale in the stored form this row's layout hook describes (codes [N, K] i8, scale f32 [K/group, N])." },
{ "ridgefill_gemm_nt_q_bias", RF_ARR(pGemmQBias), RF_ARR(oGemmQBias),
  "ridgefill_gemm_nt_q followed by the row-broadcast bias add, in one pass: y = bf16(bf16(gemm) + bias), "
  "equal bit for bit to the two ops in sequence. Optional acc i32 [M, N, K/group]: every block's int32 sum. "
  "Optional max_ctas: use at most that many SMs (a caller running another stream's kernels beside it). "
  "Optional rows i32 [M] (ridgefill_select's mask): only rows m with rows[m] == 1 are written, the others keep "
  "y's contents -- the projector and ridgefill_select(rows, y_full -> y) in one pass, bit for bit." },
{ "ridgefill_quant_act_i8g", RF_ARR(pQuant), RF_ARR(oQuant),
  "Activation codes for the int8 projector: per `group` columns of each row of x bf16 [M, n], "
  "s = absmax / 127 (1 for an all-zero group) in f32, q = round-half-even(x / s) clamped to +-127." },
{ "ridgefill_gdn_fill", RF_ARR(pGdn), RF_ARR(oGdn),
  "Gated DeltaNet chunk fill over each sequence [cu[i], cu[i+1]) with its state slot state_idx[i] (outside the "
  "pool: skipped), state f32 [slots, Hv, dv, dk] updated in place; per row t and v-head h (k-head "
  "h / (Hv/Hk)): S = exp(g[t,h]) S; S += beta[t,h] (v_t - S k_t) k_t^T; o_t = scale * S q_t (o and q optional "
  "together: absent = state-only fill). Chunked (WY form) on the device, `chunk` rows a tile." },
{ "ridgefill_gdn_conv_prep", RF_ARR(pConv), RF_ARR(oConv),
  "The DeltaNet block's input preparation over each sequence [cu[i], cu[i+1]): x bf16 [T, C] = q|k|v channels "
  "(C = 2 Hk dk + Hv dv); per channel a causal depthwise convolution of width `conv` (4) over the sequence's rows, "
  "u = bias + sum_j w[c, j] x[t - 3 + j] in f32 in j order, the rows before the start from conv_state[conv_idx[i]] "
  "(ctx_lens[i] > 0) or zero; y = u / (1 + exp(-u)); q and k heads divided by sqrt(sum y^2 + 1e-6); q, k, v bf16. "
  "g[t, h] = -exp(A_log[h]) softplus(a[t, h] + dt_bias[h]) (threshold 20), beta = sigmoid(b); f32. conv_state "
  "bf16 [slots, 3, C] then holds each sequence's last three input rows (a slot outside the pool: zero history, "
  "not written). Rows outside every sequence are not written. Optional columns = 0: only g, beta and the conv "
  "state are written (k and v come from ridgefill_gdn_in_proj, which has read the old conv state)." },
{ "ridgefill_gdn_in_proj", RF_ARR(pInProj), RF_ARR(oInProj),
  "The DeltaNet block's int8 in-projection of its k|v channels with conv_prep's per-channel arithmetic in the "
  "same pass: x[t, n] = bf16(a_scale[t] b_scale[n] sum_k a[t, k] b[n, k]) (group = K: int32 over all of K, one "
  "f32 product, one rounding) for the N = (Hk + Hv) 128 channels (k heads first); then per sequence [cu[i], "
  "cu[i+1]) ridgefill_gdn_conv_prep's convolution, SiLU and k-head L2 norm on those channels, bit for bit, into "
  "k bf16 [T, Hk, 128] and v bf16 [T, Hv, 128]; x itself is written only on each sequence's last three rows, "
  "into tail bf16 [T, N] (what the conv-state update reads). conv_state bf16 [slots, 3, N] is read, not written: "
  "run ridgefill_gdn_conv_prep with columns = 0 afterwards for the gates and the state update." },
{ "ridgefill_attn_kv_fill", RF_ARR(pAttnKv), RF_ARR(oAttnKv),
  "The attention block's K/V cache write for T prefill rows (k_norm, rope_k, kv_store as one op): per row t and "
  "kv-head h, kn = bf16(k * w / sqrt(mean(k^2) + eps)) (f32), the first rope_dim elements rotated in half pairs "
  "(j, j + rope_dim/2) by the angle pos[plane(j)][t] * rope_theta^(-2j/rope_dim) (f64 angle, f32 cos/sin, bf16 "
  "result; plane(j) by rope_mode neox / mrope / imrope and rope_sections), then kv_cache[0, slot, h] = that k "
  "and kv_cache[1, slot, h] = v[t, h] for slot = slot_mapping[t] inside [0, slots) (else nothing is stored); "
  "k_out[t, h] = that k when present. head_dim 256." },
};

/* ------------------------------------------------------------------ cold-call descriptions */

inline RadOpdDesc opd(uint32_t dtype, std::initializer_list<int64_t> dims, uint32_t fill = RAD_FILL_NORMAL) {
    RadOpdDesc d{};
    d.dtype = dtype;
    d.fill = fill;
    d.idx_const = -1;
    for (int64_t e : dims) d.shape[d.rank++] = e;
    return d;
}

inline RadOpdDesc opd_idx(std::initializer_list<int64_t> dims, int64_t idx_max, uint32_t flags = 0) {
    RadOpdDesc d = opd(RAD_I32, dims, RAD_FILL_INDEX);
    d.idx_max = idx_max;
    d.flags = flags;
    return d;
}

inline RadOpdDesc opd_absent() {
    RadOpdDesc d{};
    d.idx_const = -1;
    d.flags = RAD_OPD_F_ABSENT;
    return d;
}

/* A non-positive extent anywhere means the geometry lacks a parameter: RAD_E_UNSUPPORTED; an operand
 * index past the list is RAD_E_SHAPE. */
inline int pick(RadOpdDesc* out, int operand, std::initializer_list<RadOpdDesc> list) {
    for (const RadOpdDesc& d : list) {
        if (d.flags & RAD_OPD_F_ABSENT) continue;
        for (uint32_t i = 0; i < d.rank; ++i)
            if (d.shape[i] <= 0) return RAD_E_UNSUPPORTED;
    }
    if (!out || operand < 0 || operand >= (int)list.size()) return RAD_E_SHAPE;
    *out = list.begin()[operand];
    return RAD_OK;
}

inline int64_t dim(const RadParam* p, int n_p, const char* key) { return rad_param_getdim(p, n_p, key, 0); }

inline int shape_mask(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t n = dim(p, n_p, "M"), vocab = 4 * n;
    return pick(out, operand, { opd_idx({ 2 }, n, RAD_OPD_F_IDX_CU), opd_idx({ n }, vocab),
                                opd_idx({ n }, 64 * n, RAD_OPD_F_IDX_UNIQUE), opd(RAD_F32, { vocab }),
                                opd_idx({ n }, 2), opd_idx({ 4 }, n), opd_idx({ 8 }, 4) });
}

inline int shape_select(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t n = dim(p, n_p, "M");
    const RadOpdDesc x = opd(RAD_BF16, { n, 64 }), q = opd(RAD_I8, { n, 66 }), s = opd(RAD_F32, { n, 2 });
    return pick(out, operand, { opd_idx({ n }, 2), x, q, s, x, q, s });
}

inline int shape_drop(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t n = dim(p, n_p, "M"), top_k = rad_param_getdim(p, n_p, "top_k", -1);
    return pick(out, operand, { opd_idx({ n }, 2), opd_idx({ n, top_k >= 0 ? top_k + 3 : 0 }, 4 * n) });
}

inline int shape_rho(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t n = dim(p, n_p, "M"), heads = dim(p, n_p, "n_head"), slots = 4;
    return pick(out, operand, { opd(RAD_BF16, { n, heads }), opd_idx({ n }, 2), opd(RAD_F32, { heads }),
                                opd(RAD_F32, { heads }), opd(RAD_F32, { slots, heads, 1, 2 }, RAD_FILL_SIGMOID),
                                opd_idx({ 1, 1 }, slots), opd_idx({ 4 }, n) });
}

inline int shape_correct(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t n_seq = dim(p, n_p, "M"), heads = dim(p, n_p, "n_head");
    const int64_t sd0 = dim(p, n_p, "sd0"), sd1 = dim(p, n_p, "sd1"), slots = n_seq + 2;
    const bool apply = std::strcmp(rad_param_gets(p, n_p, "mode", ""), "apply") == 0;
    const RadOpdDesc index = opd_idx({ n_seq, 1 }, slots, RAD_OPD_F_IDX_UNIQUE);
    return pick(out, operand, { opd(RAD_F32, { slots, heads, sd0, sd1 }), index, opd(RAD_F32, { slots, heads, 1, 1 }),
                                index, opd(RAD_F32, { heads, sd0, sd1 }),
                                apply ? opd(RAD_F32, { slots, heads, 1, 2 }, RAD_FILL_SIGMOID) : opd_absent(),
                                apply ? index : opd_absent(), opd_absent() });
}

inline int shape_state_read(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t n_seq = dim(p, n_p, "M"), heads = dim(p, n_p, "n_head");
    const int64_t sd0 = dim(p, n_p, "sd0"), sd1 = dim(p, n_p, "sd1"), slots = n_seq + 2;
    return pick(out, operand, { opd(RAD_F32, { slots, heads, sd0, sd1 }), opd_idx({ n_seq, 1 }, slots),
                                opd(RAD_F32, { n_seq, heads, sd0, sd1 }) });
}

inline int shape_hazard(const RadParam*, int, int operand, RadOpdDesc* out) {
    return pick(out, operand, { opd_idx({ 2 }, 64, RAD_OPD_F_IDX_CU), opd_idx({ 64 }, 1 << 20, RAD_OPD_F_IDX_UNIQUE),
                                opd_idx({ 4 }, 64), opd_idx({ 32 }, 4), opd(RAD_F32, { 8, 1, 1, 2 }, RAD_FILL_SIGMOID),
                                opd_idx({ 1, 1 }, 8), opd(RAD_F32, { 1 }, RAD_FILL_SIGMOID) });
}

inline int shape_gemm_q(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t M = dim(p, n_p, "M"), N = dim(p, n_p, "N"), K = dim(p, n_p, "K"), g = dim(p, n_p, "group");
    const int64_t blocks = g > 0 && K % g == 0 ? K / g : 0;
    return pick(out, operand, { opd(RAD_I8, { M, K }), opd(RAD_F32, { M, blocks }, RAD_FILL_SIGMOID),
                                opd(RAD_I8, { N, K }), opd(RAD_F32, { blocks, N }, RAD_FILL_SIGMOID),
                                opd(RAD_BF16, { M, N }), opd_absent(), opd_absent() });
}

inline int shape_gemm_q_bias(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t M = dim(p, n_p, "M"), N = dim(p, n_p, "N"), K = dim(p, n_p, "K"), g = dim(p, n_p, "group");
    const int64_t blocks = g > 0 && K % g == 0 ? K / g : 0;
    return pick(out, operand, { opd(RAD_I8, { M, K }), opd(RAD_F32, { M, blocks }, RAD_FILL_SIGMOID),
                                opd(RAD_I8, { N, K }), opd(RAD_F32, { blocks, N }, RAD_FILL_SIGMOID),
                                opd(RAD_BF16, { N }), opd(RAD_BF16, { M, N }), opd_absent(), opd_absent() });
}

inline int shape_gemm_bias(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t M = dim(p, n_p, "M"), N = dim(p, n_p, "N"), K = dim(p, n_p, "K");
    return pick(out, operand, { opd(RAD_BF16, { M, K }), opd(RAD_BF16, { N, K }), opd(RAD_BF16, { N }),
                                opd(RAD_BF16, { M, N }), opd(RAD_BF16, { M, N }) });
}

inline int shape_quant(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t M = dim(p, n_p, "M"), n = dim(p, n_p, "n"), g = dim(p, n_p, "group");
    const int64_t groups = g > 0 && n % g == 0 ? n / g : 0;
    return pick(out, operand, { opd(RAD_BF16, { M, n }), opd(RAD_I8, { M, n }), opd(RAD_F32, { M, groups }) });
}

inline int shape_gdn(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t T = dim(p, n_p, "M"), hk = dim(p, n_p, "n_head_k"), hv = dim(p, n_p, "n_head_v");
    const int64_t dk = dim(p, n_p, "head_k"), dv = dim(p, n_p, "head_v"), slots = 3;
    return pick(out, operand, { opd(RAD_BF16, { T, hk, dk }), opd(RAD_BF16, { T, hk, dk }), opd(RAD_BF16, { T, hv, dv }),
                                opd(RAD_F32, { T, hv }, RAD_FILL_SIGMOID), opd(RAD_F32, { T, hv }, RAD_FILL_SIGMOID),
                                opd(RAD_F32, { slots, hv, dv, dk }), opd_idx({ 1, 1 }, slots),
                                opd_idx({ 2 }, T, RAD_OPD_F_IDX_CU), opd(RAD_BF16, { T, hv, dv }) });
}

inline int shape_conv_prep(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t T = dim(p, n_p, "M"), hk = dim(p, n_p, "n_head_k"), hv = dim(p, n_p, "n_head_v");
    const int64_t dk = dim(p, n_p, "head_k"), dv = dim(p, n_p, "head_v"), C = 2 * hk * dk + hv * dv, slots = 3;
    return pick(out, operand, { opd(RAD_BF16, { T, C }), opd(RAD_BF16, { C, 4 }), opd(RAD_BF16, { C }), opd(RAD_F32, { hv }),
                                opd(RAD_F32, { hv }), opd(RAD_BF16, { slots, 3, C }), opd_idx({ 2 }, T, RAD_OPD_F_IDX_CU),
                                opd(RAD_BF16, { T, hv }), opd(RAD_BF16, { T, hv }), opd_idx({ 1 }, slots),
                                opd(RAD_I32, { 1 }), opd(RAD_BF16, { T, hk, dk }), opd(RAD_BF16, { T, hk, dk }),
                                opd(RAD_BF16, { T, hv, dv }), opd(RAD_F32, { T, hv }), opd(RAD_F32, { T, hv }) });
}

inline int shape_in_proj(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t T = dim(p, n_p, "M"), K = dim(p, n_p, "K"), hk = dim(p, n_p, "n_head_k"), hv = dim(p, n_p, "n_head_v");
    const int64_t N = (hk + hv) * 128, slots = 3;
    return pick(out, operand, { opd(RAD_I8, { T, K }), opd(RAD_F32, { T, 1 }, RAD_FILL_SIGMOID), opd(RAD_I8, { N, K }),
                                opd(RAD_F32, { 1, N }, RAD_FILL_SIGMOID), opd(RAD_BF16, { N, 4 }), opd(RAD_BF16, { N }),
                                opd(RAD_BF16, { slots, 3, N }), opd_idx({ 2 }, T, RAD_OPD_F_IDX_CU), opd_idx({ 1 }, slots),
                                opd(RAD_I32, { 1 }), opd(RAD_BF16, { T, hk, 128 }), opd(RAD_BF16, { T, hv, 128 }),
                                opd(RAD_BF16, { T, N }) });
}

inline int shape_attn_kv(const RadParam* p, int n_p, int operand, RadOpdDesc* out) {
    const int64_t T = dim(p, n_p, "M"), h = dim(p, n_p, "n_head_kv"), D = dim(p, n_p, "head_dim"), slots = 2 * T;
    return pick(out, operand, { opd(RAD_BF16, { T, h, D }), opd(RAD_BF16, { T, h, D }), opd(RAD_F32, { D }),
                                opd_idx({ T }, 1 << 20), opd_idx({ T }, slots, RAD_OPD_F_IDX_UNIQUE),
                                opd(RAD_BF16, { 2, slots, h, D }), opd(RAD_BF16, { T, h, D }) });
}

}  // namespace ridgefill_schema

#endif /* RIDGEFILL_SCHEMAS_H */
