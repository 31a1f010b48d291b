/* rows.cpp -- the B200 RidgeFill library's row table, plugin exports and the int8 GEMM's stored-form
 * hooks.
 *
 * Exports exactly the reference plugin's seven functions (kernels/rows.cpp:382-399) and answers
 * with the reference's nine schemas first, then this library's three new ops. Every row here is a
 * DEVICE row (sm_100a CUDA); the library has no host rows and no fallback: the engine's oracle mode
 * loads a host-row library beside it, and a call whose launch the device refuses returns
 * RAD_E_DEVICE rather than computing anything on the host.
 *
 * ridgefill_gemm_nt_q keeps the reference's contract that its weight arrives in the STORED form its
 * own layout hook describes (kernels/rows.cpp:161-167, arch/ridgefill_int8.h:87-130). This row's
 * stored form: codes exactly as the folder holds them (i8 [N, K] row-major; the tensor-memory
 * loads tile them), and the bf16 [N, K/128] scale plane transposed and widened to f32 [K/128, N], so
 * the epilogue reads one contiguous scale row per K block. bf16 -> f32 is exact: the stored form
 * computes the same products as the canonical one.
 */
#include "ridgefill.h"
#include "ridgefill_schemas.h"

#include <cstring>

using namespace ridgefill_schema;

namespace {

const RadConstraint kMaskCons[] = { RAD_CIN("mode", "none class random all step"),
                                    RAD_CLE("M", RIDGEFILL_MASK_MAX_ROWS) };
const RadConstraint kCorrectCons[] = { RAD_CIN("mode", "undo apply") };
const RadConstraint kGemmCons[] = { RAD_CIN("dtype", "i8a8") };
const RadConstraint kQuantCons[] = { RAD_CIN("dtype", "bf16") };
const RadConstraint kGemmBiasCons[] = { RAD_CIN("dtype", "bf16") };

/* ------------------------------------------------------------------ stored-form hooks */

/* The hooks serve operand 2 (codes) and 3 (scale) of the i8*bf16[1x128] encoding at the N, K the
 * parameters give. */
int stored_geometry(const RadParam* p, int n_p, int operand, const RadEncoding* enc, const RadTensor* geom,
                    int64_t* N, int64_t* K) {
    *N = rad_param_getdim(p, n_p, "N", 0);
    *K = rad_param_getdim(p, n_p, "K", 0);
    const int64_t group = rad_param_getdim(p, n_p, "group", 0);
    if (!enc || !geom || (operand != GQ_B && operand != GQ_B_SCALE)) return RAD_E_INVAL;
    if (enc->codes != RAD_I8 || enc->scale != RAD_BF16 || enc->group_rows != 1 || enc->group_cols != 128 || group != 128)
        return RAD_E_UNSUPPORTED;
    if (*N <= 0 || *K <= 0 || *K % 128 != 0 || *N % 16 != 0) return RAD_E_SHAPE;
    if (geom->rank != 2) return RAD_E_SHAPE;
    if (operand == GQ_B && (geom->dtype != RAD_I8 || geom->shape[0] != *N || geom->shape[1] != *K)) return RAD_E_SHAPE;
    if (operand == GQ_B_SCALE && (geom->dtype != RAD_BF16 || geom->shape[0] != *N || geom->shape[1] != *K / 128))
        return RAD_E_SHAPE;
    return RAD_OK;
}

int gemm_layout(const RadParam* p, int n_p, int operand, const RadEncoding* enc, const int*, const RadTensor* geom,
                int n_geom, RadLayout* out) {
    int64_t N = 0, K = 0;
    if (n_geom < 1 || !out) return RAD_E_INVAL;
    const int rc = stored_geometry(p, n_p, operand, enc, geom, &N, &K);
    if (rc != RAD_OK) return rc;
    out->bytes = operand == GQ_B ? N * K : (K / 128) * N * 4;
    out->tag = operand == GQ_B ? "ridgefill.b200.codes.nk" : "ridgefill.b200.scale.f32.kn";
    out->align = 128;
    return RAD_OK;
}

/* Canonical -> stored (host memory to host memory; the caller uploads the result). */
int gemm_relayout(const RadParam* p, int n_p, int operand, const RadEncoding* enc, const int*, const RadTensor* src,
                  int n_src, void* dst, int64_t dst_bytes) {
    int64_t N = 0, K = 0;
    if (n_src < 1 || !src || !src->data || !dst) return RAD_E_INVAL;
    const int rc = stored_geometry(p, n_p, operand, enc, src, &N, &K);
    if (rc != RAD_OK) return rc;
    if (operand == GQ_B) {
        if (dst_bytes < N * K) return RAD_E_SHAPE;
        for (int64_t n = 0; n < N; ++n)
            std::memcpy((char*)dst + n * K, (const char*)src->data + n * src->stride[0], (size_t)K);
        return RAD_OK;
    }
    const int64_t blocks = K / 128;
    if (dst_bytes < blocks * N * 4) return RAD_E_SHAPE;
    float* out = (float*)dst;
    const uint16_t* in = (const uint16_t*)src->data;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t j = 0; j < blocks; ++j) out[j * N + n] = rad_bf16_to_f32(in[n * src->stride[0] + j * src->stride[1]]);
    return RAD_OK;
}

/* Stored -> canonical: `src` describes the canonical plane's geometry, its data the stored bytes. */
int gemm_unrelayout(const RadParam* p, int n_p, int operand, const RadEncoding* enc, const int*, const RadTensor* src,
                    int n_src, void* dst, int64_t dst_bytes) {
    int64_t N = 0, K = 0;
    if (n_src < 1 || !src || !src->data || !dst) return RAD_E_INVAL;
    const int rc = stored_geometry(p, n_p, operand, enc, src, &N, &K);
    if (rc != RAD_OK) return rc;
    if (operand == GQ_B) {
        if (dst_bytes < N * K) return RAD_E_SHAPE;
        std::memcpy(dst, src->data, (size_t)(N * K));
        return RAD_OK;
    }
    const int64_t blocks = K / 128;
    if (dst_bytes < blocks * N * 2) return RAD_E_SHAPE;
    const float* in = (const float*)src->data;
    uint16_t* out = (uint16_t*)dst;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t j = 0; j < blocks; ++j) out[n * blocks + j] = rad_f32_to_bf16(in[j * N + n]);
    return RAD_OK;
}

#define DEVICE_ROW(nm, op, what, shp, dts, cons, ncons, fn, scratchfn, shapefn, lay, rel, unrel)                   \
    { nm, op, "ridgefill", what, shp, dts, RAD_DOMAIN_DEVICE, 0, cons, ncons, nullptr, 0, nullptr, nullptr,         \
      nullptr, fn, nullptr, scratchfn, nullptr, shapefn, lay, rel, unrel, nullptr }

const RadKernelInfo kRows[] = {
    DEVICE_ROW("ridgefill_mask_sm100", "ridgefill_mask",
               "last-sequence window mask: one CTA, keys in shared memory, exact 8-bit radix select",
               "b up to RIDGEFILL_MASK_MAX_ROWS, any n", "i32 cu_last / ids / mask / bounds, f32 score", kMaskCons, 2,
               ridgefill_mask_device, nullptr, shape_mask, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_select_sm100", "ridgefill_select", "warp per row, 16 / 4 / 1-byte words, persistent grid",
               "any n and row widths", "any whole-byte dtype per pair, i32 mask", nullptr, 0, ridgefill_select_device,
               nullptr, shape_select, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_drop_rows_sm100", "ridgefill_drop_rows", "warp per row, persistent grid", "any n and top_k",
               "i32 mask / ids", nullptr, 0, ridgefill_drop_device, nullptr, shape_drop, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_rho_update_sm100", "ridgefill_rho_update",
               "affine-map reduction over 256 row runs: 8-CTA cluster x 32 runs, distributed shared memory",
               "any n and n_head", "bf16 or f32 a, i32 mask, f32 A_log / dt_bias / ND", nullptr, 0,
               ridgefill_rho_device, nullptr, shape_rho, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_state_correct_sm100", "ridgefill_state_correct", "CTA per (head, sequence), float4 planes",
               "any slot strides", "f32 state / applied / C / ND, i32 slots", kCorrectCons, 1, ridgefill_correct_device,
               nullptr, shape_correct, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_state_read_sm100", "ridgefill_state_read", "CTA per (head, sequence), float4 copy",
               "any slot strides", "f32 state / out, i32 slots", nullptr, 0, ridgefill_state_read_device, nullptr,
               shape_state_read, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_hazard_sm100", "ridgefill_hazard", "one thread", "any slot strides",
               "i32 cu_last / positions / slots, f32 meta / count", nullptr, 0, ridgefill_hazard_device, nullptr,
               shape_hazard, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_gemm_nt_q_sm100", "ridgefill_gemm_nt_q",
               "tcgen05 kind::i8 (cta_group::2) into tensor memory, TMA-fed, persistent 256x256 tiles on 2-CTA pairs, f32 block fold in the epilogue",
               "K a multiple of 128, N of 16", "i8 a / b, f32 a_scale / stored b_scale, bf16 y", kGemmCons, 1,
               ridgefill_gemm_nt_q_device, nullptr, shape_gemm_q, gemm_layout, gemm_relayout, gemm_unrelayout),
    DEVICE_ROW("ridgefill_gemm_nt_q_bias_sm100", "ridgefill_gemm_nt_q_bias",
               "ridgefill_gemm_nt_q with the bias add fused into the epilogue", "K a multiple of 128, N of 16",
               "i8 a / b, f32 a_scale / stored b_scale, bf16 bias / y, i32 acc", kGemmCons, 1,
               ridgefill_gemm_nt_q_bias_device, nullptr, shape_gemm_q_bias, gemm_layout, gemm_relayout, gemm_unrelayout),
    DEVICE_ROW("ridgefill_gemm_nt_bias_sm100", "ridgefill_gemm_nt_bias",
               "tcgen05 kind::f16 (bf16 operands), TMEM f32 accumulators, TMA 128-B swizzled 256x256 tiles on 2-CTA pairs, bias / silu / "
               "residual epilogue, TMA tile stores", "K a multiple of 64, N of 8", "bf16 a / b / res / y, bf16 or f32 bias",
               kGemmBiasCons, 1, ridgefill_gemm_nt_bias_device, nullptr, shape_gemm_bias, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_quant_act_i8g_sm100", "ridgefill_quant_act_i8g", "warp per row group, 16-byte loads",
               "n a multiple of group", "bf16 x, i8 q, f32 s", kQuantCons, 1, ridgefill_quant_act_device, nullptr,
               shape_quant, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_gdn_fill_sm100", "ridgefill_gdn_fill",
               "chunked gated delta rule: per-chunk WY transform on tensor cores, then the inter-chunk state carry",
               "head dims 128 (chunked, tensor cores) or at most 64 (row by row), chunk 64", "bf16 q / k / v / o, f32 g / beta / state", nullptr, 0, ridgefill_gdn_fill_device,
               ridgefill_gdn_fill_scratch, shape_gdn, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_gdn_conv_prep_sm100", "ridgefill_gdn_conv_prep",
               "warp per 16 rows of a pair of 128-channel head columns, all 16 rows' loads in flight as asynchronous "
               "copies into shared memory; a second kernel updates the conv state in place", "head dims 128, conv width 4",
               "bf16 x / w / state / a / b / q / k / v, f32 A_log / dt_bias / g / beta", nullptr, 0,
               ridgefill_gdn_conv_prep_device, nullptr, shape_conv_prep, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_gdn_in_proj_sm100", "ridgefill_gdn_in_proj",
               "the int8 projector's 2-CTA tcgen05 pipeline over 250-row pair tiles (each CTA's tile starts 3 rows early: "
               "the convolution's window); the epilogue rounds the rows into shared memory and runs the convolution, "
               "SiLU and k norm there, a warp per head and 16 rows, 4 channels a lane", "head dims 128, conv width 4, K a multiple of 128, group = K",
               "i8 a / b, f32 a_scale / b_scale, bf16 w / bias / state / k / v / tail", nullptr, 0,
               ridgefill_gdn_in_proj_device, nullptr, shape_in_proj, nullptr, nullptr, nullptr),
    DEVICE_ROW("ridgefill_attn_kv_fill_sm100", "ridgefill_attn_kv_fill",
               "warp per row: both heads' k and v rows in flight, k_norm by a warp butterfly, the row's rotary angles "
               "one a lane (f64), rotation and the paged stores in the same pass", "head_dim 256, rope_dim a multiple of 16",
               "bf16 k / v / cache / k_out, bf16 or f32 k_norm, i32 positions / slot_mapping", nullptr, 0,
               ridgefill_attn_kv_fill_device, nullptr, shape_attn_kv, nullptr, nullptr, nullptr),
};

#ifndef RIDGEFILL_BUILD_TARGET
#define RIDGEFILL_BUILD_TARGET "sm_100a"
#endif

const RadPluginInfo kInfo = {
    RAD_PLUGIN_KERNEL, "ridgefill", "0.2.0",
    "RidgeFill prefill ops on B200 (sm_100a): ridgefill_mask, ridgefill_select, ridgefill_drop_rows, "
    "ridgefill_rho_update, ridgefill_state_correct, ridgefill_state_read, ridgefill_hazard, the int8 projector "
    "ridgefill_gemm_nt_q (+ fused bias), its activation quantiser, the bf16 ridgefill_gemm_nt_bias, the Gated DeltaNet "
    "chunk fill, its input preparation (ridgefill_gdn_conv_prep) and fused k|v in-projection (ridgefill_gdn_in_proj), and the attention block's K/V cache write "
    "(ridgefill_attn_kv_fill). Device rows only.",
    RIDGEFILL_BUILD_TARGET
};

}  // namespace

extern "C" uint32_t rad_plugin_abi_version(void) { return RAD_ABI_VERSION; }
extern "C" const RadPluginInfo* rad_plugin_info(void) { return &kInfo; }
extern "C" int rad_kernel_schema_count(void) { return (int)(sizeof kSchemas / sizeof kSchemas[0]); }
extern "C" const RadOpSchema* rad_kernel_schema_at(int i) {
    return i >= 0 && i < rad_kernel_schema_count() ? &kSchemas[i] : nullptr;
}
extern "C" int rad_kernel_count(void) { return (int)(sizeof kRows / sizeof kRows[0]); }
extern "C" const RadKernelInfo* rad_kernel_at(int i) { return i >= 0 && i < rad_kernel_count() ? &kRows[i] : nullptr; }
/* No row promises to run concurrently with another launch of itself (kernels/rows.cpp:398-399). */
extern "C" int rad_kernel_concurrent(int) { return 0; }

/* The named hooks of ridgefill.h, for callers that bind them directly. */
extern "C" int ridgefill_gemm_q_layout(const RadParam* p, int n_p, int operand, const RadEncoding* enc, const int* sel,
                                       const RadTensor* geom, int n_geom, RadLayout* out) {
    return gemm_layout(p, n_p, operand, enc, sel, geom, n_geom, out);
}
extern "C" int ridgefill_gemm_q_relayout(const RadParam* p, int n_p, int operand, const RadEncoding* enc,
                                         const int* sel, const RadTensor* src, int n_src, void* dst, int64_t dst_bytes) {
    return gemm_relayout(p, n_p, operand, enc, sel, src, n_src, dst, dst_bytes);
}
extern "C" int ridgefill_gemm_q_unrelayout(const RadParam* p, int n_p, int operand, const RadEncoding* enc,
                                           const int* sel, const RadTensor* src, int n_src, void* dst,
                                           int64_t dst_bytes) {
    return gemm_unrelayout(p, n_p, operand, enc, sel, src, n_src, dst, dst_bytes);
}
