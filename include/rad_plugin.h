/* rad_plugin.h -- what a kernel plugin exports to the radiance engine, and the operand and parameter
 * readers its rows call.
 *
 * The exports are the seven functions the reference plugin defines (kernels/rows.cpp:382-399). The
 * readers are the ones the reference rows call (kernels/host_ref.cpp:64-282): an operand is read by
 * its schema position, a parameter by its key.
 */
#ifndef RAD_PLUGIN_H
#define RAD_PLUGIN_H

#include "rad_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ plugin exports */
uint32_t             rad_plugin_abi_version(void);
const RadPluginInfo* rad_plugin_info(void);
int                  rad_kernel_schema_count(void);
const RadOpSchema*   rad_kernel_schema_at(int i);
int                  rad_kernel_count(void);
const RadKernelInfo* rad_kernel_at(int i);
int                  rad_kernel_concurrent(int i);

/* ------------------------------------------------------------------ readers */

/* Operand i, or null when it is past the list or absent (null data). */
static inline const RadTensor* rad_arg_in(const RadArgs* a, int i) {
    if (!a || !a->t || i < 0 || i >= a->n_t || !a->t[i].data) return NULL;
    return &a->t[i];
}

/* An integer parameter: true and *out set when present. */
static inline int rad_args_geti(const RadArgs* a, const char* key, long long* out) {
    const RadParam* q = a ? rad_param_find(a->p, a->n_p, key) : NULL;
    if (!q || q->type != RAD_P_INT) return 0;
    *out = q->ival;
    return 1;
}

/* A string parameter, or null when absent. */
static inline const char* rad_args_gets(const RadArgs* a, const char* key) {
    const RadParam* q = a ? rad_param_find(a->p, a->n_p, key) : NULL;
    return q && q->type == RAD_P_STR ? q->sval : NULL;
}

/* A floating-point parameter (an integer one reads as its value), or `dflt` when absent. */
static inline double rad_args_getf_or(const RadArgs* a, const char* key, double dflt) {
    const RadParam* q = a ? rad_param_find(a->p, a->n_p, key) : NULL;
    if (!q) return dflt;
    if (q->type == RAD_P_F64) return q->fval;
    if (q->type == RAD_P_INT) return (double)q->ival;
    return dflt;
}

#ifdef __cplusplus
}
#endif

#endif /* RAD_PLUGIN_H */
