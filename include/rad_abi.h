/* rad_abi.h -- the part of the radiance engine's plugin ABI that the RidgeFill kernel library uses.
 *
 * The engine's own header is not part of this repository. This file declares exactly the types,
 * constants and helpers that the reference kernel library (kernels/ridgefill.h, kernels/rows.cpp,
 * kernels/host_ref.cpp, kernels/forward.cpp) and its test harness (tests/kernel_test.cpp) name, with
 * the field order their aggregate initialisers imply:
 *   RadParam    {key, type, ival, ival_hi, sval, fval}        tests/kernel_test.cpp:138-140
 *   RadOpSchema {op, params, n_params, operands, n_operands, doc}   kernels/rows.cpp:84-168
 *   RadKernelInfo, positional as the ROW macro fills it        kernels/rows.cpp:310-315
 *   RadOpdDesc  {dtype, rank, shape, fill, flags, idx_max, idx_const}  kernels/rows.cpp:176-199
 * Binary compatibility with a real radiance build cannot be checked without that build; source
 * compatibility with the reference's sources is checked by compiling them against this header.
 *
 * Everything is plain C so a ctypes, cgo or JNI binding can mirror it field for field.
 */
#ifndef RAD_ABI_H
#define RAD_ABI_H

#include <stddef.h>
#include <stdint.h>
#include <string.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Major 15, minor 0, patch 0: the ABI the reference plugin was built against (its CMakeLists.txt:36
 * names radiance ABI 15.0.0). */
#define RAD_ABI_VERSION ((15u << 16) | (0u << 8) | 0u)

enum { RAD_MAX_RANK = 8 };

/* ------------------------------------------------------------------ status codes */
enum {
    RAD_OK = 0,
    RAD_E_INVAL = -1,        /* a required operand or parameter is missing or out of range */
    RAD_E_DTYPE = -2,        /* an operand has the wrong element type */
    RAD_E_SHAPE = -3,        /* extents do not agree, or exceed what the row serves */
    RAD_E_STRIDE = -4,       /* a layout the row does not read (e.g. a gap in a dense operand) */
    RAD_E_UNSUPPORTED = -5,  /* the row exists but does not serve this call */
    RAD_E_DEVICE = -6,       /* the launch failed on the device */
    RAD_E_NOMEM = -7
};

static inline const char* rad_strerror(int rc) {
    switch (rc) {
    case RAD_OK: return "ok";
    case RAD_E_INVAL: return "invalid operand or parameter";
    case RAD_E_DTYPE: return "wrong dtype";
    case RAD_E_SHAPE: return "wrong shape";
    case RAD_E_STRIDE: return "unsupported stride";
    case RAD_E_UNSUPPORTED: return "unsupported";
    case RAD_E_DEVICE: return "device error";
    case RAD_E_NOMEM: return "out of memory";
    default: return "unknown error";
    }
}

/* ------------------------------------------------------------------ element types */
enum {
    RAD_F32 = 1,
    RAD_BF16 = 2,
    RAD_F16 = 3,
    RAD_I32 = 4,
    RAD_I8 = 5,
    RAD_U8 = 6,
    RAD_F8E4M3 = 7,
    RAD_I4 = 8,
    RAD_I64 = 9
};

static inline int rad_dtype_bits(uint32_t dtype) {
    switch (dtype) {
    case RAD_F32: case RAD_I32: return 32;
    case RAD_BF16: case RAD_F16: return 16;
    case RAD_I8: case RAD_U8: case RAD_F8E4M3: return 8;
    case RAD_I4: return 4;
    case RAD_I64: return 64;
    default: return 0;
    }
}

/* Bytes that `n` packed elements of `dtype` occupy (sub-byte types round up). */
static inline int64_t rad_dtype_bytes(uint32_t dtype, int64_t n) {
    return (n * (int64_t)rad_dtype_bits(dtype) + 7) / 8;
}

static inline float rad_bf16_to_f32(uint16_t h) {
    const uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* Round to nearest, ties to even; a NaN stays a (quiet) NaN. */
static inline uint16_t rad_f32_to_bf16(float f) {
    uint32_t bits;
    memcpy(&bits, &f, sizeof bits);
    if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x007fffffu)) return (uint16_t)((bits >> 16) | 0x40u);
    bits += 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

static inline float rad_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1f, man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else {   /* subnormal: renormalise */
            int e = -1;
            uint32_t m = man;
            do { ++e; m <<= 1; } while (!(m & 0x400));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ff) << 13);
        }
    } else if (exp == 31) bits = sign | 0x7f800000u | (man << 13);
    else bits = sign | ((exp + 112) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* Element i of a packed buffer as f32 (f32, bf16, f16, i32, i8, u8). */
static inline float rad_load_f32(const void* base, uint32_t dtype, int64_t i) {
    const unsigned char* p = (const unsigned char*)base;
    switch (dtype) {
    case RAD_F32: { float v; memcpy(&v, p + 4 * i, 4); return v; }
    case RAD_BF16: { uint16_t v; memcpy(&v, p + 2 * i, 2); return rad_bf16_to_f32(v); }
    case RAD_F16: { uint16_t v; memcpy(&v, p + 2 * i, 2); return rad_f16_to_f32(v); }
    case RAD_I32: { int32_t v; memcpy(&v, p + 4 * i, 4); return (float)v; }
    case RAD_I8: return (float)(int8_t)p[i];
    case RAD_U8: return (float)p[i];
    default: return 0.0f;
    }
}

/* Store v as element i of a packed buffer (f32, bf16, i32, i8, u8; integers truncate). */
static inline void rad_store_f32(void* base, uint32_t dtype, int64_t i, float v) {
    unsigned char* p = (unsigned char*)base;
    switch (dtype) {
    case RAD_F32: memcpy(p + 4 * i, &v, 4); break;
    case RAD_BF16: { const uint16_t h = rad_f32_to_bf16(v); memcpy(p + 2 * i, &h, 2); break; }
    case RAD_I32: { const int32_t x = (int32_t)v; memcpy(p + 4 * i, &x, 4); break; }
    case RAD_I8: p[i] = (unsigned char)(int8_t)v; break;
    case RAD_U8: p[i] = (unsigned char)v; break;
    default: break;
    }
}

/* ------------------------------------------------------------------ tensors
 * A strided view: element (i0, i1, ...) is at data + sum(i_k * stride[k]) elements. A null `data`
 * is an ABSENT operand; a zero-extent operand is present with a non-null data pointer. */
typedef struct RadTensor {
    uint32_t dtype;
    uint32_t rank;
    int64_t  shape[RAD_MAX_RANK];
    int64_t  stride[RAD_MAX_RANK];
    void*    data;
} RadTensor;

static inline int64_t rad_tensor_numel(const RadTensor* t) {
    int64_t n = 1;
    for (uint32_t i = 0; i < t->rank; ++i) n *= t->shape[i];
    return n;
}

/* Packed row-major strides for t's shape. */
static inline void rad_tensor_pack(RadTensor* t) {
    int64_t s = 1;
    for (uint32_t i = t->rank; i-- > 0;) {
        t->stride[i] = s;
        s *= t->shape[i];
    }
}

/* True when t's strides are the packed row-major ones (extent-1 and empty axes are not checked). */
static inline int rad_tensor_is_contiguous(const RadTensor* t) {
    int64_t s = 1;
    for (uint32_t i = t->rank; i-- > 0;) {
        if (t->shape[i] == 0) return 1;
        if (t->shape[i] != 1 && t->stride[i] != s) return 0;
        s *= t->shape[i];
    }
    return 1;
}

/* ------------------------------------------------------------------ parameters */
enum { RAD_P_INT = 1, RAD_P_STR = 2, RAD_P_F64 = 3 };
enum { RAD_OPTIONAL = 0, RAD_REQUIRED = 1 };
enum { RAD_PROLE_NONE = 0, RAD_PROLE_SEQ_CHUNK = 1, RAD_PROLE_CAPACITY = 2 };

typedef struct RadParam {
    const char* key;
    int         type;      /* RAD_P_* */
    long long   ival;      /* RAD_P_INT value (a ranged parameter: its lower bound) */
    long long   ival_hi;   /* a ranged parameter's upper bound, 0 otherwise */
    const char* sval;      /* RAD_P_STR value */
    double      fval;      /* RAD_P_F64 value */
} RadParam;

#define RAD_INT(k, v) { (k), RAD_P_INT, (long long)(v), 0, NULL, 0.0 }
#define RAD_STR(k, v) { (k), RAD_P_STR, 0, 0, (v), 0.0 }
#define RAD_F64(k, v) { (k), RAD_P_F64, 0, 0, NULL, (double)(v) }

static inline const RadParam* rad_param_find(const RadParam* p, int n_p, const char* key) {
    for (int i = 0; p && key && i < n_p; ++i)
        if (p[i].key && strcmp(p[i].key, key) == 0) return &p[i];
    return NULL;
}

/* An integer parameter's value; `dflt` when absent or not an integer. */
static inline int64_t rad_param_getdim(const RadParam* p, int n_p, const char* key, int64_t dflt) {
    const RadParam* q = rad_param_find(p, n_p, key);
    return q && q->type == RAD_P_INT ? (int64_t)q->ival : dflt;
}

static inline const char* rad_param_gets(const RadParam* p, int n_p, const char* key, const char* dflt) {
    const RadParam* q = rad_param_find(p, n_p, key);
    return q && q->type == RAD_P_STR && q->sval ? q->sval : dflt;
}

/* ------------------------------------------------------------------ schemas */
enum { RAD_OPD_IN = 0, RAD_OPD_OUT = 1, RAD_OPD_INOUT = 2, RAD_OPD_WEIGHT = 3 };

typedef struct RadParamSpec {
    const char* key;
    uint32_t    type;      /* RAD_P_* */
    uint32_t    required;  /* RAD_REQUIRED / RAD_OPTIONAL */
    uint32_t    role;      /* RAD_PROLE_* */
} RadParamSpec;

typedef struct RadOperandSpec {
    const char* name;
    uint32_t    kind;      /* RAD_OPD_* */
    uint32_t    optional;  /* 1: may be absent */
} RadOperandSpec;

typedef struct RadOpSchema {
    const char*           op;
    const RadParamSpec*   params;
    int                   n_params;
    const RadOperandSpec* operands;
    int                   n_operands;
    const char*           doc;
} RadOpSchema;

/* ------------------------------------------------------------------ launches */
typedef void* RadStream;   /* a cudaStream_t on a device row, ignored by a host row */

typedef struct RadArgs {
    const RadTensor* t;           /* operands in schema order */
    int              n_t;
    const RadParam*  p;
    int              n_p;
    int              rank;        /* tensor-parallel rank of this launch */
    int              world_size;
    void*            scratch;     /* device scratch the row's scratch hook asked for, or null */
    int64_t          scratch_bytes;
} RadArgs;

/* ------------------------------------------------------------------ row constraints */
enum { RAD_C_IN = 1, RAD_C_LE = 2, RAD_C_GE = 3, RAD_C_EQ = 4 };

typedef struct RadConstraint {
    const char* key;
    int         op;      /* RAD_C_* */
    long long   ival;    /* RAD_C_LE / GE / EQ bound */
    const char* sval;    /* RAD_C_IN: space-separated admitted strings */
} RadConstraint;

#define RAD_CIN(k, s) { (k), RAD_C_IN, 0, (s) }
#define RAD_CLE(k, v) { (k), RAD_C_LE, (long long)(v), NULL }

/* ------------------------------------------------------------------ operand descriptions (cold calls) */
enum { RAD_FILL_NORMAL = 0, RAD_FILL_INDEX = 1, RAD_FILL_SIGMOID = 2, RAD_FILL_ZERO = 3 };
enum { RAD_OPD_F_ABSENT = 1, RAD_OPD_F_IDX_CU = 2, RAD_OPD_F_IDX_UNIQUE = 4 };

typedef struct RadOpdDesc {
    uint32_t dtype;
    uint32_t rank;
    int64_t  shape[RAD_MAX_RANK];
    uint32_t fill;       /* RAD_FILL_* */
    uint32_t flags;      /* RAD_OPD_F_* */
    int64_t  idx_max;    /* RAD_FILL_INDEX: values drawn in [0, idx_max) (0: the previous operand's extent) */
    int64_t  idx_const;  /* >= 0: every index is this value */
} RadOpdDesc;

/* ------------------------------------------------------------------ stored weight forms */
typedef struct RadEncoding {
    uint32_t codes;        /* element type of the codes plane */
    uint32_t scale;        /* element type of the scale plane */
    int32_t  group_rows;   /* one scale per group_rows x group_cols codes */
    int32_t  group_cols;
} RadEncoding;

static inline RadEncoding rad_enc_affine(uint32_t codes, uint32_t scale, int32_t group_rows, int32_t group_cols) {
    RadEncoding e;
    e.codes = codes;
    e.scale = scale;
    e.group_rows = group_rows;
    e.group_cols = group_cols;
    return e;
}

typedef struct RadLayout {
    int64_t     bytes;     /* size of the stored form */
    const char* tag;       /* names the arrangement; equal tags describe equal bytes */
    int64_t     align;     /* required alignment of the stored form's base address */
} RadLayout;

/* ------------------------------------------------------------------ kernel rows */
enum { RAD_DOMAIN_HOST = 0, RAD_DOMAIN_DEVICE = 1 };

typedef struct RadTunable { const char* key; long long lo, hi, dflt; } RadTunable;

typedef int     (*RadLaunchFn)(const RadArgs* a, RadStream s);
typedef int     (*RadDescribeFn)(const RadArgs* a, char* out, size_t n);
typedef int64_t (*RadScratchFn)(const RadArgs* a);
typedef int     (*RadInitFn)(void);
typedef void    (*RadFiniFn)(void);
typedef int     (*RadOpdShapeFn)(const RadParam* p, int n_p, int operand, RadOpdDesc* out);
typedef int     (*RadLayoutFn)(const RadParam* p, int n_p, int operand, const RadEncoding* enc, const int* sel,
                               const RadTensor* geom, int n_geom, RadLayout* out);
typedef int     (*RadRelayoutFn)(const RadParam* p, int n_p, int operand, const RadEncoding* enc, const int* sel,
                                 const RadTensor* src, int n_src, void* dst, int64_t dst_bytes);
typedef int     (*RadHookFn)(const RadArgs* a);

typedef struct RadKernelInfo {
    const char*          name;
    const char*          op;
    const char*          plugin;
    const char*          computes;
    const char*          shapes;
    const char*          dtypes;
    int                  domain;          /* RAD_DOMAIN_* */
    int                  priority;
    const RadConstraint* constraints;
    int                  n_constraints;
    const RadTunable*    tunables;
    int                  n_tunables;
    RadInitFn            init;
    RadFiniFn            fini;
    RadHookFn            prepare;
    RadLaunchFn          launch;
    RadDescribeFn        describe;
    RadScratchFn         scratch;
    RadHookFn            validate;
    RadOpdShapeFn        opd_shape;
    RadLayoutFn          layout;
    RadRelayoutFn        relayout;
    RadRelayoutFn        unrelayout;
    const char*          replaces;
} RadKernelInfo;

/* ------------------------------------------------------------------ plugins */
enum { RAD_PLUGIN_KERNEL = 1, RAD_PLUGIN_ARCH = 2 };

typedef struct RadPluginInfo {
    uint32_t    kind;          /* RAD_PLUGIN_* */
    const char* name;
    const char* version;
    const char* description;
    const char* build_target;
} RadPluginInfo;

#ifdef __cplusplus
}
#endif

#endif /* RAD_ABI_H */
