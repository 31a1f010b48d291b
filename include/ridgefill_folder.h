/* ridgefill_folder.h -- the RidgeFill projector folder read, checked and held resident in HBM.
 *
 * The reference's arch plugin reads the folder once a process (arch/ridgefill_folder.h:246-293: the manifest
 * ridgefill.json of format 1, every file it lists mapped read-only and checked against its sha256, each
 * .safetensors file's tensors named), checks it against the model (arch/ridgefill_projector.h:84-129) and keeps
 * every late layer's map in HOST memory, streaming each layer through one VRAM slot on every approximate pass
 * (arch/ridgefill_projector.h:10-18, 282-336). A B200 has the room to keep them all: 24 maps of the served model
 * are 0.64 GB of 180 GB. This API reads and checks the folder the same way and uploads it ONCE into one device
 * block: every late layer's map in the int8 GEMM row's stored form (relaid out through the row's own hooks,
 * arch/ridgefill_int8.h:106-130) or as bf16, its bias, this rank's value heads of each layer's correction, the row
 * tables and the MTP final map when the folder has one. The GEMM rows then read their weights where they lie; no
 * pass copies a map.
 *
 * Ownership: a RidgeFillFolder owns its file mappings (the host views point into them); a RidgeFillResident owns
 * its device block (cudaMalloc'd on the device current at upload, freed by ridgefill_resident_free). Errors:
 * RAD_OK, or a code with `why` (NUL-terminated, truncated to why_bytes) naming the file or tensor: RAD_E_INVAL for
 * a folder that is missing, damaged or does not fit the model, RAD_E_UNSUPPORTED for maps the GEMM row cannot
 * store, RAD_E_NOMEM / RAD_E_DEVICE for the device allocation or copies.
 */
#ifndef RIDGEFILL_FOLDER_H
#define RIDGEFILL_FOLDER_H

#include "rad_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct RidgeFillFolder RidgeFillFolder;
typedef struct RidgeFillResident RidgeFillResident;

/* What the model needs of the folder (the facts arch/ridgefill_projector.h:91-129 checks against). */
typedef struct RidgeFillModelGeom {
    int64_t n_embd;      /* rows of each map (the block input width) */
    int64_t wide;        /* columns of each map (the stream width) */
    int64_t n_layer;     /* layers of the model; late layers are [split, n_layer) */
    int64_t split_lo;    /* the lowest layer a split may name */
    int64_t n_vocab;     /* entries of each row table */
    int64_t st_heads, st_sd0, st_sd1;   /* the correction's [heads, V, K] */
    const uint8_t* full; /* n_layer flags, 1 = full-attention layer (no correction); null: the manifest's "layers" */
} RidgeFillModelGeom;

/* Reads the folder at `dir`: ridgefill.json (format 1, a non-empty "files" object of bare file names), every
 * listed file mapped and its sha256 compared (one thread a file), every .safetensors file's tensors named
 * (dtypes BF16, F32, F16, I8, I32; each tensor's byte span equal to its shape times its dtype and inside the
 * file; a name in two files refuses the folder). Unlisted files (a README) are not read. */
int ridgefill_folder_open(const char* dir, RidgeFillFolder** out, char* why, size_t why_bytes);
void ridgefill_folder_close(RidgeFillFolder* f);

/* The folder's tensor `name` as a host view into its file's mapping (dense, read-only): RAD_OK, or RAD_E_INVAL
 * when absent. */
int ridgefill_folder_tensor(const RidgeFillFolder* f, const char* name, RadTensor* out);
int64_t ridgefill_folder_tensor_count(const RidgeFillFolder* f);
int64_t ridgefill_folder_file_bytes(const RidgeFillFolder* f);

/* The folder against the model: the split a late layer at or above split_lo; the projector dtype "bf16" or
 * "i8"; every late layer's map (bf16 `proj.L.weight` [n_embd, wide], or i8 `proj.L.codes` [n_embd, wide] with
 * bf16 `proj.L.scale` [n_embd, wide/128]) and bf16 `proj.L.bias` [n_embd]; the correction `st.L` f32
 * [st_heads, st_sd0, st_sd1] on all of the late recurrent layers or none; `final.weight` bf16 [wide, wide] and
 * `final.bias` [wide] when the manifest names a final map; each row table (score, score_none, score_all) present
 * f32 [n_vocab]. *split and *int8 (either may be null) receive what was read. */
int ridgefill_folder_check(const RidgeFillFolder* f, const RidgeFillModelGeom* m, int64_t* split, int* int8,
                           char* why, size_t why_bytes);

/* Checks the folder (as ridgefill_folder_check) and uploads it on `s` (a cudaStream_t) into one device block on
 * the current device, 256-byte aligned pieces: per late layer the map (i8: the stored codes and f32 scale the
 * int8 GEMM row's layout hook describes; bf16: [n_embd, wide]) and its bias; heads [head_first, head_first +
 * n_heads) of each correction (n_heads < 0: all); every row table; the final map. Synchronises `s` once at the
 * end. */
int ridgefill_folder_upload(const RidgeFillFolder* f, const RidgeFillModelGeom* m, int64_t head_first,
                            int64_t n_heads, RadStream s, RidgeFillResident** out, char* why, size_t why_bytes);
void ridgefill_resident_free(RidgeFillResident* r);
int64_t ridgefill_resident_bytes(const RidgeFillResident* r);

/* Device views of what was uploaded (RAD_E_INVAL when the folder holds none):
 *  map: i8 folder -> w = codes i8 [n_embd, wide] (ridgefill_gemm_nt_q's operand 2), scale = f32 [wide/128,
 *       n_embd] (operand 3), bias bf16 [n_embd]; bf16 folder -> w = bf16 [n_embd, wide] (ridgefill_gemm_nt_bias's
 *       b), scale absent (data null), bias bf16 [n_embd];
 *  correction: f32 [n_heads, st_sd0, st_sd1] (ridgefill_state_correct's C);
 *  table: f32 [n_vocab] by name (ridgefill_mask's score);
 *  final: bf16 [wide, wide] and [wide]. */
int ridgefill_resident_map(const RidgeFillResident* r, int64_t layer, RadTensor* w, RadTensor* scale, RadTensor* bias);
int ridgefill_resident_correction(const RidgeFillResident* r, int64_t layer, RadTensor* out);
int ridgefill_resident_table(const RidgeFillResident* r, const char* name, RadTensor* out);
int ridgefill_resident_final(const RidgeFillResident* r, RadTensor* w, RadTensor* bias);

#ifdef __cplusplus
}
#endif

#endif /* RIDGEFILL_FOLDER_H */
