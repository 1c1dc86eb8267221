/*
 * hf_ingest.h -- checkpoint ingest: safetensors shards -> resident HBM weights.
 *
 * Replaces the reference's weight path for the MoE layer: SafeTensorsFile
 * (model/safetensors.h:18-80, safetensors.cpp:52-223) parses and validates a
 * shard, WeightIndex::build (model/weight_index.cpp:79-250) maps tensor names
 * to layer / expert slots, and ExpertGpuCache (compute/cuda_backend.cpp:
 * 196-364) stages each expert through pinned host buffers into device memory.
 * Here the whole layer is made resident in one call: the shards' tensor bytes
 * are read (pread, several threads) into a ring of pinned buffers and copied
 * asynchronously to their final device addresses -- the expert blocks of the
 * [gate|up|down] layout, the router, the bias, the shared expert -- with no
 * host-side concatenation.
 *
 * Validation follows SafeTensorsOptions (safetensors.h:32-48): JSON header of
 * a multiple of 8 bytes inside the file, known dtypes, BF16 only except F32
 * for names containing an allowed fragment (e_score_correction_bias in the
 * loader, weight_index.cpp:20-27), non-empty integer shapes, data_offsets
 * [begin, end) with begin < end inside the file, 8-byte aligned absolute data
 * start, shape x dtype size == byte span. Rejected tensors are counted
 * (hf_st_stats) and left out, as the reference does; a name given twice keeps
 * its last entry (the reference's JSON object does the same, so its duplicate
 * counter stays 0).
 */
#ifndef HF_INGEST_H
#define HF_INGEST_H

#include "hf_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* SafeTensorsOptions (model/safetensors.h:38-48). */
typedef struct hf_st_options {
    int require_bf16;              /* dtype must be BF16 (or an allowed F32)          */
    const char* const* allow_f32;  /* name fragments whose tensors may be F32         */
    int num_allow_f32;
    int require_aligned_header;    /* JSON header length a multiple of 8              */
    int require_aligned_data;      /* absolute data start 8-byte aligned              */
} hf_st_options;

/* SafeTensorsStats (model/safetensors.h:50-61). */
typedef struct hf_st_stats {
    uint64_t total, accepted, rejected;
    uint64_t duplicate_rejected, dtype_rejected, f32_allowed_accepted, shape_rejected;
    uint64_t bounds_rejected, byte_mismatch_rejected, alignment_rejected;
} hf_st_stats;

typedef struct hf_st_file hf_st_file;

/* SafeTensorsFile::open (safetensors.cpp:52-223). opts NULL: the checkpoint
 * loader's strict options (BF16, F32 only for e_score_correction_bias,
 * aligned header and data). Fails (HF_ERR_ARG) when the file cannot be read,
 * the header is not a JSON object or lies outside the file; individual bad
 * tensors are rejected and counted in *stats (may be NULL). */
HF_API hf_status hf_st_open(const char* path, const hf_st_options* opts, hf_st_file** out,
                            hf_st_stats* stats);
HF_API hf_status hf_st_close(hf_st_file* f);
/* Accepted tensors, in header order. */
HF_API int hf_st_count(const hf_st_file* f);
/* Tensor i: name, dtype ("BF16", "F32", ...), its number of dims (the first
 * shape_cap of them go to shape), absolute file offset of its data and its
 * byte size. Strings live as long as the file; they are C strings, so a name
 * whose JSON spells \u0000 ends there. */
HF_API hf_status hf_st_tensor(const hf_st_file* f, int i, const char** name, const char** dtype,
                              int* ndim, int64_t* shape, int shape_cap, uint64_t* file_offset,
                              uint64_t* bytes);
/* Index of the tensor named `name`, or -1 (SafeTensorsFile::find). */
HF_API int hf_st_find(const hf_st_file* f, const char* name);
/* SafeTensorsFile::readTensor (safetensors.cpp:230-262) into host memory. */
HF_API hf_status hf_st_read(const hf_st_file* f, int i, void* host_dst, uint64_t capacity);
/* Tensor i straight to device memory on `device` through the pinned ring;
 * returns when the bytes are on the device. */
HF_API hf_status hf_st_upload(const hf_st_file* f, int i, void* dev_dst, uint64_t capacity,
                              int device);

/* The shards of checkpoint directory `dir` that hold model layer
 * `model_layer`'s MLP tensors (model.layers.<L>.mlp.*), as WeightIndex::build
 * finds them (weight_index.cpp:79-130): the directory's *.safetensors files,
 * sorted; when model.safetensors.index.json is there and has a weight_map,
 * only the shards it names for those tensors. The paths are written
 * NUL-separated into buf; *num_shards receives their count. HF_ERR_ARG: no
 * shard in dir, an index whose weight_map names no tensor of that layer's MLP
 * (a wrong layer number), an index entry naming a missing shard, or buf too
 * small (*num_shards is still set). No device is touched. */
HF_API hf_status hf_st_layer_shards(const char* dir, int model_layer, char* buf,
                                    size_t buf_bytes, int* num_shards);

/* What hf_moe_load_safetensors did. */
typedef struct hf_ingest_stats {
    uint64_t bytes;         /* tensor bytes copied to the device            */
    int tensors;            /* tensors copied                               */
    int experts;            /* routed experts loaded (owned by this context) */
    int skipped_experts;    /* routed experts owned by another rank         */
    int has_bias;           /* e_score_correction_bias found                */
    double seconds;         /* wall time of the call                        */
} hf_ingest_stats;

/* Makes context layer `layer` resident from the shards holding model layer
 * `model_layer` (tensor names of weight_index.cpp:219-244):
 *   model.layers.<L>.mlp.gate.weight                       [E x H]  BF16
 *   model.layers.<L>.mlp.gate.e_score_correction_bias      [E]      F32 (optional)
 *   model.layers.<L>.mlp.experts.<e>.{gate,up}_proj.weight [I x H]  BF16
 *   model.layers.<L>.mlp.experts.<e>.down_proj.weight      [H x I]  BF16
 *   model.layers.<L>.mlp.shared_experts.{gate,up,down}_proj.weight (when I_s > 0)
 * Every owned expert (all E on one device, E/W under expert parallelism) must
 * be present with exactly these shapes; other tensors are ignored. Marks the
 * layer loaded. Synchronous. */
HF_API hf_status hf_moe_load_safetensors(hf_moe_ctx* ctx, int layer, int model_layer,
                                         const char* const* shard_paths, int num_shards,
                                         hf_ingest_stats* stats);

/* One routed expert from three separate tensors -- the checkpoint's
 * experts.<e>.{gate,up,down}_proj (ExpertWeights, model/weight_index.h:26-34) --
 * written into its [gate|up|down] block; host or device pointers. */
HF_API hf_status hf_moe_set_expert_parts(hf_moe_ctx* ctx, int layer, int eid, const uint16_t* gate,
                                         const uint16_t* up, const uint16_t* down,
                                         hf_mem_kind kind);

/* Frees the process-wide pinned staging ring (allocated by the first upload). */
HF_API hf_status hf_ingest_release_staging(void);

#ifdef __cplusplus
}
#endif
#endif /* HF_INGEST_H */
