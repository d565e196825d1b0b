/*
 * sacc_scan_plugin.h -- the scan's TensorRT plugin surface as a C ABI.
 *
 * The reference exposes its scan to TensorRT as three IPluginV3 plugins
 * (include/saccade/scan_trt_plugin.hpp:26-49, src/scan_trt_plugin.cpp):
 *   saccade::SelectiveScan   v2  fields: has_d (INT32)
 * plus, without a reference counterpart, the FP16-activation version of the
 * scan for FP16 engines (the reference keeps its scan plugins FP32 there and
 * lets TensorRT cast around them, include/saccade/head_trt_network.hpp:25-28):
 *   saccade::SelectiveScan   v3  fields: has_d (INT32); u, delta, B, C and y
 *                                kHALF, A and D kFLOAT (sacc_selective_scan_f16)
 * and the whole head Mamba block as one plugin (the reference builds it from
 * TensorRT layers around its scan plugin, src/head_trt_network.cpp:181-233):
 *   saccade::MambaBlock      v1  fields: dt_rank, residual (INT32); inputs x
 *                                (B, L, d_model), w_in (2 d_inner, d_model),
 *                                conv_w (d_inner, d_conv), conv_b (d_inner),
 *                                w_x (dt_rank + d_state + 1 or 2 d_state, d_inner),
 *                                w_dt (d_inner, dt_rank), dt_bias (d_inner),
 *                                A (d_inner, d_state), D (d_inner),
 *                                w_out (d_model, d_inner); output (B, L, d_model).
 *                                x, the weights and the output kHALF or kBF16
 *                                (all alike), conv_w / conv_b / dt_bias / A / D
 *                                kFLOAT; a workspace (sacc_plugin_workspace_bytes)
 *                                runs sacc_mamba_block_forward; no status output.
 *   saccade::CrossScanMambaBlock v1  fields: dt_rank, residual (INT32); the
 *                                head level's CrossScanExpand -> block -> merge
 *                                (src/head_trt_network.cpp:200-232) as one plugin
 *                                (sacc_cross_scan_block_forward): inputs as
 *                                MambaBlock except x, the kFLOAT map (B, d_model,
 *                                H, W); the weights' type (w_in) sets the
 *                                activation type; output the kFLOAT map
 *                                (B, d_model, H, W); workspace required.
 *   saccade::CrossScanExpand v1  fields: none
 *   saccade::CrossScanMerge  v1  fields: height, width (INT32)
 * Each entry point below implements one IPluginV3 / IPluginCreatorV3One method
 * with the reference's semantics and messages, on plain structs; a TensorRT
 * adapter only translates TensorRT's descriptors (PluginTensorDesc) and fields
 * (PluginField) into these.  Errors: SACC_EINVAL (nothing enqueued) or SACC_ECUDA,
 * message from sacc_plugin_last_error().
 */
#ifndef SACC_SCAN_PLUGIN_H
#define SACC_SCAN_PLUGIN_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#include "sacc_scan.h"

#ifdef __cplusplus
extern "C" {
#endif

#define SACC_PLUGIN_NAMESPACE "saccade"
#define SACC_PLUGIN_SCAN_NAME "SelectiveScan"
#define SACC_PLUGIN_SCAN_VERSION "2"
#define SACC_PLUGIN_SCAN_F16_VERSION "3"
#define SACC_PLUGIN_EXPAND_NAME "CrossScanExpand"
#define SACC_PLUGIN_EXPAND_VERSION "1"
#define SACC_PLUGIN_MERGE_NAME "CrossScanMerge"
#define SACC_PLUGIN_MERGE_VERSION "1"
#define SACC_PLUGIN_BLOCK_NAME "MambaBlock"
#define SACC_PLUGIN_BLOCK_VERSION "1"
#define SACC_PLUGIN_LEVEL_NAME "CrossScanMambaBlock"
#define SACC_PLUGIN_LEVEL_VERSION "1"

/* Field and tensor type tags (the adapter maps TensorRT's PluginFieldType,
 * DataType and TensorFormat values onto these). */
#define SACC_FIELD_INT32 1
#define SACC_FIELD_OTHER 0
#define SACC_TENSOR_FLOAT 0
#define SACC_TENSOR_HALF 1
#define SACC_TENSOR_BF16 7
#define SACC_TENSOR_INT32 3
#define SACC_TENSOR_OTHER 99
#define SACC_FORMAT_LINEAR 0
#define SACC_FORMAT_OTHER 99

typedef struct SaccPluginField {
    const char* name;
    const void* data;
    int32_t type;   /* SACC_FIELD_* */
    int32_t length; /* number of values */
} SaccPluginField;

typedef struct SaccTensorDesc {
    int32_t nb_dims;
    int64_t dims[8];
    int32_t type;   /* SACC_TENSOR_* */
    int32_t format; /* SACC_FORMAT_* */
} SaccTensorDesc;

typedef struct SaccScanPlugin SaccScanPlugin;

/* IPluginCreatorV3One::createPlugin (src/scan_trt_plugin.cpp:365-393): exactly
 * the advertised fields, each one INT32 value; unknown, duplicate, missing,
 * wrong-typed or null fields are rejected. */
int sacc_plugin_create(const char* name, const char* version, const SaccPluginField* fields, int32_t nb_fields,
                       SaccScanPlugin** out);
void sacc_plugin_destroy(SaccScanPlugin* plugin);
/* IPluginV3::clone (:83-89): semantic fields and the context binding. */
int sacc_plugin_clone(const SaccScanPlugin* plugin, SaccScanPlugin** out);
/* getFieldsToSerialize (:244): -1 for a field the plugin does not have. */
int sacc_plugin_fields(const SaccScanPlugin* plugin, int32_t* has_d, int32_t* height, int32_t* width);
/* getOutputDataTypes (:102-109). */
int sacc_plugin_output_types(const SaccScanPlugin* plugin, const int32_t* in_types, int32_t nb_in, int32_t* out_types,
                             int32_t nb_out);
/* getOutputShapes (:111-160) for concrete input dims. */
int sacc_plugin_output_shapes(const SaccScanPlugin* plugin, const SaccTensorDesc* in, int32_t nb_in, SaccTensorDesc* out,
                              int32_t nb_out);
/* supportsFormatCombination (:163-167): 1 when supported. */
int sacc_plugin_supports_format(const SaccScanPlugin* plugin, int32_t pos, const SaccTensorDesc* io, int32_t nb_in,
                                int32_t nb_out);
/* getWorkspaceSize (:184-186): always 0 for the scan plugins. */
size_t sacc_plugin_workspace_size(const SaccScanPlugin* plugin);
/* getWorkspaceSize with the (maximum) input shapes: the MambaBlock and
 * CrossScanMambaBlock plugins' workspace in bytes, 0 for the others. */
int sacc_plugin_workspace_bytes(const SaccScanPlugin* plugin, const SaccTensorDesc* in, int32_t nb_in, size_t* bytes);
/* getFieldsToSerialize of the MambaBlock and CrossScanMambaBlock plugins. */
int sacc_plugin_block_fields(const SaccScanPlugin* plugin, int32_t* dt_rank, int32_t* residual);
/* configurePlugin / attachToContext (:171-180, 233-242): load every kernel in
 * the current CUDA context and bind the plugin to that context. */
int sacc_plugin_bind(SaccScanPlugin* plugin);
/* enqueue (:201-229): explicit non-default stream of the bound context,
 * descriptor checks (:299-341), then the operator on `stream`. */
int sacc_plugin_enqueue(const SaccScanPlugin* plugin, const SaccTensorDesc* in_desc, const SaccTensorDesc* out_desc,
                        const void* const* inputs, void* const* outputs, cudaStream_t stream);
/* enqueue with TensorRT's workspace (required by MambaBlock and
 * CrossScanMambaBlock, ignored by the scan plugins). */
int sacc_plugin_enqueue_ws(const SaccScanPlugin* plugin, const SaccTensorDesc* in_desc, const SaccTensorDesc* out_desc,
                           const void* const* inputs, void* const* outputs, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream);
const char* sacc_plugin_last_error(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SACC_SCAN_PLUGIN_H */
