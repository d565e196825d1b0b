// scan_plugin.cpp -- the TensorRT plugin surface of the scan, without TensorRT.
//
// The reference registers three IPluginV3 plugins, saccade::SelectiveScan v2,
// saccade::CrossScanExpand v1 and saccade::CrossScanMerge v1
// (src/scan_trt_plugin.cpp:69-455); saccade::SelectiveScan v3 is the same
// scan with FP16 activations (u, delta, B, C, y) for FP16 engines, and
// saccade::MambaBlock v1 the whole head block (sacc_mamba_block_forward) with
// TensorRT's workspace, and saccade::CrossScanMambaBlock v1 a head level's
// expand -> block -> merge on the FP32 maps (sacc_cross_scan_block_forward).  TensorRT itself is not available on this
// platform, so the plugin's logic lives here behind a C ABI whose calls map
// one to one onto the IPluginV3 methods; a thin TensorRT adapter translates
// TensorRT's descriptor and field types (PluginTensorDesc, PluginField) into
// these structs and forwards:
//
//   sacc_plugin_create           IPluginCreatorV3One::createPlugin   :365-393
//   sacc_plugin_fields           getFieldsToSerialize                :244
//   sacc_plugin_output_types     getOutputDataTypes                  :102-109
//   sacc_plugin_output_shapes    getOutputShapes (concrete dims)     :111-160
//   sacc_plugin_supports_format  supportsFormatCombination           :163-167
//   sacc_plugin_bind             configurePlugin / attachToContext   :171-180, 233-242, 267-279
//   sacc_plugin_enqueue          enqueue (+ require_bound, check)    :201-229, 283-341
//   sacc_plugin_workspace_size   getWorkspaceSize                    :184-186
//   sacc_plugin_workspace_bytes  getWorkspaceSize with shapes (MambaBlock)
//   sacc_plugin_enqueue_ws       enqueue with TensorRT's workspace (MambaBlock)
//
// Messages keep the reference's text ("saccade::SelectiveScan: ..." and
// "... creator: ..."); rejections return SACC_EINVAL before any GPU work.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "internal.h"
#include "../../include/sacc_scan_plugin.h"

namespace sacc {
namespace {

enum class Op { scan, expand, merge, block, level };

struct Identity {
    const char* name;
    const char* version;
};

Identity identity_of(Op op) {
    return op == Op::scan    ? Identity{SACC_PLUGIN_SCAN_NAME, SACC_PLUGIN_SCAN_VERSION}
         : op == Op::expand  ? Identity{SACC_PLUGIN_EXPAND_NAME, SACC_PLUGIN_EXPAND_VERSION}
         : op == Op::merge   ? Identity{SACC_PLUGIN_MERGE_NAME, SACC_PLUGIN_MERGE_VERSION}
         : op == Op::block   ? Identity{SACC_PLUGIN_BLOCK_NAME, SACC_PLUGIN_BLOCK_VERSION}
                             : Identity{SACC_PLUGIN_LEVEL_NAME, SACC_PLUGIN_LEVEL_VERSION};
}

// MambaBlock inputs: x, w_in, conv_w, conv_b, w_x, w_dt, dt_bias, A, D, w_out.
constexpr int kBlockInputs = 10;
bool block_fp32_input(int pos) { return pos == 2 || pos == 3 || pos == 6 || pos == 7 || pos == 8; }
bool activation_type(int32_t t) { return t == SACC_TENSOR_HALF || t == SACC_TENSOR_BF16; }

struct PluginError {
    int code;
    std::string what;
};

// Driver entry points for the context binding (resolved through the runtime,
// so the library does not link libcuda directly).
struct Driver {
    PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    PFN_cuStreamGetCtx_v9020 stream_ctx = nullptr;
    PFN_cuCtxGetId_v12000 ctx_id = nullptr;
};

const Driver& driver() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q{};
        void* p = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess)
            d.get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        if (cudaGetDriverEntryPointByVersion("cuStreamGetCtx", &p, 12000, cudaEnableDefault, &q) == cudaSuccess)
            d.stream_ctx = reinterpret_cast<PFN_cuStreamGetCtx_v9020>(p);
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) == cudaSuccess)
            d.ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
    });
    return d;
}

bool equal(const SaccTensorDesc& d, std::initializer_list<std::int64_t> want) {
    if (d.nb_dims != static_cast<int>(want.size())) return false;
    int i = 0;
    for (const auto w : want)
        if (d.dims[i++] != w) return false;
    return true;
}

std::string text(const SaccTensorDesc& d) {
    std::string s = "(";
    for (int i = 0; i < d.nb_dims; ++i) s += (i ? "," : "") + std::to_string(d.dims[i]);
    return s + ")";
}

} // namespace
} // namespace sacc

struct SaccScanPlugin {
    sacc::Op op;
    std::int32_t has_d, height, width;
    unsigned long long bound_context = 0; // 0: kernels not loaded for any context
    bool half = false;                    // SelectiveScan v3: FP16 activations
    std::int32_t dt_rank = 0, residual = 0; // MambaBlock / CrossScanMambaBlock fields
    bool blockish() const { return op == sacc::Op::block || op == sacc::Op::level; }
    int inputs() const { return op == sacc::Op::scan ? 5 + has_d : blockish() ? sacc::kBlockInputs : 1; }
    int outputs() const { return blockish() ? 1 : 2; }
    std::string prefix() const { return std::string(SACC_PLUGIN_NAMESPACE) + "::" + sacc::identity_of(op).name + ": "; }
    // Data type of tensor `pos` (inputs, then y, then status).
    int32_t type_at(int pos) const {
        if (pos == inputs() + 1) return SACC_TENSOR_INT32;
        if (!half) return SACC_TENSOR_FLOAT;
        if (pos == inputs()) return SACC_TENSOR_HALF;                         // y
        return (pos == 2 || pos == 5) ? SACC_TENSOR_FLOAT : SACC_TENSOR_HALF; // A and D stay FP32
    }
};

namespace sacc {
namespace {

thread_local std::string g_plugin_error;

template <typename F>
int plugin_guard(F&& body) {
    try {
        body();
        g_plugin_error.clear();
        return SACC_OK;
    } catch (const PluginError& e) {
        g_plugin_error = e.what;
        return e.code;
    } catch (const std::exception& e) {
        g_plugin_error = e.what();
        return SACC_ECUDA;
    }
}

[[noreturn]] void fail(const SaccScanPlugin* p, const std::string& why, int code = SACC_EINVAL) {
    throw PluginError{code, p->prefix() + why};
}

// Why the descriptors break the plugin contract, or "" (reference :299-341).
const char* type_name(int32_t t) { return t == SACC_TENSOR_HALF ? "FP16" : t == SACC_TENSOR_INT32 ? "INT32" : "FP32"; }

std::string check(const SaccScanPlugin& p, const SaccTensorDesc* in, const SaccTensorDesc* out, SaccScanShape& scan,
                  SaccCrossScanShape& cross) {
    for (int i = 0; i < p.inputs(); ++i)
        if (in[i].type != p.type_at(i) || in[i].format != SACC_FORMAT_LINEAR)
            return "input " + std::to_string(i) + " is not linear " + type_name(p.type_at(i));
    if (out[0].type != p.type_at(p.inputs()) || out[0].format != SACC_FORMAT_LINEAR)
        return std::string("output 0 is not linear ") + type_name(p.type_at(p.inputs()));
    if (out[1].type != SACC_TENSOR_INT32 || out[1].format != SACC_FORMAT_LINEAR || !equal(out[1], {2}))
        return "status output is not linear INT32[2]";
    for (int i = 0; i < p.inputs(); ++i)
        for (int k = 0; k < in[i].nb_dims; ++k)
            if (in[i].dims[k] < 0) return "input " + std::to_string(i) + " has an unresolved dimension";
    const SaccTensorDesc& d0 = in[0];
    switch (p.op) {
    case Op::scan: {
        if (d0.nb_dims != 3 || in[2].nb_dims != 2) return "u must be (batch, length, channels) and A (rows, state)";
        const std::int64_t batch = d0.dims[0], length = d0.dims[1], channels = d0.dims[2];
        const std::int64_t rows = in[2].dims[0], state = in[2].dims[1];
        const SaccTensorDesc& c = in[4];
        if (!equal(in[1], {batch, length, channels})) return "delta " + text(in[1]) + " differs from u " + text(d0);
        if (!equal(in[3], {batch, length, state})) return "B " + text(in[3]) + " is not (batch, length, state)";
        if (c.nb_dims != 3 || c.dims[0] != batch || c.dims[1] != length) return "C " + text(c) + " is not (batch, length, width)";
        if (p.has_d && !equal(in[5], {channels})) return "D " + text(in[5]) + " is not (channels)";
        if (!equal(out[0], {batch, length, channels})) return "y " + text(out[0]) + " differs from u";
        scan = SaccScanShape{static_cast<std::uint64_t>(batch), static_cast<std::uint64_t>(length),
                             static_cast<std::uint64_t>(channels), static_cast<std::uint64_t>(state),
                             static_cast<std::uint64_t>(rows), static_cast<std::uint64_t>(c.dims[2]), p.has_d};
        return "";
    }
    case Op::expand: {
        if (d0.nb_dims != 4) return "x " + text(d0) + " is not (batch, channels, height, width)";
        if (!equal(out[0], {4 * d0.dims[0], d0.dims[2] * d0.dims[3], d0.dims[1]}))
            return "tokens " + text(out[0]) + " do not match x " + text(d0);
        cross = SaccCrossScanShape{static_cast<std::uint64_t>(d0.dims[0]), static_cast<std::uint64_t>(d0.dims[1]),
                                   static_cast<std::uint64_t>(d0.dims[2]), static_cast<std::uint64_t>(d0.dims[3])};
        return "";
    }
    case Op::merge: {
        if (d0.nb_dims != 3 || d0.dims[0] % 4 != 0 || d0.dims[1] != std::int64_t{p.height} * p.width)
            return "y " + text(d0) + " is not (4 * batch, " + std::to_string(p.height) + " * " + std::to_string(p.width) +
                   ", channels)";
        if (!equal(out[0], {d0.dims[0] / 4, d0.dims[2], p.height, p.width}))
            return "out " + text(out[0]) + " does not match y " + text(d0);
        cross = SaccCrossScanShape{static_cast<std::uint64_t>(d0.dims[0] / 4), static_cast<std::uint64_t>(d0.dims[2]),
                                   static_cast<std::uint64_t>(p.height), static_cast<std::uint64_t>(p.width)};
        return "";
    }
    }
    return "unknown plugin";
}

// MambaBlock descriptors -> block arguments (shapes and dtype), or why not.
std::string check_block(const SaccScanPlugin& p, const SaccTensorDesc* in, const SaccTensorDesc* out, SaccMambaBlockArgs& a) {
    const int32_t act = in[0].type;
    if (!activation_type(act)) return "input 0 is not FP16 or BF16";
    for (int i = 0; i < kBlockInputs; ++i) {
        if (in[i].format != SACC_FORMAT_LINEAR) return "input " + std::to_string(i) + " is not linear";
        if (in[i].type != (block_fp32_input(i) ? SACC_TENSOR_FLOAT : act))
            return "input " + std::to_string(i) + (block_fp32_input(i) ? " is not FP32" : " differs in type from x");
        for (int k = 0; k < in[i].nb_dims; ++k)
            if (in[i].dims[k] < 1) return "input " + std::to_string(i) + " has an empty or unresolved dimension";
    }
    if (out[0].type != act || out[0].format != SACC_FORMAT_LINEAR) return "output 0 differs in type from x";
    const SaccTensorDesc &x = in[0], &w_in = in[1], &conv_w = in[2], &w_x = in[4], &A = in[7];
    if (x.nb_dims != 3 || w_in.nb_dims != 2 || conv_w.nb_dims != 2 || A.nb_dims != 2 || w_x.nb_dims != 2)
        return "x must be (batch, length, d_model) and the weights matrices";
    const std::int64_t dm = x.dims[2], D = conv_w.dims[0], K = conv_w.dims[1], N = A.dims[1], R = p.dt_rank;
    if (!equal(w_in, {2 * D, dm})) return "w_in " + text(w_in) + " is not (2 d_inner, d_model)";
    if (!equal(in[3], {D})) return "conv_b " + text(in[3]) + " is not (d_inner)";
    const std::int64_t cw = w_x.dims[0] - R - N;
    if (w_x.dims[1] != D || (cw != 1 && cw != N)) return "w_x " + text(w_x) + " is not (dt_rank + d_state + 1 or 2 d_state, d_inner)";
    if (!equal(in[5], {D, R})) return "w_dt " + text(in[5]) + " is not (d_inner, dt_rank)";
    if (!equal(in[6], {D})) return "dt_bias " + text(in[6]) + " is not (d_inner)";
    if (A.dims[0] != D) return "A " + text(A) + " is not (d_inner, d_state)";
    if (!equal(in[8], {D})) return "D " + text(in[8]) + " is not (d_inner)";
    if (!equal(in[9], {dm, D})) return "w_out " + text(in[9]) + " is not (d_model, d_inner)";
    if (!equal(out[0], {x.dims[0], x.dims[1], dm})) return "out " + text(out[0]) + " differs from x";
    a = SaccMambaBlockArgs{};
    a.batch = static_cast<std::uint64_t>(x.dims[0]);
    a.length = static_cast<std::uint64_t>(x.dims[1]);
    a.d_model = static_cast<std::uint64_t>(dm);
    a.d_inner = static_cast<std::uint64_t>(D);
    a.d_state = static_cast<std::uint64_t>(N);
    a.d_conv = static_cast<std::uint64_t>(K);
    a.dt_rank = static_cast<std::uint64_t>(R);
    a.dtype = act == SACC_TENSOR_BF16 ? SACC_DTYPE_BF16 : SACC_DTYPE_F16;
    a.residual = p.residual;
    a.eps = 0.0f;
    a.c_width = static_cast<std::int32_t>(cw);
    return "";
}

// CrossScanMambaBlock descriptors -> level arguments, or why not: x and the
// output are the FP32 maps (batch, d_model, height, width), w_in sets the
// activation type, and the weights follow MambaBlock's rules.
std::string check_level(const SaccScanPlugin& p, const SaccTensorDesc* in, const SaccTensorDesc* out, SaccCrossScanBlockArgs& c) {
    const SaccTensorDesc& x = in[0];
    if (x.type != SACC_TENSOR_FLOAT || x.format != SACC_FORMAT_LINEAR) return "input 0 is not linear FP32";
    if (x.nb_dims != 4) return "x must be (batch, d_model, height, width)";
    for (int k = 0; k < 4; ++k)
        if (x.dims[k] < 1) return "input 0 has an empty or unresolved dimension";
    if (!activation_type(in[1].type)) return "input 1 is not FP16 or BF16";
    if (out[0].type != SACC_TENSOR_FLOAT || out[0].format != SACC_FORMAT_LINEAR ||
        !equal(out[0], {x.dims[0], x.dims[1], x.dims[2], x.dims[3]}))
        return "out " + text(out[0]) + " differs from x";
    // The block's view: (batch, height * width, d_model) tokens of w_in's type.
    SaccTensorDesc tok[kBlockInputs];
    for (int i = 0; i < kBlockInputs; ++i) tok[i] = in[i];
    tok[0] = SaccTensorDesc{3, {x.dims[0], x.dims[2] * x.dims[3], x.dims[1]}, in[1].type, SACC_FORMAT_LINEAR};
    const SaccTensorDesc o = tok[0];
    SaccMambaBlockArgs a{};
    const std::string why = check_block(p, tok, &o, a);
    if (!why.empty()) return why;
    c = SaccCrossScanBlockArgs{};
    c.block = a;
    c.height = static_cast<std::uint64_t>(x.dims[2]);
    c.width = static_cast<std::uint64_t>(x.dims[3]);
    return "";
}

} // namespace
} // namespace sacc

using namespace sacc;

extern "C" {

const char* sacc_plugin_last_error(void) { return g_plugin_error.c_str(); }

// Accepts exactly the advertised fields, each one INT32 value (reference :365-393).
int sacc_plugin_create(const char* name, const char* version, const SaccPluginField* fields, int32_t nb_fields,
                       SaccScanPlugin** out) {
    return plugin_guard([&] {
        if (out == nullptr) throw PluginError{SACC_EINVAL, "sacc_plugin_create: out is required"};
        *out = nullptr;
        Op op;
        bool half = false;
        if (name && !std::strcmp(name, SACC_PLUGIN_SCAN_NAME) && version && !std::strcmp(version, SACC_PLUGIN_SCAN_VERSION))
            op = Op::scan;
        else if (name && !std::strcmp(name, SACC_PLUGIN_SCAN_NAME) && version &&
                 !std::strcmp(version, SACC_PLUGIN_SCAN_F16_VERSION))
            op = Op::scan, half = true;
        else if (name && !std::strcmp(name, SACC_PLUGIN_EXPAND_NAME) && version &&
                 !std::strcmp(version, SACC_PLUGIN_EXPAND_VERSION))
            op = Op::expand;
        else if (name && !std::strcmp(name, SACC_PLUGIN_MERGE_NAME) && version && !std::strcmp(version, SACC_PLUGIN_MERGE_VERSION))
            op = Op::merge;
        else if (name && !std::strcmp(name, SACC_PLUGIN_BLOCK_NAME) && version && !std::strcmp(version, SACC_PLUGIN_BLOCK_VERSION))
            op = Op::block;
        else if (name && !std::strcmp(name, SACC_PLUGIN_LEVEL_NAME) && version && !std::strcmp(version, SACC_PLUGIN_LEVEL_VERSION))
            op = Op::level;
        else
            throw PluginError{SACC_EINVAL, std::string("plugin creator not registered: ") + SACC_PLUGIN_NAMESPACE + "::" +
                                               (name ? name : "(null)") + " v" + (version ? version : "(null)")};
        const char* names[2] = {nullptr, nullptr};
        std::size_t n_names = 0;
        if (op == Op::scan) names[n_names++] = "has_d";
        if (op == Op::merge) {
            names[n_names++] = "height";
            names[n_names++] = "width";
        }
        const bool blockish = op == Op::block || op == Op::level;
        if (blockish) {
            names[n_names++] = "dt_rank";
            names[n_names++] = "residual";
        }
        const std::string who = std::string(SACC_PLUGIN_NAMESPACE) + "::" + identity_of(op).name + " creator: ";
        std::int32_t value[2] = {0, 0};
        bool seen[2] = {false, false};
        if (nb_fields < 0) throw PluginError{SACC_EINVAL, who + "negative field count"};
        if (nb_fields > 0 && fields == nullptr) throw PluginError{SACC_EINVAL, who + "null field list"};
        for (std::int32_t i = 0; i < nb_fields; ++i) {
            const SaccPluginField& f = fields[i];
            std::size_t k = 0;
            while (k < n_names && (f.name == nullptr || std::strcmp(f.name, names[k]) != 0)) ++k;
            if (k == n_names) throw PluginError{SACC_EINVAL, who + "unknown field " + (f.name ? f.name : "(null)")};
            if (seen[k]) throw PluginError{SACC_EINVAL, who + "duplicate field " + f.name};
            if (f.type != SACC_FIELD_INT32 || f.length != 1 || f.data == nullptr)
                throw PluginError{SACC_EINVAL, who + "field " + f.name + " must hold one INT32"};
            std::memcpy(&value[k], f.data, sizeof(std::int32_t));
            seen[k] = true;
        }
        for (std::size_t k = 0; k < n_names; ++k)
            if (!seen[k]) throw PluginError{SACC_EINVAL, who + "missing field " + names[k]};
        if (op == Op::scan && value[0] != 0 && value[0] != 1) throw PluginError{SACC_EINVAL, who + "has_d must be 0 or 1"};
        if (op == Op::merge && (value[0] < 1 || value[1] < 1))
            throw PluginError{SACC_EINVAL, who + "height and width must be positive"};
        if (blockish && value[0] < 1) throw PluginError{SACC_EINVAL, who + "dt_rank must be positive"};
        if (blockish && value[1] != 0 && value[1] != 1) throw PluginError{SACC_EINVAL, who + "residual must be 0 or 1"};
        *out = new SaccScanPlugin{op, op == Op::scan ? value[0] : 1, op == Op::merge ? value[0] : 0,
                                  op == Op::merge ? value[1] : 0, 0, half,
                                  blockish ? value[0] : 0, blockish ? value[1] : 0};
    });
}

void sacc_plugin_destroy(SaccScanPlugin* p) { delete p; }

int sacc_plugin_clone(const SaccScanPlugin* p, SaccScanPlugin** out) {
    return plugin_guard([&] {
        if (!p || !out) throw PluginError{SACC_EINVAL, "sacc_plugin_clone: plugin and out are required"};
        *out = new SaccScanPlugin(*p); // keeps the semantic fields and the context binding
    });
}

// Serialized fields: the semantic attributes only (reference :244).
int sacc_plugin_fields(const SaccScanPlugin* p, int32_t* has_d, int32_t* height, int32_t* width) {
    return plugin_guard([&] {
        if (!p) throw PluginError{SACC_EINVAL, "sacc_plugin_fields: plugin is required"};
        if (has_d) *has_d = p->op == Op::scan ? p->has_d : -1;
        if (height) *height = p->op == Op::merge ? p->height : -1;
        if (width) *width = p->op == Op::merge ? p->width : -1;
    });
}

int sacc_plugin_block_fields(const SaccScanPlugin* p, int32_t* dt_rank, int32_t* residual) {
    return plugin_guard([&] {
        if (!p || !p->blockish())
            throw PluginError{SACC_EINVAL, "sacc_plugin_block_fields: a MambaBlock or CrossScanMambaBlock plugin is required"};
        if (dt_rank) *dt_rank = p->dt_rank;
        if (residual) *residual = p->residual;
    });
}

int sacc_plugin_output_types(const SaccScanPlugin* p, const int32_t* in_types, int32_t nb_in, int32_t* out_types, int32_t nb_out) {
    return plugin_guard([&] {
        if (!p) throw PluginError{SACC_EINVAL, "sacc_plugin_output_types: plugin is required"};
        if (nb_in != p->inputs() || nb_out != p->outputs() || !in_types || !out_types) fail(p, "input or output count");
        if (p->op == Op::level) {
            if (in_types[0] != SACC_TENSOR_FLOAT) fail(p, "input 0 is not FP32");
            if (!activation_type(in_types[1])) fail(p, "input 1 is not FP16 or BF16");
            for (std::int32_t i = 2; i < nb_in; ++i)
                if (in_types[i] != (block_fp32_input(i) ? SACC_TENSOR_FLOAT : in_types[1]))
                    fail(p, "input " + std::to_string(i) + (block_fp32_input(i) ? " is not FP32" : " differs in type from w_in"));
            out_types[0] = SACC_TENSOR_FLOAT;
            return;
        }
        if (p->op == Op::block) {
            if (!activation_type(in_types[0])) fail(p, "input 0 is not FP16 or BF16");
            for (std::int32_t i = 1; i < nb_in; ++i)
                if (in_types[i] != (block_fp32_input(i) ? SACC_TENSOR_FLOAT : in_types[0]))
                    fail(p, "input " + std::to_string(i) + (block_fp32_input(i) ? " is not FP32" : " differs in type from x"));
            out_types[0] = in_types[0];
            return;
        }
        for (std::int32_t i = 0; i < nb_in; ++i)
            if (in_types[i] != p->type_at(i)) fail(p, "input " + std::to_string(i) + " is not " + type_name(p->type_at(i)));
        out_types[0] = p->type_at(nb_in);
        out_types[1] = SACC_TENSOR_INT32;
    });
}

// Output shapes for concrete input dims; same static checks as the reference's
// symbolic getOutputShapes (:111-160).
int sacc_plugin_output_shapes(const SaccScanPlugin* p, const SaccTensorDesc* in, int32_t nb_in, SaccTensorDesc* out,
                              int32_t nb_out) {
    return plugin_guard([&] {
        if (!p) throw PluginError{SACC_EINVAL, "sacc_plugin_output_shapes: plugin is required"};
        if (nb_in != p->inputs() || nb_out != p->outputs() || !in || !out) fail(p, "input or output count");
        if (p->op == Op::level) {
            SaccTensorDesc o{4, {in[0].dims[0], in[0].dims[1], in[0].dims[2], in[0].dims[3]}, SACC_TENSOR_FLOAT, SACC_FORMAT_LINEAR};
            SaccCrossScanBlockArgs c{};
            const std::string why = check_level(*p, in, &o, c);
            if (!why.empty()) fail(p, why);
            out[0] = o;
            return;
        }
        if (p->op == Op::block) {
            SaccTensorDesc o{3, {in[0].dims[0], in[0].dims[1], in[0].dims[2]}, in[0].type, SACC_FORMAT_LINEAR};
            SaccMambaBlockArgs a{};
            const std::string why = check_block(*p, in, &o, a);
            if (!why.empty()) fail(p, why);
            out[0] = o;
            return;
        }
        out[1] = SaccTensorDesc{1, {2}, SACC_TENSOR_INT32, SACC_FORMAT_LINEAR};
        switch (p->op) {
        case Op::scan: {
            const int ranks[6] = {3, 3, 2, 3, 3, 1};
            for (std::int32_t i = 0; i < nb_in; ++i)
                if (in[i].nb_dims != ranks[i]) fail(p, "input " + std::to_string(i) + " rank");
            const auto &u = in[0], &delta = in[1], &a = in[2], &b = in[3], &c = in[4];
            bool differ = b.dims[2] != a.dims[1];
            for (int k = 0; k < 3; ++k) differ = differ || u.dims[k] != delta.dims[k];
            for (int k = 0; k < 2; ++k) differ = differ || u.dims[k] != b.dims[k] || u.dims[k] != c.dims[k];
            if (p->has_d) differ = differ || in[5].dims[0] != u.dims[2];
            if (differ) fail(p, "input dimensions disagree");
            const std::int64_t n = a.dims[1], rows = a.dims[0], width = c.dims[2], channels = u.dims[2];
            if (n < 1 || n > 32 || (n & (n - 1)) != 0) fail(p, "state must be a power of two in [1, 32]");
            if (rows > 1 && rows != channels) fail(p, "A rows must be 1 or channels");
            if (width > 1 && width != n) fail(p, "C width must be 1 or state");
            out[0] = SaccTensorDesc{3, {u.dims[0], u.dims[1], u.dims[2]}, p->type_at(nb_in), SACC_FORMAT_LINEAR};
            return;
        }
        case Op::expand: {
            const auto& x = in[0];
            if (x.nb_dims != 4) fail(p, "x must be (batch, channels, height, width)");
            out[0] = SaccTensorDesc{3, {4 * x.dims[0], x.dims[2] * x.dims[3], x.dims[1]}, SACC_TENSOR_FLOAT, SACC_FORMAT_LINEAR};
            return;
        }
        case Op::merge: {
            const auto& y = in[0];
            if (y.nb_dims != 3) fail(p, "y must be (4 * batch, height * width, channels)");
            if (y.dims[1] != std::int64_t{p->height} * p->width) fail(p, "y length differs from height * width");
            out[0] = SaccTensorDesc{4, {y.dims[0] / 4, y.dims[2], p->height, p->width}, SACC_TENSOR_FLOAT, SACC_FORMAT_LINEAR};
            return;
        }
        }
    });
}

// Dense row-major FP32 everywhere except the INT32 status output (:163-167);
// v3: FP16 u, delta, B, C and y.
int sacc_plugin_supports_format(const SaccScanPlugin* p, int32_t pos, const SaccTensorDesc* io, int32_t nb_in, int32_t nb_out) {
    if (!p || !io || nb_in != p->inputs() || nb_out != p->outputs() || pos < 0 || pos >= nb_in + nb_out) return 0;
    if (io[pos].format != SACC_FORMAT_LINEAR) return 0;
    if (p->op == Op::level) {
        // The maps (x, output) FP32; w_in decides the activation type (FP16 or
        // BF16) of the other weights; conv, bias, A and D rows FP32.
        if (pos == 0 || pos == nb_in) return io[pos].type == SACC_TENSOR_FLOAT;
        if (pos == 1) return activation_type(io[1].type);
        return io[pos].type == (block_fp32_input(pos) ? SACC_TENSOR_FLOAT : io[1].type);
    }
    if (p->op == Op::block) {
        // x decides the activation type (FP16 or BF16); weights in that type, the
        // conv, bias, A and D rows in FP32, the output like x.
        if (pos == 0) return activation_type(io[0].type);
        return io[pos].type == (pos < nb_in && block_fp32_input(pos) ? SACC_TENSOR_FLOAT : io[0].type);
    }
    return io[pos].type == p->type_at(pos);
}

size_t sacc_plugin_workspace_size(const SaccScanPlugin*) { return 0; }

// Loads every kernel in the current CUDA context and remembers that context's
// unique id (reference bind(), :267-279).
int sacc_plugin_bind(SaccScanPlugin* p) {
    return plugin_guard([&] {
        if (!p) throw PluginError{SACC_EINVAL, "sacc_plugin_bind: plugin is required"};
        if (sacc_scan_load_kernels(nullptr, 0) != SACC_OK) fail(p, sacc_last_error(), SACC_ECUDA);
        const Driver& d = driver();
        CUcontext ctx{};
        unsigned long long id = 0;
        if (!d.get_current || !d.ctx_id || d.get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
            d.ctx_id(ctx, &id) != CUDA_SUCCESS)
            fail(p, "no current CUDA context to load the kernels in", SACC_ECUDA);
        p->bound_context = id;
    });
}

// Enqueues the operator on `stream` with the engine's buffers (:201-229): the
// stream must be explicit, non-default and of the bound context; descriptors
// are checked before anything is enqueued.
int sacc_plugin_enqueue(const SaccScanPlugin* p, const SaccTensorDesc* in_desc, const SaccTensorDesc* out_desc,
                        const void* const* in, void* const* out, cudaStream_t stream) {
    return sacc_plugin_enqueue_ws(p, in_desc, out_desc, in, out, nullptr, 0, stream);
}

int sacc_plugin_workspace_bytes(const SaccScanPlugin* p, const SaccTensorDesc* in_desc, int32_t nb_in, size_t* bytes) {
    return plugin_guard([&] {
        if (!p || !bytes) throw PluginError{SACC_EINVAL, "sacc_plugin_workspace_bytes: plugin and bytes are required"};
        *bytes = 0;
        if (!p->blockish()) return;
        if (!in_desc || nb_in != p->inputs()) fail(p, "input count");
        if (p->op == Op::level) {
            SaccTensorDesc o{4, {in_desc[0].dims[0], in_desc[0].dims[1], in_desc[0].dims[2], in_desc[0].dims[3]}, SACC_TENSOR_FLOAT,
                             SACC_FORMAT_LINEAR};
            SaccCrossScanBlockArgs c{};
            const std::string why = check_level(*p, in_desc, &o, c);
            if (!why.empty()) fail(p, why);
            if (sacc_cross_scan_block_workspace(&c, bytes) != SACC_OK) fail(p, sacc_last_error());
            return;
        }
        SaccTensorDesc o{3, {in_desc[0].dims[0], in_desc[0].dims[1], in_desc[0].dims[2]}, in_desc[0].type, SACC_FORMAT_LINEAR};
        SaccMambaBlockArgs a{};
        const std::string why = check_block(*p, in_desc, &o, a);
        if (!why.empty()) fail(p, why);
        if (sacc_mamba_block_workspace(&a, bytes) != SACC_OK) fail(p, sacc_last_error());
    });
}

int sacc_plugin_enqueue_ws(const SaccScanPlugin* p, const SaccTensorDesc* in_desc, const SaccTensorDesc* out_desc,
                           const void* const* in, void* const* out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    return plugin_guard([&] {
        if (!p || !in_desc || !out_desc || !in || !out) throw PluginError{SACC_EINVAL, "sacc_plugin_enqueue: arguments are required"};
        if (stream == nullptr || stream == cudaStreamLegacy || stream == cudaStreamPerThread)
            fail(p, "an explicit non-default stream is required");
        if (p->bound_context == 0) fail(p, "kernels are not loaded for any CUDA context");
        const Driver& d = driver();
        CUcontext of_stream{}, current{};
        unsigned long long id = 0;
        if (!d.stream_ctx || !d.get_current || !d.ctx_id ||
            d.stream_ctx(reinterpret_cast<CUstream>(stream), &of_stream) != CUDA_SUCCESS ||
            d.get_current(&current) != CUDA_SUCCESS || of_stream == nullptr || of_stream != current ||
            d.ctx_id(of_stream, &id) != CUDA_SUCCESS)
            fail(p, "the stream does not belong to the current CUDA context");
        if (id != p->bound_context) fail(p, "the kernels were loaded in another CUDA context");
        if (p->blockish()) {
            SaccCrossScanBlockArgs c{};
            SaccMambaBlockArgs& a = c.block;
            const std::string why = p->op == Op::level ? check_level(*p, in_desc, out_desc, c) : check_block(*p, in_desc, out_desc, a);
            if (!why.empty()) fail(p, why);
            a.x = in[0];
            a.w_in = in[1];
            a.conv_w = static_cast<const float*>(in[2]);
            a.conv_b = static_cast<const float*>(in[3]);
            a.w_x = in[4];
            a.w_dt = in[5];
            a.dt_bias = static_cast<const float*>(in[6]);
            a.a = static_cast<const float*>(in[7]);
            a.d = static_cast<const float*>(in[8]);
            a.w_out = in[9];
            a.out = out[0];
            int rc;
            if (p->op == Op::level) {
                c.x = static_cast<const float*>(in[0]);
                c.out = static_cast<float*>(out[0]);
                a.x = nullptr;
                a.out = nullptr;
                rc = sacc_cross_scan_block_forward(&c, workspace, workspace_bytes, stream);
            } else {
                rc = sacc_mamba_block_forward(&a, workspace, workspace_bytes, stream);
            }
            if (rc != SACC_OK) fail(p, sacc_last_error(), rc);
            return;
        }
        SaccScanShape scan{};
        SaccCrossScanShape cross{};
        const std::string why = check(*p, in_desc, out_desc, scan, cross);
        if (!why.empty()) fail(p, why);
        auto* status = static_cast<SaccScanStatus*>(out[1]);
        int rc = SACC_OK;
        switch (p->op) {
        case Op::scan: {
            const auto* d = p->has_d ? static_cast<const float*>(in[5]) : nullptr;
            if (p->half) {
                const SaccScanInputsF16 ins{static_cast<const std::uint16_t*>(in[0]), static_cast<const std::uint16_t*>(in[1]),
                                            static_cast<const float*>(in[2]), static_cast<const std::uint16_t*>(in[3]),
                                            static_cast<const std::uint16_t*>(in[4]), d};
                rc = sacc_selective_scan_f16(&scan, &ins, static_cast<std::uint16_t*>(out[0]), status, stream);
            } else {
                const SaccScanInputs ins{static_cast<const float*>(in[0]), static_cast<const float*>(in[1]),
                                         static_cast<const float*>(in[2]), static_cast<const float*>(in[3]),
                                         static_cast<const float*>(in[4]), d};
                rc = sacc_selective_scan_f32(&scan, &ins, static_cast<float*>(out[0]), status, stream);
            }
            break;
        }
        case Op::expand:
            rc = sacc_cross_scan_expand_f32(&cross, static_cast<const float*>(in[0]), static_cast<float*>(out[0]), status, stream);
            break;
        case Op::merge:
            rc = sacc_cross_scan_merge_f32(&cross, static_cast<const float*>(in[0]), static_cast<float*>(out[0]), status, stream);
            break;
        }
        if (rc != SACC_OK) fail(p, sacc_last_error(), rc);
    });
}

} // extern "C"
