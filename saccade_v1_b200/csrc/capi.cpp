// capi.cpp -- extern "C" entry points of libsacc_scan.so (include/sacc_scan.h).
//
// Host validation restates the reference's selective_scan_cuda host side
// (cuda/selective_scan.cu:198-311) with the same diagnostics, but reports
// them as return codes plus a thread-local message instead of exceptions.
// A rejected call enqueues nothing, so the caller's status words stay as they
// were.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/sacc_shard.h"
#include "internal.h"

#ifndef SACC_BUILD_FLAGS
#define SACC_BUILD_FLAGS "unknown"
#endif

namespace sacc {
namespace {

thread_local std::string g_error;

int set_error(int code, const std::string& what) {
    g_error = what;
    return code;
}

struct Reject {
    std::string what;
};

[[noreturn]] void reject(const char* api, const std::string& what) { throw Reject{std::string(api) + ": " + what}; }

std::size_t elements(const char* api, std::initializer_list<std::uint64_t> dims, const char* tensor) {
    std::size_t product = 1;
    for (const auto dim : dims) {
        if (dim != 0 && product > kMaxElements / dim) reject(api, std::string(tensor) + " element count exceeds int32 capacity");
        product *= static_cast<std::size_t>(dim);
    }
    return product;
}

void require_stream(const char* api, cudaStream_t stream) {
    if (stream == nullptr || stream == cudaStreamLegacy || stream == cudaStreamPerThread)
        reject(api, "an explicit non-default stream is required");
}

struct Region {
    const void* data;
    std::size_t bytes;
    const char* name;
    std::size_t align = alignof(float); // element alignment the kernels need
};

void require_pointer(const char* api, const Region& r, std::size_t align = 0) {
    if (align == 0) align = r.align;
    if (r.bytes == 0) return;
    if (r.data == nullptr) reject(api, std::string(r.name) + " is null");
    if (reinterpret_cast<std::uintptr_t>(r.data) % align != 0)
        reject(api, std::string(r.name) + " is not " + std::to_string(align) + "-byte aligned");
}

bool overlaps(const Region& a, const Region& b) {
    if (a.bytes == 0 || b.bytes == 0) return false;
    const auto a0 = reinterpret_cast<std::uintptr_t>(a.data), b0 = reinterpret_cast<std::uintptr_t>(b.data);
    return a0 < b0 + b.bytes && b0 < a0 + a.bytes;
}

// Outputs (output tensor, status) must not overlap inputs or each other
// (reference cuda/selective_scan.cu:227-236).
void require_regions(const char* api, std::initializer_list<Region> inputs, const Region& out, const Region& status) {
    for (const auto& r : inputs) require_pointer(api, r);
    require_pointer(api, out);
    require_pointer(api, status);
    for (const auto& r : inputs) {
        if (overlaps(out, r)) reject(api, std::string(out.name) + " overlaps " + r.name);
        if (overlaps(status, r)) reject(api, std::string("status overlaps ") + r.name);
    }
    if (overlaps(status, out)) reject(api, std::string("status overlaps ") + out.name);
}

struct CudaFail {
    std::string what;
};
void ck(cudaError_t e, const char* call) {
    if (e != cudaSuccess) throw CudaFail{std::string(call) + ": " + cudaGetErrorString(e)};
}
#define CK(call) ck((call), #call)

// SM count of the current device, cached per device ordinal.
int sm_count() {
    static std::mutex mu;
    static int cached[64] = {0};
    int dev = 0;
    CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) {
        int n = 0;
        CK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        return n;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == 0) CK(cudaDeviceGetAttribute(&cached[dev], cudaDevAttrMultiProcessorCount, dev));
    return cached[dev];
}

template <typename F>
int guarded(F&& body) {
    try {
        body();
        g_error.clear();
        return SACC_OK;
    } catch (const Reject& r) {
        return set_error(SACC_EINVAL, r.what);
    } catch (const CudaFail& f) {
        return set_error(SACC_ECUDA, f.what);
    } catch (const std::exception& e) {
        return set_error(SACC_ECUDA, e.what());
    }
}

std::size_t dtype_bytes(int dtype) { return dtype == SACC_DTYPE_F32 ? 4 : 2; }

// Host side of the reference ABI (cuda/selective_scan.cu:198-311): FP32
// activations, or FP16 ones (u, delta, B, C, y) with `half`.
void reference_scan(const char* api, const SaccScanShape& s, const void* u, const void* delta, const float* a, const void* b,
                    const void* c, const float* d, void* y, SaccScanStatus* status, cudaStream_t stream, bool half) {
    require_stream(api, stream);
    if (s.batch == 0 || s.channels == 0) reject(api, "batch and channels must be positive");
    if (s.state == 0 || s.state > 32 || (s.state & (s.state - 1)) != 0)
        reject(api, "state " + std::to_string(s.state) + " must be a power of two in [1, 32]");
    if (s.a_rows != 1 && s.a_rows != s.channels) reject(api, "A rows must be 1 or channels");
    if (s.c_width != 1 && s.c_width != s.state) reject(api, "C width must be 1 or state");
    const auto ud = elements(api, {s.batch, s.length, s.channels}, "u/delta/y");
    const auto bn = elements(api, {s.batch, s.length, s.state}, "B");
    const auto cn = elements(api, {s.batch, s.length, s.c_width}, "C");
    const auto an = elements(api, {s.a_rows, s.state}, "A");
    const std::size_t dn = s.has_d ? static_cast<std::size_t>(s.channels) : 0;
    constexpr auto f = sizeof(float);
    const std::size_t e = half ? 2 : 4; // activation element bytes
    require_regions(api,
                    {{u, ud * e, "u", e}, {delta, ud * e, "delta", e}, {a, an * f, "A"}, {b, bn * e, "B", e},
                     {c, cn * e, "C", e}, {d, dn * f, "D"}},
                    {y, ud * e, "y", e}, {status, sizeof(SaccScanStatus), "status"});
    const int sms = sm_count();
    CK(cudaMemsetAsync(status, 0, sizeof(SaccScanStatus), stream));
    const int h = half ? 1 : 0;
    CheckList list{{{u, ud, SACC_SCAN_NONFINITE_U, h},
                    {delta, ud, SACC_SCAN_NONFINITE_DELTA, h},
                    {a, an, SACC_SCAN_NONFINITE_A, 0},
                    {b, bn, SACC_SCAN_NONFINITE_B, h},
                    {c, cn, SACC_SCAN_NONFINITE_C, h},
                    {d, dn, SACC_SCAN_NONFINITE_D, 0}},
                   6};
    // memset, check, scan, finalize: the reference's four operations per call
    // (cuda/selective_scan.cu:298-310); the scan overlaps the check.
    CK(launch_check(list, status, sms, stream));
    if (s.length > 0) {
        ScanF32Launch p{u, delta, a, b, c, d, y, s.batch, s.length, s.channels,
                        s.batch * s.channels, static_cast<unsigned>(s.state), s.a_rows == 1, s.c_width != 1,
                        s.has_d != 0, half};
        CK(launch_scan_f32(p, status, sms, stream));
    }
    CK(launch_finalize(y, ud, status, sms, stream, half));
}

// ---- frame protocol / producer argument checks

void require_frame_control(const char* api, const SaccScanFrameControl* c) {
    require_pointer(api, {c, sizeof(SaccScanFrameControl), "control"}, alignof(SaccScanFrameControl));
}

void require_status_list(const char* api, const SaccScanStatusList* list) {
    if (list == nullptr) reject(api, "status list is required");
    if (list->count > SACC_FRAME_MAX_STATUSES) reject(api, "too many statuses"); // reference cuda/scan_frame.cu:169
    for (unsigned i = 0; i < list->count; ++i)
        require_pointer(api, {list->status[i], sizeof(SaccScanStatus), "status"}, alignof(SaccScanStatus));
}

void require_records(const char* api, const SaccScanFrameRecord* records, int64_t capacity) {
    if (records == nullptr || capacity <= 0) return; // no record is written
    if (static_cast<std::uint64_t>(capacity) > SIZE_MAX / sizeof(SaccScanFrameRecord)) reject(api, "record capacity overflows");
    require_pointer(api, {records, static_cast<std::size_t>(capacity) * sizeof(SaccScanFrameRecord), "records"},
                    alignof(SaccScanFrameRecord));
}

void require_payload(const char* api, const float* payload, std::size_t count, const float* results, const int64_t* result_frames) {
    if (count > SIZE_MAX / (2 * sizeof(float))) reject(api, "payload count overflows");
    const Region in{payload, count * sizeof(float), "payload"}, out{results, 2 * count * sizeof(float), "results"};
    require_pointer(api, in);
    require_pointer(api, out);
    require_pointer(api, {result_frames, 2 * sizeof(int64_t), "result_frames"}, alignof(int64_t));
    if (overlaps(in, out)) reject(api, "results overlap payload");
}

// cuMemGetAddressRange through the runtime's driver entry point (no link
// against libcuda).
using AddressRangeFn = int (*)(unsigned long long* base, std::size_t* size, unsigned long long ptr);
AddressRangeFn address_range_fn() {
    static AddressRangeFn fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 12000, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<AddressRangeFn>(nullptr);
        return reinterpret_cast<AddressRangeFn>(ptr);
    }();
    return fn;
}

// reference cuda/model_producer.cu:75-105: non-null, aligned, device memory of
// the current device, inside one queryable allocation.
void require_device_range(const char* api, const Region& r, int device) {
    const auto start = reinterpret_cast<std::uintptr_t>(r.data);
    if (r.data == nullptr || start % alignof(float) != 0 || r.bytes > UINTPTR_MAX - start)
        reject(api, "null, unaligned or overflowing model producer pointer");
    cudaPointerAttributes attr{};
    const cudaError_t e = cudaPointerGetAttributes(&attr, r.data);
    if (e == cudaErrorInvalidValue) {
        (void)cudaGetLastError();
        reject(api, "model producer pointer must be device memory");
    }
    CK(e);
    if (attr.type != cudaMemoryTypeDevice || attr.device != device)
        reject(api, "model producer pointer must be on the current CUDA device");
    const AddressRangeFn range = address_range_fn();
    if (range == nullptr) throw CudaFail{"cuMemGetAddressRange is unavailable"};
    unsigned long long base = 0;
    std::size_t bytes = 0;
    const int rc = range(&base, &bytes, static_cast<unsigned long long>(start));
    if (rc != 0) reject(api, "model producer requires a queryable device allocation extent");
    if (start < base || r.bytes > base + bytes - start) reject(api, "model producer range exceeds its device allocation");
}

} // namespace
} // namespace sacc

using namespace sacc;

extern "C" {

const char* sacc_last_error(void) { return g_error.c_str(); }

const char* sacc_scan_identity(void) {
    static const std::string id = [] {
        std::string s = "library=libsacc_scan\nnvcc=" + std::to_string(__CUDACC_VER_MAJOR__) + "." +
                        std::to_string(__CUDACC_VER_MINOR__) + "." + std::to_string(__CUDACC_VER_BUILD__) +
                        "\nflags=" SACC_BUILD_FLAGS "\narch=sm_100a\n";
        int rt = 0;
        if (cudaRuntimeGetVersion(&rt) == cudaSuccess) s += "cudart=" + std::to_string(rt) + "\n";
        return s;
    }();
    return id.c_str();
}

int sacc_scan_load_kernels(char* report, size_t report_bytes) {
    return guarded([&] {
        std::string text;
        CK(load_scan_f32_kernels(text));
        CK(load_cross_kernels(text));
        CK(load_scan_ex_kernels(text));
        CK(load_scan_step_kernels(text));
        CK(load_gemm_kernels(text));
        CK(load_block_kernels(text));
        CK(load_cross_block_kernels(text));
        CK(load_frame_kernels(text));
        CK(load_producer_kernels(text));
        (void)sm_count();
        if (report && report_bytes) {
            std::snprintf(report, report_bytes, "%s", text.c_str());
        }
    });
}

// reference cuda/selective_scan.cu:270-311
int sacc_selective_scan_f32(const SaccScanShape* shape, const SaccScanInputs* in, float* y, SaccScanStatus* status,
                            cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "selective_scan_cuda";
        if (shape == nullptr || in == nullptr) reject(api, "shape and inputs are required");
        reference_scan(api, *shape, in->u, in->delta, in->a, in->b, in->c, in->d, y, status, stream, false);
    });
}

// The reference ABI with FP16 activations (plugin SelectiveScan v3).
int sacc_selective_scan_f16(const SaccScanShape* shape, const SaccScanInputsF16* in, uint16_t* y, SaccScanStatus* status,
                            cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "selective_scan_f16";
        if (shape == nullptr || in == nullptr) reject(api, "shape and inputs are required");
        reference_scan(api, *shape, in->u, in->delta, in->a, in->b, in->c, in->d, y, status, stream, true);
    });
}

static std::size_t cross_total(const char* api, const SaccCrossScanShape& s) {
    if (s.batch == 0 || s.channels == 0 || s.height == 0 || s.width == 0) reject(api, "dimensions must be positive");
    return elements(api, {4, s.batch, s.height, s.width, s.channels}, "tokens");
}

// reference cuda/selective_scan.cu:313-328
int sacc_cross_scan_expand_f32(const SaccCrossScanShape* shape, const float* x, float* tokens, SaccScanStatus* status,
                               cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "cross_scan_expand_cuda";
        if (shape == nullptr) reject(api, "shape is required");
        require_stream(api, stream);
        const auto total = cross_total(api, *shape);
        require_regions(api, {{x, total / 4 * sizeof(float), "x"}}, {tokens, total * sizeof(float), "tokens"},
                        {status, sizeof(SaccScanStatus), "status"});
        const int sms = sm_count();
        CK(cudaMemsetAsync(status, 0, sizeof(SaccScanStatus), stream));
        const CheckList list{{{x, total / 4, SACC_CROSS_SCAN_NONFINITE_INPUT}}, 1};
        CK(launch_check(list, status, sms, stream));
        const CrossLaunch p{shape->batch, shape->channels, shape->height, shape->width};
        CK(launch_cross_expand(p, x, tokens, sms, stream));
        CK(launch_finalize(tokens, total, status, sms, stream));
    });
}

// reference cuda/selective_scan.cu:330-345
int sacc_cross_scan_merge_f32(const SaccCrossScanShape* shape, const float* y, float* out, SaccScanStatus* status,
                              cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "cross_scan_merge_cuda";
        if (shape == nullptr) reject(api, "shape is required");
        require_stream(api, stream);
        const auto total = cross_total(api, *shape);
        require_regions(api, {{y, total * sizeof(float), "y"}}, {out, total / 4 * sizeof(float), "out"},
                        {status, sizeof(SaccScanStatus), "status"});
        const int sms = sm_count();
        CK(cudaMemsetAsync(status, 0, sizeof(SaccScanStatus), stream));
        const CheckList list{{{y, total, SACC_CROSS_SCAN_NONFINITE_INPUT}}, 1};
        CK(launch_check(list, status, sms, stream));
        const CrossLaunch p{shape->batch, shape->channels, shape->height, shape->width};
        CK(launch_cross_merge(p, y, out, sms, stream));
        CK(launch_finalize(out, total / 4, status, sms, stream));
    });
}

int sacc_scan_fault(uint32_t* out, int clear) {
    return guarded([&] {
        if (out == nullptr) reject("sacc_scan_fault", "out is required");
        unsigned scan = 0, step = 0, gemm = 0, block = 0;
        CK(read_bulk_fault(&scan, clear != 0));
        CK(read_step_fault(&step, clear != 0));
        CK(read_gemm_fault(&gemm, clear != 0));
        CK(read_block_fault(&block, clear != 0));
        *out = (scan || step || block ? 1u : 0u) | (gemm ? 2u : 0u);
    });
}

int sacc_scan_wait_probe(uint32_t limit, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "sacc_scan_wait_probe";
        require_stream(api, stream);
        if (limit == 0 || limit > (1u << 20)) reject(api, "limit must be in [1, 2^20] polls");
        CK(launch_wait_probe(limit, stream));
    });
}

// Host checks of one extended scan (throws Reject; enqueues nothing).
static void validate_scan_ex(const char* api, const SaccScanExArgs& a, cudaStream_t stream) {
    require_stream(api, stream);
    if (a.dtype != SACC_DTYPE_F32 && a.dtype != SACC_DTYPE_BF16 && a.dtype != SACC_DTYPE_F16)
        reject(api, "dtype must be f32, bf16 or f16");
    if (a.layout != SACC_LAYOUT_BLD && a.layout != SACC_LAYOUT_BDL) reject(api, "layout must be BLD or BDL");
    if (a.batch == 0 || a.channels == 0) reject(api, "batch and channels must be positive");
    if (a.state == 0 || a.state > 32 || (a.state & (a.state - 1)) != 0)
        reject(api, "state " + std::to_string(a.state) + " must be a power of two in [1, 32]");
    if (a.groups == 0 || a.channels % a.groups != 0) reject(api, "groups must divide channels");
    if (a.a_rows != 1 && a.a_rows != a.channels) reject(api, "A rows must be 1 or channels");
    if (a.c_width != 1 && a.c_width != a.state) reject(api, "C width must be 1 or state");
    std::uint64_t nseq = a.batch;
    if (a.cu_seqlens) {
        if (a.batch != 1) reject(api, "cu_seqlens needs batch 1");
        if (a.nseq <= 0) reject(api, "nseq must be positive with cu_seqlens");
        nseq = static_cast<std::uint64_t>(a.nseq);
    }
    // Kernels index in 64 bits; the 32-bit limit here is per tensor, as in
    // the reference ABI, so the int32 sequence offsets stay valid.
    const auto ud = elements(api, {a.batch, a.length, a.channels}, "u/delta/y");
    const auto bn = elements(api, {a.batch, a.length, a.groups, a.state}, "B");
    const auto cn = elements(api, {a.batch, a.length, a.groups, a.c_width}, "C");
    const auto an = elements(api, {a.a_rows, a.state}, "A");
    const auto hn = elements(api, {nseq, a.channels, a.state}, "state");
    const std::size_t e = dtype_bytes(a.dtype), f = sizeof(float);
    const std::size_t dn = a.d ? a.channels : 0, bias_n = a.delta_bias ? a.channels : 0;
    const std::size_t align = a.dtype == SACC_DTYPE_F32 ? 4 : 2;
    for (const Region& r : {Region{a.u, ud * e, "u"}, Region{a.delta, ud * e, "delta"}, Region{a.b, bn * e, "B"},
                            Region{a.c, cn * e, "C"}, Region{a.z, a.z ? ud * e : 0, "z"}, Region{a.y, ud * e, "y"}})
        require_pointer(api, r, align);
    for (const Region& r : {Region{a.a, an * f, "A"}, Region{a.d, dn * f, "D"}, Region{a.delta_bias, bias_n * f, "delta_bias"},
                            Region{a.h0, a.h0 ? hn * f : 0, "h0"}, Region{a.h_final, a.h_final ? hn * f : 0, "h_final"},
                            Region{a.cu_seqlens, a.cu_seqlens ? (nseq + 1) * sizeof(std::int32_t) : 0, "cu_seqlens"}})
        require_pointer(api, r);
    if (a.u == nullptr || a.delta == nullptr || a.a == nullptr || a.y == nullptr) reject(api, "u, delta, A and y are required");
    if (a.length > 0 && (a.b == nullptr || a.c == nullptr)) reject(api, "B and C are required");
    const Region yr{a.y, ud * e, "y"};
    for (const Region& r : {Region{a.u, ud * e, "u"}, Region{a.delta, ud * e, "delta"}, Region{a.b, bn * e, "B"},
                            Region{a.c, cn * e, "C"}, Region{a.z, a.z ? ud * e : 0, "z"}})
        if (overlaps(yr, r)) reject(api, std::string("y overlaps ") + r.name);
    if (a.h_final) {
        const Region hr{a.h_final, hn * f, "h_final"};
        if (overlaps(hr, yr)) reject(api, "h_final overlaps y");
    }
}

int sacc_selective_scan_ex(const SaccScanExArgs* args, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "selective_scan_ex";
        if (args == nullptr) reject(api, "args are required");
        validate_scan_ex(api, *args, stream);
        CK(launch_scan_ex(*args, sm_count(), stream));
    });
}

int sacc_selective_scan_step(const SaccScanStepArgs* args, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "selective_scan_step";
        if (args == nullptr) reject(api, "args are required");
        const SaccScanStepArgs& a = *args;
        require_stream(api, stream);
        if (a.dtype != SACC_DTYPE_F32 && a.dtype != SACC_DTYPE_BF16 && a.dtype != SACC_DTYPE_F16)
            reject(api, "dtype must be f32, bf16 or f16");
        if (a.channels == 0) reject(api, "channels must be positive");
        if (a.state == 0 || a.state > 32 || (a.state & (a.state - 1)) != 0)
            reject(api, "state " + std::to_string(a.state) + " must be a power of two in [1, 32]");
        if (a.groups == 0 || a.channels % a.groups != 0) reject(api, "groups must divide channels");
        if (a.a_rows != 1 && a.a_rows != a.channels) reject(api, "A rows must be 1 or channels");
        if (a.c_width != 1 && a.c_width != a.state) reject(api, "C width must be 1 or state");
        const std::uint64_t slots = a.slot ? a.slots : a.nseq;
        if (!a.slot && a.slots != 0 && a.slots != a.nseq) reject(api, "slots must equal nseq without a slot map");
        const auto ud = elements(api, {a.nseq, a.channels}, "u/delta/y");
        const auto bn = elements(api, {a.nseq, a.groups, a.state}, "B");
        const auto cn = elements(api, {a.nseq, a.groups, a.c_width}, "C");
        const auto an = elements(api, {a.a_rows, a.state}, "A");
        const auto sn = elements(api, {slots, a.channels, a.state}, "state");
        const std::size_t e = dtype_bytes(a.dtype), f = sizeof(float), align = a.dtype == SACC_DTYPE_F32 ? 4 : 2;
        for (const Region& r : {Region{a.u, ud * e, "u"}, Region{a.delta, ud * e, "delta"}, Region{a.b, bn * e, "B"},
                                Region{a.c, cn * e, "C"}, Region{a.z, a.z ? ud * e : 0, "z"}, Region{a.y, ud * e, "y"}})
            require_pointer(api, r, align);
        for (const Region& r : {Region{a.a, an * f, "A"}, Region{a.d, a.d ? a.channels * f : 0, "D"},
                                Region{a.delta_bias, a.delta_bias ? a.channels * f : 0, "delta_bias"},
                                Region{a.slot, a.slot ? a.nseq * sizeof(std::int32_t) : 0, "slot"}})
            require_pointer(api, r);
        require_pointer(api, Region{a.state_io, sn * f, "state"}, a.state >= 4 ? 16 : 4);
        if (ud == 0) return;
        if (a.u == nullptr || a.delta == nullptr || a.a == nullptr || a.y == nullptr || a.b == nullptr ||
            a.c == nullptr || a.state_io == nullptr)
            reject(api, "u, delta, A, B, C, state and y are required");
        const Region yr{a.y, ud * e, "y"}, sr{a.state_io, sn * f, "state"};
        for (const Region& r : {Region{a.u, ud * e, "u"}, Region{a.delta, ud * e, "delta"}, Region{a.b, bn * e, "B"},
                                Region{a.c, cn * e, "C"}, Region{a.z, a.z ? ud * e : 0, "z"}}) {
            if (overlaps(yr, r)) reject(api, std::string("y overlaps ") + r.name);
            if (overlaps(sr, r)) reject(api, std::string("state overlaps ") + r.name);
        }
        if (overlaps(sr, yr)) reject(api, "state overlaps y");
        SaccScanStepArgs fixed = a;
        fixed.slots = slots;
        CK(launch_scan_step(fixed, stream));
    });
}

int sacc_gemm(const SaccGemmArgs* args, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "gemm";
        if (args == nullptr) reject(api, "args are required");
        const SaccGemmArgs& a = *args;
        require_stream(api, stream);
        if (a.in_dtype != SACC_DTYPE_BF16 && a.in_dtype != SACC_DTYPE_F16) reject(api, "in_dtype must be bf16 or f16");
        if (a.out_dtype != SACC_DTYPE_F32 && a.out_dtype != SACC_DTYPE_BF16 && a.out_dtype != SACC_DTYPE_F16)
            reject(api, "out_dtype must be f32, bf16 or f16");
        if (a.m == 0 || a.n == 0 || a.k == 0) reject(api, "m, n and k must be positive");
        if (a.lda < a.k || a.ldb < a.k || a.ldc < a.n || (a.residual && a.ldr < a.n)) reject(api, "leading dimensions too small");
        if (a.lda % 8 != 0 || a.ldb % 8 != 0) reject(api, "lda and ldb must be multiples of 8 (16-byte rows)");
        if (a.m > 0x7fffffffull || a.n > 0x7fffffffull || a.k > 0x7fffffffull) reject(api, "dimensions exceed int32");
        const std::size_t eo = dtype_bytes(a.out_dtype);
        const Region ar{a.a, ((a.m - 1) * a.lda + a.k) * 2, "A"}, br{a.b, ((a.n - 1) * a.ldb + a.k) * 2, "B"};
        const Region cr{a.c, ((a.m - 1) * a.ldc + a.n) * eo, "C"};
        require_pointer(api, ar, 16);
        require_pointer(api, br, 16);
        require_pointer(api, cr, eo);
        require_pointer(api, Region{a.bias, a.bias ? a.n * sizeof(float) : 0, "bias"});
        require_pointer(api, Region{a.row_scale, a.row_scale ? a.m * sizeof(float) : 0, "row_scale"});
        const Region rr{a.residual, a.residual ? ((a.m - 1) * a.ldr + a.n) * eo : 0, "residual"};
        require_pointer(api, rr, eo);
        if (overlaps(cr, ar) || overlaps(cr, br)) reject(api, "C overlaps an operand");
        CK(launch_gemm(a, stream));
    });
}

static void check_block_shape(const char* api, const SaccMambaBlockArgs& a) {
    if (a.dtype != SACC_DTYPE_BF16 && a.dtype != SACC_DTYPE_F16) reject(api, "dtype must be bf16 or f16");
    if (a.batch == 0 || a.length == 0) reject(api, "batch and length must be positive");
    if (a.d_conv != 4) reject(api, "d_conv must be 4");
    if (a.d_state != 16) reject(api, "d_state must be 16");
    if (a.d_inner == 0 || a.d_inner % 128 != 0 || a.d_model == 0 || a.d_model % 128 != 0)
        reject(api, "d_inner and d_model must be positive multiples of 128");
    if (a.dt_rank == 0 || a.dt_rank % 8 != 0) reject(api, "dt_rank must be a positive multiple of 8");
    if (a.c_width != 0 && a.c_width != 1 && static_cast<std::uint64_t>(a.c_width) != a.d_state)
        reject(api, "c_width must be 1 or d_state");
    if (!(a.eps > 0.0f) && a.norm_w) reject(api, "eps must be positive");
    const std::uint64_t M = a.batch * a.length;
    if (M > 0x7fffffffull) reject(api, "batch * length exceeds int32");
    if (a.length * a.d_inner > kMaxElements) reject(api, "length * d_inner exceeds int32 capacity");
}

static void check_block(const char* api, const SaccMambaBlockArgs& a) {
    check_block_shape(api, a);
    const std::uint64_t M = a.batch * a.length;
    const std::uint64_t D = a.d_inner, dm = a.d_model, R = a.dt_rank, N = a.d_state;
    for (const Region& r : {Region{a.x, M * dm * 2, "x"}, Region{a.w_in, 2 * D * dm * 2, "w_in"},
                            Region{a.w_x, (R + N + (a.c_width == 1 ? 1 : N)) * D * 2, "w_x"}, Region{a.w_dt, D * R * 2, "w_dt"},
                            Region{a.w_out, dm * D * 2, "w_out"}, Region{a.out, M * dm * 2, "out"}})
        require_pointer(api, r, 16);
    for (const Region& r : {Region{a.conv_w, D * 4 * 4, "conv_w"}, Region{a.a, D * N * 4, "A"}})
        require_pointer(api, r);
    for (const Region& r : {Region{a.norm_w, a.norm_w ? dm * 4 : 0, "norm_w"}, Region{a.conv_b, a.conv_b ? D * 4 : 0, "conv_b"},
                            Region{a.dt_bias, a.dt_bias ? D * 4 : 0, "dt_bias"}, Region{a.d, a.d ? D * 4 : 0, "D"}})
        require_pointer(api, r);
    if (overlaps(Region{a.out, M * dm * 2, "out"}, Region{a.x, M * dm * 2, "x"})) reject(api, "out overlaps x");
}

int sacc_mamba_block_workspace(const SaccMambaBlockArgs* args, size_t* bytes) {
    return guarded([&] {
        if (args == nullptr || bytes == nullptr) reject("mamba_block", "args and bytes are required");
        check_block_shape("mamba_block", *args);
        *bytes = mamba_block_workspace(*args);
    });
}

int sacc_mamba_block_forward(const SaccMambaBlockArgs* args, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "mamba_block";
        if (args == nullptr) reject(api, "args are required");
        require_stream(api, stream);
        check_block(api, *args);
        const std::size_t need = mamba_block_workspace(*args);
        if (workspace_bytes < need) reject(api, "workspace holds " + std::to_string(workspace_bytes) + " bytes, needs " +
                                                    std::to_string(need));
        require_pointer(api, Region{workspace, need, "workspace"}, 256);
        CK(launch_mamba_block(*args, workspace, stream));
    });
}

int sacc_mamba_block_forward_noalloc(const SaccMambaBlockArgs* args, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "mamba_block_noalloc";
        if (args == nullptr) reject(api, "args are required");
        require_stream(api, stream);
        check_block(api, *args);
        const std::size_t need = mamba_block_workspace(*args);
        if (need > kNoAllocScratchBytes)
            reject(api, "needs " + std::to_string(need) + " bytes of scratch, more than the static maximum of " +
                            std::to_string(kNoAllocScratchBytes) + "; use sacc_mamba_block_forward with a workspace");
        CK(launch_mamba_block_noalloc(*args, stream));
    });
}

// One Cross-Scan head level (reference src/head_trt_network.cpp:200-232):
// the block's shape rules with 4 x images sequences of height x width tokens,
// FP32 maps for x and out.
static void check_cross_block(const char* api, const SaccCrossScanBlockArgs& c) {
    const SaccMambaBlockArgs& a = c.block;
    if (c.height == 0 || c.width == 0) reject(api, "height and width must be positive");
    if (c.height > 0xffffffffull || c.width > 0xffffffffull || a.length != c.height * c.width)
        reject(api, "block.length must be height * width");
    if (a.batch == 0 || a.batch > 65535) reject(api, "batch (images) must be in [1, 65535]");
    SaccMambaBlockArgs v = a;
    v.batch = 4 * a.batch; // the four directions' sequences
    check_block_shape(api, v);
    const std::uint64_t P = a.batch * a.length, D = a.d_inner, dm = a.d_model, R = a.dt_rank, N = a.d_state;
    const Region x{c.x, P * dm * 4, "x"}, out{c.out, P * dm * 4, "out"};
    require_pointer(api, x, 16);
    require_pointer(api, out, 16);
    for (const Region& r : {Region{a.w_in, 2 * D * dm * 2, "w_in"}, Region{a.w_x, (R + N + (a.c_width == 1 ? 1 : N)) * D * 2, "w_x"},
                            Region{a.w_dt, D * R * 2, "w_dt"}, Region{a.w_out, dm * D * 2, "w_out"}})
        require_pointer(api, r, 16);
    for (const Region& r : {Region{a.conv_w, D * 4 * 4, "conv_w"}, Region{a.a, D * N * 4, "A"}})
        require_pointer(api, r);
    for (const Region& r : {Region{a.norm_w, a.norm_w ? dm * 4 : 0, "norm_w"}, Region{a.conv_b, a.conv_b ? D * 4 : 0, "conv_b"},
                            Region{a.dt_bias, a.dt_bias ? D * 4 : 0, "dt_bias"}, Region{a.d, a.d ? D * 4 : 0, "D"}})
        require_pointer(api, r);
    if (overlaps(out, x)) reject(api, "out overlaps x");
}

int sacc_cross_scan_block_workspace(const SaccCrossScanBlockArgs* args, size_t* bytes) {
    return guarded([&] {
        constexpr const char* api = "cross_scan_block";
        if (args == nullptr || bytes == nullptr) reject(api, "args and bytes are required");
        const SaccCrossScanBlockArgs& c = *args;
        if (c.height == 0 || c.width == 0 || c.height > 0xffffffffull || c.width > 0xffffffffull ||
            c.block.length != c.height * c.width)
            reject(api, "block.length must be height * width, both positive");
        if (c.block.batch == 0 || c.block.batch > 65535) reject(api, "batch (images) must be in [1, 65535]");
        SaccMambaBlockArgs v = c.block;
        v.batch = 4 * c.block.batch;
        check_block_shape(api, v);
        *bytes = cross_block_workspace(c);
    });
}

int sacc_cross_scan_block_forward(const SaccCrossScanBlockArgs* args, void* workspace, size_t workspace_bytes,
                                  cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "cross_scan_block";
        if (args == nullptr) reject(api, "args are required");
        require_stream(api, stream);
        check_cross_block(api, *args);
        const std::size_t need = cross_block_workspace(*args);
        if (workspace_bytes < need) reject(api, "workspace holds " + std::to_string(workspace_bytes) + " bytes, needs " +
                                                    std::to_string(need));
        require_pointer(api, Region{workspace, need, "workspace"}, 256);
        CK(launch_cross_block(*args, workspace, stream));
    });
}

// ------------------------------------------------------------ frame protocol
// reference cuda/scan_frame.cu:144-209; kernels in scan_frame.cu.

int sacc_scan_frame_load_kernels(char* report, size_t report_bytes) {
    return guarded([&] {
        std::string text;
        CK(load_frame_kernels(text));
        if (report && report_bytes) std::snprintf(report, report_bytes, "%s", text.c_str());
    });
}

int sacc_scan_frame_initialize(SaccScanFrameControl* control, uint64_t epoch, int64_t* result_frames, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "scan_frame_initialize";
        require_stream(api, stream);
        require_frame_control(api, control);
        require_pointer(api, {result_frames, 2 * sizeof(int64_t), "result_frames"}, alignof(int64_t));
        CK(launch_frame_initialize(control, epoch, result_frames, stream));
    });
}

int sacc_scan_frame_begin(SaccScanFrameControl* control, uint64_t epoch, int64_t frame, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "scan_frame_begin";
        require_stream(api, stream);
        require_frame_control(api, control);
        CK(launch_frame_begin(control, epoch, frame, stream));
    });
}

int sacc_scan_frame_gate(SaccScanFrameControl* control, const SaccScanStatusList* statuses, SaccScanFrameRecord* records,
                         int64_t capacity, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "scan_frame_gate";
        require_stream(api, stream);
        require_frame_control(api, control);
        require_status_list(api, statuses);
        require_records(api, records, capacity);
        CK(launch_frame_gate(control, *statuses, records, capacity, stream));
    });
}

int sacc_scan_frame_publish(SaccScanFrameControl* control, const float* payload, size_t count, float* results,
                            int64_t* result_frames, SaccScanFrameRecord* records, int64_t capacity, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "scan_frame_publish";
        require_stream(api, stream);
        require_frame_control(api, control);
        require_payload(api, payload, count, results, result_frames);
        require_records(api, records, capacity);
        CK(launch_frame_publish(control, payload, count, results, result_frames, records, capacity, sm_count(), stream));
    });
}

int sacc_scan_frame_commit(SaccScanFrameControl* control, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "scan_frame_commit";
        require_stream(api, stream);
        require_frame_control(api, control);
        CK(launch_frame_commit(control, stream));
    });
}

int sacc_scan_frame_packet(const SaccScanFrameControl* control, unsigned char* packet, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "scan_frame_packet";
        require_stream(api, stream);
        require_frame_control(api, control);
        require_pointer(api, {packet, SACC_PACKET_BYTES, "packet"}, 1);
        CK(launch_frame_packet(control, packet, stream));
    });
}

int sacc_scan_frame_step(SaccScanFrameControl* control, uint64_t epoch, int64_t frame, const SaccScanStatusList* statuses,
                         const float* payload, size_t count, float* results, int64_t* result_frames,
                         SaccScanFrameRecord* records, int64_t capacity, unsigned char* packet, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "scan_frame_step";
        require_stream(api, stream);
        require_frame_control(api, control);
        require_status_list(api, statuses);
        require_payload(api, payload, count, results, result_frames);
        require_records(api, records, capacity);
        const FrameStep f{*statuses, payload, count, results, result_frames, records, capacity, packet, epoch, frame};
        CK(launch_frame_step(control, f, sm_count(), stream));
    });
}

int sacc_scan_frame_check_finite(const float* data, size_t count, SaccScanStatus* status, uint32_t flag, cudaStream_t stream) {
    return guarded([&] {
        constexpr const char* api = "scan_frame_check_finite";
        require_stream(api, stream);
        require_pointer(api, {data, count * sizeof(float), "data"});
        require_pointer(api, {status, sizeof(SaccScanStatus), "status"});
        if (overlaps({data, count * sizeof(float), "data"}, {status, sizeof(SaccScanStatus), "status"}))
            reject(api, "status overlaps data");
        CK(launch_frame_check_finite(data, count, status, flag, sm_count(), stream));
    });
}

int sacc_scan_frame_delay(unsigned cycles, cudaStream_t stream) {
    return guarded([&] {
        require_stream("scan_frame_delay", stream);
        CK(launch_frame_delay(cycles, stream));
    });
}

uint64_t sacc_scan_frame_digest(const float* payload, size_t count) { return payload ? frame_digest(payload, count) : 0; }

// ---------------------------------------------------- model producer status
// reference cuda/model_producer.cu:117-196; kernels in model_producer.cu.

size_t sacc_model_producer_workspace_bytes(void) { return producer_workspace_bytes(); }

int sacc_model_producer_load_kernels(char* report, size_t report_bytes) {
    return guarded([&] {
        std::string text;
        CK(load_producer_kernels(text));
        if (report && report_bytes) std::snprintf(report, report_bytes, "%s", text.c_str());
    });
}

int sacc_model_producer_cuda(const float* images, size_t image_elements, const SaccRawView* raw,
                             SaccScanStatus* const plugins[SACC_MODEL_PRODUCER_PLUGINS], SaccProducerStatus* producer,
                             void* workspace, size_t workspace_bytes, cudaStream_t stream, int profile) {
    return guarded([&] {
        constexpr const char* api = "model_producer_cuda";
        if (raw == nullptr || plugins == nullptr) reject(api, "raw view and plugin statuses are required");
        if (profile != SACC_PROFILE_T01_640X640 && profile != SACC_PROFILE_HR_1280X768) reject(api, "unknown model profile");
        // Profile shapes (include/saccade/model_profile.hpp:14-38): image
        // 3 x H x W; per level of stride 8 / 16 / 32, cls 80 x h x w, reg 4 x h x w.
        const std::size_t width = profile == SACC_PROFILE_HR_1280X768 ? 1280 : 640;
        const std::size_t height = profile == SACC_PROFILE_HR_1280X768 ? 768 : 640;
        if (image_elements != 3 * width * height || workspace_bytes < producer_workspace_bytes())
            reject(api, "incorrect model producer input/workspace capacity");
        // reference src/postprocess.cpp:71-80
        for (int level = 0; level < 3; ++level) {
            const std::size_t stride = std::size_t{8} << level, spatial = (height / stride) * (width / stride);
            if (raw->cls[level] == nullptr || raw->reg[level] == nullptr || raw->cls_elements[level] != 80 * spatial ||
                raw->reg_elements[level] != 4 * spatial)
                reject(api, "F04 requires all six fixed-shape raw tensors");
            if (reinterpret_cast<std::uintptr_t>(raw->cls[level]) % alignof(float) != 0 ||
                reinterpret_cast<std::uintptr_t>(raw->reg[level]) % alignof(float) != 0)
                reject(api, "F04 requires aligned FP32 raw tensors");
        }
        require_stream(api, stream);
        int device = -1, stream_device = -1;
        CK(cudaGetDevice(&device));
        CK(cudaStreamGetDevice(stream, &stream_device));
        if (stream_device != device) reject(api, "model producer stream belongs to another CUDA device");
        ProducerLaunch p{};
        Region regions[18]{};
        p.tensor[0] = images;
        p.count[0] = image_elements;
        for (int l = 0; l < 3; ++l) {
            p.tensor[1 + l] = raw->cls[l];
            p.count[1 + l] = raw->cls_elements[l];
            p.tensor[4 + l] = raw->reg[l];
            p.count[4 + l] = raw->reg_elements[l];
        }
        for (int i = 0; i < 7; ++i) regions[i] = {p.tensor[i], p.count[i] * sizeof(float), "model producer tensor"};
        for (unsigned i = 0; i < SACC_MODEL_PRODUCER_PLUGINS; ++i) {
            p.plugin[i] = plugins[i];
            regions[7 + i] = {plugins[i], sizeof(SaccScanStatus), "plugin status"};
        }
        regions[16] = {producer, sizeof(SaccProducerStatus), "producer"};
        regions[17] = {workspace, producer_workspace_bytes(), "workspace"};
        // reference cuda/model_producer.cu:75-110, 159-165
        for (const auto& r : regions) require_device_range(api, r, device);
        for (int i = 0; i < 18; ++i)
            for (int j = i + 1; j < 18; ++j)
                if (overlaps(regions[i], regions[j])) reject(api, "overlapping model producer buffers");
        CK(launch_model_producer(p, producer, workspace, sm_count(), stream));
    });
}

// ---- batch-sharded scan over the GPUs of one process (include/sacc_shard.h)

int sacc_shard_rows(uint64_t total, int world, int rank, uint64_t* row0, uint64_t* rows) {
    return guarded([&] {
        constexpr const char* api = "shard_rows";
        if (world <= 0 || rank < 0 || rank >= world) reject(api, "rank must be in [0, world)");
        if (row0 == nullptr || rows == nullptr) reject(api, "row0 and rows are required");
        const uint64_t base = total / static_cast<uint64_t>(world), extra = total % static_cast<uint64_t>(world);
        const uint64_t r = static_cast<uint64_t>(rank);
        *row0 = r * base + (r < extra ? r : extra);
        *rows = base + (r < extra ? 1 : 0);
    });
}

} // extern "C"

namespace {
// NCCL entry points, resolved from libnccl.so.2 on first use (a process that
// already loaded NCCL, e.g. through its framework, gets that copy).
struct Nccl {
    ncclResult_t (*comm_init_all)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    std::string why;
};

const Nccl& nccl() {
    static const Nccl lib = [] {
        Nccl n;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr) {
            n.why = std::string("NCCL is not available: ") + dlerror();
            return n;
        }
        n.comm_init_all = reinterpret_cast<decltype(n.comm_init_all)>(dlsym(h, "ncclCommInitAll"));
        n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
        n.group_start = reinterpret_cast<decltype(n.group_start)>(dlsym(h, "ncclGroupStart"));
        n.group_end = reinterpret_cast<decltype(n.group_end)>(dlsym(h, "ncclGroupEnd"));
        n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
        if (!n.comm_init_all || !n.comm_destroy || !n.all_gather || !n.group_start || !n.group_end || !n.error_string)
            n.why = "NCCL library lacks an entry point (ncclCommInitAll, ncclCommDestroy, ncclAllGather, ncclGroupStart, "
                    "ncclGroupEnd, ncclGetErrorString)";
        return n;
    }();
    return lib;
}

void nck(ncclResult_t r, const char* call) {
    if (r != ncclSuccess) throw sacc::CudaFail{std::string(call) + ": " + nccl().error_string(r)};
}

// Restores the caller's current device on every exit.
struct DeviceGuard {
    int saved = 0;
    bool ok = false;
    DeviceGuard() { ok = cudaGetDevice(&saved) == cudaSuccess; }
    ~DeviceGuard() {
        if (ok) cudaSetDevice(saved);
    }
};
} // namespace

struct SaccShardGroup {
    std::vector<int> devices;
    std::vector<ncclComm_t> comms;
};

extern "C" {

int sacc_shard_group_create(int ndev, const int* devices, SaccShardGroup** group) {
    return guarded([&] {
        constexpr const char* api = "shard_group";
        if (group == nullptr) reject(api, "group is required");
        *group = nullptr;
        int count = 0;
        CK(cudaGetDeviceCount(&count));
        if (ndev <= 0 || devices == nullptr) reject(api, "at least one device is required");
        for (int i = 0; i < ndev; ++i) {
            if (devices[i] < 0 || devices[i] >= count) reject(api, "device " + std::to_string(devices[i]) + " does not exist");
            for (int j = 0; j < i; ++j)
                if (devices[j] == devices[i]) reject(api, "device " + std::to_string(devices[i]) + " is listed twice");
        }
        const Nccl& n = nccl();
        if (!n.why.empty()) throw CudaFail{std::string(api) + ": " + n.why};
        DeviceGuard keep;
        auto* g = new SaccShardGroup{std::vector<int>(devices, devices + ndev), std::vector<ncclComm_t>(ndev, nullptr)};
        const ncclResult_t r = n.comm_init_all(g->comms.data(), ndev, devices);
        if (r != ncclSuccess) {
            delete g;
            nck(r, "ncclCommInitAll");
        }
        *group = g;
    });
}

int sacc_shard_group_destroy(SaccShardGroup* group) {
    return guarded([&] {
        if (group == nullptr) return;
        DeviceGuard keep;
        std::string first_error;
        for (ncclComm_t c : group->comms) {
            const ncclResult_t r = c ? nccl().comm_destroy(c) : ncclSuccess;
            if (r != ncclSuccess && first_error.empty()) first_error = nccl().error_string(r);
        }
        delete group;
        if (!first_error.empty()) throw CudaFail{std::string("ncclCommDestroy: ") + first_error};
    });
}

int sacc_scan_sharded_forward(SaccShardGroup* group, const SaccScanExArgs* args, const cudaStream_t* streams,
                              void* const* gather, size_t shard_y_bytes) {
    return guarded([&] {
        constexpr const char* api = "scan_sharded";
        if (group == nullptr || args == nullptr || streams == nullptr) reject(api, "group, args and streams are required");
        const int ndev = static_cast<int>(group->devices.size());
        DeviceGuard keep;
        // Every shard is checked on the host before any device gets work.
        for (int i = 0; i < ndev; ++i) {
            const std::string shard = std::string(api) + " shard " + std::to_string(i);
            CK(cudaSetDevice(group->devices[i]));
            int stream_device = -1;
            if (streams[i] != nullptr && streams[i] != cudaStreamLegacy && streams[i] != cudaStreamPerThread) {
                CK(cudaStreamGetDevice(streams[i], &stream_device));
                if (stream_device != group->devices[i]) reject(shard.c_str(), "stream belongs to another CUDA device");
            }
            validate_scan_ex(shard.c_str(), args[i], streams[i]);
            if (gather) {
                const std::size_t ybytes = args[i].batch * args[i].length * args[i].channels * dtype_bytes(args[i].dtype);
                if (ybytes != shard_y_bytes) reject(shard.c_str(), "y must hold exactly shard_y_bytes bytes to be gathered");
                if (gather[i] == nullptr) reject(shard.c_str(), "gather buffer is null");
            }
        }
        for (int i = 0; i < ndev; ++i) {
            CK(cudaSetDevice(group->devices[i]));
            CK(launch_scan_ex(args[i], sm_count(), streams[i]));
        }
        if (gather) {
            const Nccl& n = nccl();
            nck(n.group_start(), "ncclGroupStart");
            ncclResult_t r = ncclSuccess;
            for (int i = 0; i < ndev && r == ncclSuccess; ++i)
                r = n.all_gather(args[i].y, gather[i], shard_y_bytes, ncclUint8, group->comms[i], streams[i]);
            const ncclResult_t e = n.group_end();
            nck(r, "ncclAllGather");
            nck(e, "ncclGroupEnd");
        }
    });
}

} // extern "C"
