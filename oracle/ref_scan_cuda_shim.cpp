// ref_scan_cuda_shim.cpp -- C entry points around the reference's own CUDA FP32
// selective scan (cuda/selective_scan.cu), compiled for sm_100a.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file with the
// reference's cuda/selective_scan.cu, taken from where it lies in the
// reference checkout (never copied), into oracle/_ref/libref_scan_cuda.so, with
// the reference's own scan flags (CMakeLists.txt:194).  It needs a CUDA driver,
// so only GPU runs load it: tests/test_ref_scan_cuda_gpu.py checks its outputs
// against the oracle, and bench.py times it beside this library's kernel at
// the reference's deploy shapes on the same B200.
//
// Wrapped interfaces (include/saccade/selective_scan_cuda.hpp):
//   selective_scan_cuda_load_kernels (:64), selective_scan_cuda (:72-73).
// Each returns 0, or -1 with the exception's text in msg.
#include "saccade/selective_scan_cuda.hpp"

#include <cstdint>
#include <cstdio>
#include <exception>
#include <string>

extern "C" {

struct RefCudaShape {
    std::uint64_t batch, length, channels, state, a_rows, c_width;
    std::int32_t has_d;
};

int ref_scan_cuda_load(char* msg, std::size_t cap) {
    try {
        const std::string report = saccade::selective_scan_cuda_load_kernels();
        if (msg && cap) std::snprintf(msg, cap, "%s", report.c_str());
        return 0;
    } catch (const std::exception& e) {
        if (msg && cap) std::snprintf(msg, cap, "%s", e.what());
    }
    return -1;
}

int ref_scan_cuda(const RefCudaShape* s, const float* u, const float* delta, const float* a, const float* b, const float* c,
                  const float* d, float* y, void* status, void* stream, char* msg, std::size_t cap) {
    try {
        saccade::SelectiveScanShape shape;
        shape.batch = s->batch;
        shape.length = s->length;
        shape.channels = s->channels;
        shape.state = s->state;
        shape.a_rows = s->a_rows;
        shape.c_width = s->c_width;
        shape.has_d = s->has_d != 0;
        saccade::selective_scan_cuda(shape, {u, delta, a, b, c, d}, y, static_cast<saccade::ScanStatus*>(status),
                                     static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception& e) {
        if (msg && cap) std::snprintf(msg, cap, "%s", e.what());
    }
    return -1;
}

} // extern "C"
