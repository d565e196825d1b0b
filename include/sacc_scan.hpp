// sacc_scan.hpp -- header-only C++ adapter with the reference's C++ signatures
// on top of the C ABI in sacc_scan.h, so that code written against
// include/saccade/selective_scan_cuda.hpp (the TensorRT plugin, the reference's
// tests and benchmark) compiles unchanged against libsacc_scan.so:
//
//   saccade::selective_scan_cuda(shape, inputs, y, status, stream)   cuda/selective_scan.cu:270-311
//   saccade::selective_scan_cuda_load_kernels()                       cuda/selective_scan.cu:252-268
//   saccade::cross_scan_expand_cuda / cross_scan_merge_cuda           cuda/selective_scan.cu:313-345
//   saccade::selective_scan_cuda_identity()                           cuda/selective_scan.cu:347-357
//
// include/saccade/selective_scan_cuda.hpp of this repository includes this
// file, so a tree that builds against the reference's headers replaces that
// one file and links libsacc_scan.so.  saccade::SelectiveScanShape comes from
// the reference's own include/saccade/selective_scan.hpp whenever that header
// is on the include path (it is the host reference's type too); only without
// it is the same shape defined here.
//
// Error behaviour is the reference's: SACC_EINVAL becomes std::invalid_argument
// (nothing was enqueued), SACC_ECUDA becomes std::runtime_error, each with the
// library's diagnostic text.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "sacc_scan.h"

#if __has_include("saccade/selective_scan.hpp")
#include "saccade/selective_scan.hpp"
#else
namespace saccade {
// include/saccade/selective_scan.hpp:19-27
struct SelectiveScanShape {
    std::size_t batch = 0;
    std::size_t length = 0;
    std::size_t channels = 0;
    std::size_t state = 0;
    std::size_t a_rows = 1;
    std::size_t c_width = 1;
    bool has_d = true;
};
} // namespace saccade
#endif

namespace saccade {

// include/saccade/selective_scan_cuda.hpp:21-55
using ScanStatus = SaccScanStatus;
inline constexpr std::uint32_t kScanDone = SACC_SCAN_DONE;
enum ScanFailure : std::uint32_t {
    kScanNonFiniteU = SACC_SCAN_NONFINITE_U,
    kScanNonFiniteDelta = SACC_SCAN_NONFINITE_DELTA,
    kScanNonFiniteA = SACC_SCAN_NONFINITE_A,
    kScanNonFiniteB = SACC_SCAN_NONFINITE_B,
    kScanNonFiniteC = SACC_SCAN_NONFINITE_C,
    kScanNonFiniteD = SACC_SCAN_NONFINITE_D,
    kScanDecayRange = SACC_SCAN_DECAY_RANGE,
    kScanDriveRange = SACC_SCAN_DRIVE_RANGE,
    kScanStateRange = SACC_SCAN_STATE_RANGE,
    kScanTermRange = SACC_SCAN_TERM_RANGE,
    kScanSkipRange = SACC_SCAN_SKIP_RANGE,
    kScanOutputRange = SACC_SCAN_OUTPUT_RANGE,
    kCrossScanNonFiniteInput = SACC_CROSS_SCAN_NONFINITE_INPUT,
};
inline constexpr std::uint32_t kScanInputFailures = SACC_SCAN_INPUT_FAILURES;
inline constexpr std::uint32_t kScanRangeFailures = SACC_SCAN_RANGE_FAILURES;

struct SelectiveScanDeviceInputs {
    const float* u = nullptr;
    const float* delta = nullptr;
    const float* a = nullptr;
    const float* b = nullptr;
    const float* c = nullptr;
    const float* d = nullptr;
};

struct CrossScanShape {
    std::size_t batch = 0, channels = 0, height = 0, width = 0;
};

namespace sacc_detail {
inline void check(int rc) {
    if (rc == SACC_OK) return;
    const std::string what = sacc_last_error();
    if (rc == SACC_EINVAL) throw std::invalid_argument(what);
    throw std::runtime_error(what);
}
} // namespace sacc_detail

inline std::string selective_scan_cuda_load_kernels() {
    std::string report(1 << 16, '\0');
    sacc_detail::check(sacc_scan_load_kernels(report.data(), report.size()));
    report.resize(std::char_traits<char>::length(report.c_str()));
    return report;
}

inline void selective_scan_cuda(const SelectiveScanShape& s, const SelectiveScanDeviceInputs& in, float* y,
                                ScanStatus* status, cudaStream_t stream) {
    const SaccScanShape shape{s.batch, s.length, s.channels, s.state, s.a_rows, s.c_width, s.has_d ? 1 : 0};
    const SaccScanInputs inputs{in.u, in.delta, in.a, in.b, in.c, in.d};
    sacc_detail::check(sacc_selective_scan_f32(&shape, &inputs, y, status, stream));
}

inline void cross_scan_expand_cuda(const CrossScanShape& s, const float* x, float* tokens, ScanStatus* status,
                                   cudaStream_t stream) {
    const SaccCrossScanShape shape{s.batch, s.channels, s.height, s.width};
    sacc_detail::check(sacc_cross_scan_expand_f32(&shape, x, tokens, status, stream));
}

inline void cross_scan_merge_cuda(const CrossScanShape& s, const float* y, float* out, ScanStatus* status,
                                  cudaStream_t stream) {
    const SaccCrossScanShape shape{s.batch, s.channels, s.height, s.width};
    sacc_detail::check(sacc_cross_scan_merge_f32(&shape, y, out, status, stream));
}

inline std::string selective_scan_cuda_identity() { return sacc_scan_identity(); }

} // namespace saccade
