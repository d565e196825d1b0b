// A C++ caller written against the reference's C++ interface
// (saccade::selective_scan_cuda and friends), compiled against
// include/saccade/selective_scan_cuda.hpp of this repository with no
// reference headers on the include path, and linked to libsacc_scan.so by
// tests/test_callers_cpu.py.  main() checks the host-side rejection (no GPU
// work is enqueued for a rejected call) and prints the build identity.
#include "saccade/selective_scan_cuda.hpp"

#include <cstdio>
#include <stdexcept>
#include <string>

namespace {
// 0 when the call throws std::invalid_argument naming `diagnostic`.
int rejects(const saccade::SelectiveScanShape& shape, cudaStream_t stream, const char* diagnostic) {
    try {
        saccade::selective_scan_cuda(shape, {}, nullptr, nullptr, stream);
    } catch (const std::invalid_argument& e) {
        return std::string(e.what()).find(diagnostic) == std::string::npos ? 2 : 0;
    }
    return 1;
}
} // namespace

int main() {
    // Host-side rejections come first and touch no device (the stream handle is never used).
    const auto some_stream = reinterpret_cast<cudaStream_t>(0x1000);
    if (rejects({1, 4, 4, 3, 1, 1, true}, some_stream, "must be a power of two in [1, 32]")) return 1;
    if (rejects({1, 4, 4, 16, 1, 1, true}, cudaStreamLegacy, "an explicit non-default stream is required")) return 2;
    std::printf("%s", saccade::selective_scan_cuda_identity().c_str());
    return 0;
}
