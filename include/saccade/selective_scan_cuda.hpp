// saccade/selective_scan_cuda.hpp -- drop-in for the reference's header of the
// same name (include/saccade/selective_scan_cuda.hpp of the reference): the
// same declarations (ScanStatus, kScanDone, ScanFailure, SelectiveScanDeviceInputs,
// CrossScanShape, selective_scan_cuda, selective_scan_cuda_load_kernels,
// cross_scan_expand_cuda, cross_scan_merge_cuda, selective_scan_cuda_identity)
// as inline functions over this library's C ABI (sacc_scan.h).  Put this
// repository's include/ ahead of the reference's on the include path and link
// libsacc_scan.so instead of the reference's CUDA scan library; the
// reference's other headers (selective_scan.hpp with SelectiveScanShape, ...)
// stay as they are.
#pragma once

#include "../sacc_scan.hpp"
