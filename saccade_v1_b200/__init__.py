"""saccade_v1_b200 -- B200-native (sm_100a) selective-scan hot path of saccade_v1.

The product is libsacc_scan.so (C ABI in include/sacc_scan.h); this package is
its in-tree build recipe (build.py), ctypes binding (_lib.py) and the host-side
front end for torch device buffers (scan.py).
"""
from .scan import (  # noqa: F401
    CrossScanShape,
    ScanCudaError,
    ScanInvalidArgument,
    SelectiveScanShape,
    SCAN_DONE,
    cross_scan_expand_cuda,
    cross_scan_merge_cuda,
    gemm,
    identity,
    load_kernels,
    cross_scan_block_forward,
    cross_scan_block_workspace,
    mamba_block_forward,
    mamba_block_forward_noalloc,
    mamba_block_workspace,
    scan_fault,
    selective_scan_cuda,
    selective_scan_ex,
    selective_scan_f16,
    selective_scan_step,
)
