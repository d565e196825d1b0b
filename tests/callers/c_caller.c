/* A C caller of the C ABI (include/sacc_scan.h), as a TensorRT-free host would
 * write it: one reference-ABI scan of the HR deploy level-0 shape on caller
 * device buffers, and the Cross-Scan head level on FP32 maps.  Compiled and
 * linked against libsacc_scan.so by tests/test_callers_cpu.py; main() only
 * prints the build identity, so it runs without a GPU. */
#include <stdio.h>
#include <string.h>

#include "sacc_scan.h"

int scan_level0(const float* u, const float* delta, const float* a, const float* b, const float* c, const float* d,
                float* y, SaccScanStatus* status, cudaStream_t stream) {
    SaccScanShape shape = {4, 960, 256, 16, 1, 1, 1};
    SaccScanInputs in = {u, delta, a, b, c, d}; /* device pointers */
    int rc = sacc_selective_scan_f32(&shape, &in, y, status, stream);
    if (rc != SACC_OK) fprintf(stderr, "%s\n", sacc_last_error());
    return rc;
}

int head_level(SaccMambaBlockArgs block_args, size_t hs, size_t ws, const float* down, float* merged, void* workspace,
               size_t workspace_bytes, cudaStream_t stream) {
    SaccCrossScanBlockArgs lv;
    size_t bytes = 0;
    memset(&lv, 0, sizeof lv);
    lv.block = block_args;          /* weights and shapes as for sacc_mamba_block_forward */
    lv.block.batch = 1;             /* images */
    lv.block.length = hs * ws;      /* map positions; block.x and block.out are not used */
    lv.height = hs;
    lv.width = ws;
    lv.x = down;                    /* (1, 128, hs, ws) FP32, the downsample conv's output */
    lv.out = merged;                /* (1, 128, hs, ws) FP32, the upsample conv's input */
    if (sacc_cross_scan_block_workspace(&lv, &bytes) != SACC_OK || bytes > workspace_bytes) return SACC_EINVAL;
    return sacc_cross_scan_block_forward(&lv, workspace, bytes, stream);
}

int main(void) {
    printf("%s", sacc_scan_identity());
    return 0;
}
