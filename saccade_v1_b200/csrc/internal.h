// internal.h -- declarations shared by the CUDA translation units and the
// C-ABI layer (capi.cpp).  Not part of the public interface (include/).
#pragma once

#include <cuda_runtime_api.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <string>

#include "../../include/sacc_frame.h"
#include "../../include/sacc_scan.h"

namespace sacc {

// Launches `fn` with programmatic stream serialization (its set-up may overlap
// the previous kernel of the stream; the kernel itself waits for that
// kernel's results with griddepcontrol.wait).
inline cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, std::size_t smem, cudaStream_t stream, void** args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// Runs `set` (a kernel attribute setting, which CUDA applies to the current
// device's copy of the kernel) once per device ordinal; `done` holds one flag
// per ordinal for the call site.  Concurrent first calls may both run `set`,
// which is idempotent.
template <typename F>
cudaError_t once_per_device(std::atomic<int> (&done)[64], F&& set) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return set();
    if (done[dev].load(std::memory_order_acquire) == 1) return cudaSuccess;
    e = set();
    if (e == cudaSuccess) done[dev].store(1, std::memory_order_release);
    return e;
}

// int32 element capacity of every tensor of the reference ABI
// (reference src/selective_scan.cpp:15, cuda/selective_scan.cu:30).
constexpr std::size_t kMaxElements = 2147483647u;

struct CheckedTensor {
    const void* data; // FP32, or FP16 when `half`
    unsigned long long count;
    std::uint32_t bit;
    int half = 0;
};
struct CheckList {
    CheckedTensor tensor[6];
    unsigned size;
};

// One reference-ABI call, resolved on the host; `half`: u, delta, B, C and y
// are FP16 (plugin v3), A and D FP32 either way.
struct ScanF32Launch {
    const void *u, *delta;
    const float* a;
    const void *b, *c;
    const float* d;
    void* y;
    unsigned long long batch, length, channels, lanes;
    unsigned state;
    bool a_shared, c_full, has_d;
    bool half = false;
};

// Enqueues the scan kernel on `stream` right after the input check
// (launch_check), with programmatic stream serialization: the check releases
// it at once and it waits for the check grid before it completes (status
// already cleared by the caller).  Returns a CUDA error (launch only).
cudaError_t launch_scan_f32(const ScanF32Launch& p, SaccScanStatus* status, int sm_count, cudaStream_t stream);
// Poisons `count` outputs (FP32, or FP16 when `half`) with quiet NaN when
// flags != 0, then writes done.
cudaError_t launch_finalize(void* out, unsigned long long count, SaccScanStatus* status, int sm_count, cudaStream_t stream,
                            bool half = false);
// Exact NaN / Inf bits of the listed tensors (every reference-ABI and
// Cross-Scan call runs it first).
cudaError_t launch_check(const CheckList& list, SaccScanStatus* status, int sm_count, cudaStream_t stream);

struct CrossLaunch {
    unsigned long long batch, channels, height, width;
};
cudaError_t launch_cross_expand(const CrossLaunch& p, const float* x, float* tokens, int sm_count, cudaStream_t stream);
cudaError_t launch_cross_merge(const CrossLaunch& p, const float* y, float* out, int sm_count, cudaStream_t stream);

// Extended scan (bf16/fp16/fp32 activations, FP32 state).
cudaError_t launch_scan_ex(const SaccScanExArgs& a, int sm_count, cudaStream_t stream);
cudaError_t launch_scan_general(const SaccScanExArgs& a, cudaStream_t stream);
cudaError_t load_scan_general_kernels(std::string& report);
// Row pitches (elements between consecutive tokens) of z, B and C in the
// (B, L, .) layout when they are column slices of wider matrices; 0 = dense.
struct RowStrides {
    unsigned long long z, b, c;
};
bool bulk_eligible(const SaccScanExArgs& a, const RowStrides* rs = nullptr);
cudaError_t launch_scan_step(const SaccScanStepArgs& a, cudaStream_t stream);
cudaError_t launch_gemm(const SaccGemmArgs& a, cudaStream_t stream);
// RMSNorm folded into in_proj, one launch: r[i] = 1 / sqrt(mean_k x[i, k]^2
// + eps) for the m rows of x (k wide), and out = W_in (n x k) with column j
// scaled by w[j].
cudaError_t launch_rms_prep(int dtype, const void* x, unsigned long long m, unsigned k, float eps, float* r, const void* w_in,
                            const float* w, unsigned long long n, void* out, cudaStream_t stream);
// Words that a kernel of the block pipeline zeroes as a side job (block 0,
// after griddepcontrol.wait): the fused chunk-parallel scan's hand-off flags,
// cleared by the conv kernel that precedes the scan in every block call, so
// the scan needs no memset node of its own.
struct ZeroSpan {
    unsigned long long* ptr = nullptr;
    unsigned long long words = 0;
};
cudaError_t launch_conv_silu(int dtype, int kwidth, const void* x, unsigned long long ldx, const float* w, const float* bias,
                             unsigned long long batch, unsigned long long len, unsigned long long dim, void* u,
                             cudaStream_t stream, ZeroSpan zero = {});
// dst = src (rows x cols) with its last row repeated `copies` times in total.
cudaError_t launch_repeat_last_row(int dtype, const void* src, unsigned long long rows, unsigned long long copies,
                                   unsigned long long cols, void* dst, cudaStream_t stream);
cudaError_t load_block_kernels(std::string& report);
cudaError_t read_block_fault(unsigned* out, bool clear);
std::size_t mamba_block_workspace(const SaccMambaBlockArgs& a);
cudaError_t launch_mamba_block(const SaccMambaBlockArgs& a, void* workspace, cudaStream_t stream);
// Same forward with the intermediates in a static device array of
// kNoAllocScratchBytes (block_noalloc.cu); cudaErrorInvalidValue when the
// block needs more.
constexpr std::size_t kNoAllocScratchBytes = SACC_NOALLOC_SCRATCH_BYTES;
cudaError_t launch_mamba_block_noalloc(const SaccMambaBlockArgs& a, cudaStream_t stream);

// One Cross-Scan head level, expand and merge fused into the block
// (mamba_block.cpp; elementwise stages in cross_block.cu).
std::size_t cross_block_workspace(const SaccCrossScanBlockArgs& c);
cudaError_t launch_cross_block(const SaccCrossScanBlockArgs& c, void* workspace, cudaStream_t stream);
// rows (batch, L, C) in dtype = x (batch, C, L) FP32, transposed.
cudaError_t launch_rows_from_maps(int dtype, const float* x, unsigned long long batch, unsigned long long L,
                                  unsigned long long C, void* rows, cudaStream_t stream);
// out (batch, C, L) FP32 = rows (batch, L, C) FP32 transposed (+ x).
cudaError_t launch_maps_from_rows(const float* rows, const float* x, unsigned long long batch, unsigned long long L,
                                  unsigned long long C, float* out, cudaStream_t stream);
// u, z (4 batch, H W, D): conv + SiLU and gate of every direction, read from
// the position-major in_proj rows xz (batch, H W, 2 D) through the flips.
cudaError_t launch_cross_conv(int dtype, const void* xz, const float* w, const float* bias, unsigned long long batch,
                              unsigned long long H, unsigned long long W, unsigned long long D, void* u, void* z,
                              cudaStream_t stream, ZeroSpan zero = {});
// mean (batch, H W, D) = the merge of y (4 batch, H W, D) at each position.
cudaError_t launch_cross_mean(int dtype, const void* y, unsigned long long batch, unsigned long long H, unsigned long long W,
                              unsigned long long D, void* mean, cudaStream_t stream);
cudaError_t load_cross_block_kernels(std::string& report);
cudaError_t load_gemm_kernels(std::string& report);
cudaError_t read_gemm_fault(unsigned* out, bool clear);
cudaError_t load_scan_step_kernels(std::string& report);
cudaError_t read_step_fault(unsigned* out, bool clear);
// delta formed inside the scan as dt (rows of pitch `ld` elements, `rank`
// columns) x w^T (w: channels x rank), for rank 8 or 16 with the (B, L, D)
// layout, a gate and a full-width C (the block's small dt_proj).
struct DtFusion {
    const void* dt;
    unsigned long long ld;
    const void* w;
    int rank;
};
bool dt_fusable(const SaccScanExArgs& a, const DtFusion& f);
// `scratch` (optional, 16-byte aligned): lets few-unit long-sequence calls run
// the chunk-parallel scan as one fused launch; bulk_scan_scratch_bytes() says
// how much this call would use (0: none).  The fused launch's hand-off flags
// sit at the end of the scratch (bulk_scan_flags) and must be zero when it
// starts: `flags_zeroed` says that an earlier kernel of the stream cleared
// them, otherwise the launch clears them with a memset first.
cudaError_t launch_scan_bulk(const SaccScanExArgs& a, cudaStream_t stream, const RowStrides* rs = nullptr,
                             void* scratch = nullptr, std::size_t scratch_bytes = 0, const DtFusion* dtf = nullptr,
                             bool flags_zeroed = false);
std::size_t bulk_scan_scratch_bytes(const SaccScanExArgs& a, const DtFusion* dtf = nullptr);
// The hand-off flags of a fused scan whose scratch is `scratch_bytes` long
// (as bulk_scan_scratch_bytes gave it) at `scratch`.
ZeroSpan bulk_scan_flags(void* scratch, std::size_t scratch_bytes);
cudaError_t load_scan_bulk_kernels(std::string& report);
// Fault word of the kernels with bounded waits (host-synchronous read; optionally cleared).
cudaError_t read_bulk_fault(unsigned* out, bool clear);
// One CTA whose bounded waits (a flag, an mbarrier) run out after `limit` polls.
cudaError_t launch_wait_probe(std::uint32_t limit, cudaStream_t stream);

// Loads every kernel (cudaFuncGetAttributes) and sets shared-memory limits;
// appends one report line per kernel.
cudaError_t load_scan_f32_kernels(std::string& report);
cudaError_t load_cross_kernels(std::string& report);
cudaError_t load_scan_ex_kernels(std::string& report);

// Frame protocol over the status words (scan_frame.cu).
struct FrameStep {
    SaccScanStatusList list;
    const float* payload;
    unsigned long long count;
    float* results;
    std::int64_t* result_frames;
    SaccScanFrameRecord* records;
    std::int64_t capacity;
    unsigned char* packet;
    std::uint64_t epoch;
    std::int64_t frame;
};
cudaError_t launch_frame_initialize(SaccScanFrameControl* ctl, std::uint64_t epoch, std::int64_t* result_frames, cudaStream_t s);
cudaError_t launch_frame_begin(SaccScanFrameControl* ctl, std::uint64_t epoch, std::int64_t frame, cudaStream_t s);
cudaError_t launch_frame_gate(SaccScanFrameControl* ctl, const SaccScanStatusList& list, SaccScanFrameRecord* records,
                              std::int64_t capacity, cudaStream_t s);
cudaError_t launch_frame_publish(SaccScanFrameControl* ctl, const float* payload, unsigned long long count, float* results,
                                 std::int64_t* result_frames, SaccScanFrameRecord* records, std::int64_t capacity, int sms,
                                 cudaStream_t s);
cudaError_t launch_frame_commit(SaccScanFrameControl* ctl, cudaStream_t s);
cudaError_t launch_frame_packet(const SaccScanFrameControl* ctl, unsigned char* packet, cudaStream_t s);
cudaError_t launch_frame_step(SaccScanFrameControl* ctl, const FrameStep& f, int sms, cudaStream_t s);
cudaError_t launch_frame_check_finite(const float* data, unsigned long long count, SaccScanStatus* status, std::uint32_t flag,
                                      int sms, cudaStream_t s);
cudaError_t launch_frame_delay(unsigned cycles, cudaStream_t s);
std::uint64_t frame_digest(const float* payload, std::size_t count);
cudaError_t load_frame_kernels(std::string& report);

// Model producer status aggregate (model_producer.cu): the image and the six
// raw tensors checked for NaN / Inf, nine plugin statuses gated.
struct ProducerLaunch {
    const float* tensor[7];
    unsigned long long count[7];
    SaccScanStatus* plugin[SACC_MODEL_PRODUCER_PLUGINS];
};
std::size_t producer_workspace_bytes();
cudaError_t launch_model_producer(const ProducerLaunch& p, SaccProducerStatus* producer, void* workspace, int sms, cudaStream_t s);
cudaError_t load_producer_kernels(std::string& report);

} // namespace sacc
