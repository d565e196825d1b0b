/*
 * sacc_scan.h -- C ABI of the B200 selective-scan library (libsacc_scan.so).
 *
 * Drop-in boundary for saccade_v1's selective-scan hot path.  Every entry
 * point takes plain pointers and sizes, never throws, and returns SACC_OK or
 * an error code; the message of the last failure on the calling thread is
 * sacc_last_error().  All GPU work is enqueued on the caller's stream only;
 * no entry point allocates, synchronises or reads back to the host (once the
 * kernels are loaded), so every call is capturable in a CUDA graph.
 *
 * Reference interfaces replaced (paths in the saccade_v1 project):
 *   SaccScanStatus / SACC_SCAN_*    include/saccade/selective_scan_cuda.hpp:21-46
 *   SaccScanShape                   include/saccade/selective_scan.hpp:19-27
 *   SaccScanInputs                  include/saccade/selective_scan_cuda.hpp:48-55
 *   sacc_scan_load_kernels          selective_scan_cuda_load_kernels, cuda/selective_scan.cu:252-268
 *   sacc_selective_scan_f32         selective_scan_cuda, cuda/selective_scan.cu:270-311
 *   sacc_cross_scan_expand_f32      cross_scan_expand_cuda, cuda/selective_scan.cu:313-328
 *   sacc_cross_scan_merge_f32       cross_scan_merge_cuda, cuda/selective_scan.cu:330-345
 *   sacc_scan_identity              selective_scan_cuda_identity, cuda/selective_scan.cu:347-357
 *   sacc_selective_scan_f16         no counterpart: the FP16-activation form behind plugin
 *                                   SelectiveScan v3 (the reference's FP16 engine keeps its scan
 *                                   plugins FP32 and casts around them,
 *                                   include/saccade/head_trt_network.hpp:25-28)
 * The reference throws std::invalid_argument (host rejection, nothing
 * enqueued) and std::runtime_error (a CUDA API call failed); here those are
 * SACC_EINVAL and SACC_ECUDA with the same diagnostic text.
 */
#ifndef SACC_SCAN_H
#define SACC_SCAN_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SACC_OK 0
#define SACC_EINVAL 1 /* host rejection before any GPU work (reference: std::invalid_argument) */
#define SACC_ECUDA 2  /* a CUDA API call failed (reference: std::runtime_error) */

/* Device-side outcome of one call, in caller-owned device memory.  Cleared on
 * the stream before any other work; `done` is written last.  An output is
 * valid only when done == SACC_SCAN_DONE and flags == 0; on failure every
 * output element is the quiet NaN 0x7fc00000. */
typedef struct SaccScanStatus {
    uint32_t flags;
    uint32_t done;
} SaccScanStatus;
#define SACC_SCAN_DONE 0x4E414353u /* "SCAN" */

/* Input bits: exact, set iff that tensor holds a NaN or an infinity.
 * Range bits: per (batch, channel) lane, the first quantity in the
 * reference's order (decay, drive, state, C*state, then D*u, output) whose
 * FP32 value left the finite range, united over lanes. */
#define SACC_SCAN_NONFINITE_U (1u << 0)
#define SACC_SCAN_NONFINITE_DELTA (1u << 1)
#define SACC_SCAN_NONFINITE_A (1u << 2)
#define SACC_SCAN_NONFINITE_B (1u << 3)
#define SACC_SCAN_NONFINITE_C (1u << 4)
#define SACC_SCAN_NONFINITE_D (1u << 5)
#define SACC_SCAN_DECAY_RANGE (1u << 8)
#define SACC_SCAN_DRIVE_RANGE (1u << 9)
#define SACC_SCAN_STATE_RANGE (1u << 10)
#define SACC_SCAN_TERM_RANGE (1u << 11)
#define SACC_SCAN_SKIP_RANGE (1u << 12)
#define SACC_SCAN_OUTPUT_RANGE (1u << 13)
#define SACC_CROSS_SCAN_NONFINITE_INPUT (1u << 16)
#define SACC_SCAN_INPUT_FAILURES 0x3Fu
#define SACC_SCAN_RANGE_FAILURES 0x3F00u

/* Reference ABI: dense row-major FP32,
 *   u, delta, y (batch, length, channels)   delta raw, before softplus
 *   a (a_rows, state)                       a_rows = 1 or channels
 *   b (batch, length, state)
 *   c (batch, length, c_width)              c_width = 1 or state
 *   d (channels)                            only when has_d
 * state is a power of two in [1, 32]; length 0 is valid (empty output);
 * every tensor holds at most INT32_MAX elements; zero initial state. */
typedef struct SaccScanShape {
    uint64_t batch, length, channels, state, a_rows, c_width;
    int32_t has_d;
} SaccScanShape;

typedef struct SaccScanInputs {
    const float *u, *delta, *a, *b, *c, *d;
} SaccScanInputs;

/* Loads every kernel of the library in the current CUDA context (defeats lazy
 * loading, which would otherwise wait for device work at the first launch).
 * Call once per context during initialisation.  Writes one line per kernel
 * (registers, local, shared, max threads) into `report` when it is non-NULL. */
int sacc_scan_load_kernels(char* report, size_t report_bytes);

/* Validates on the host, then enqueues on `stream` only: status clear, input
 * check + scan (one kernel), finalize.  `stream` must be an explicit
 * non-default stream.  Zero workspace.  Pointers must be 4-byte aligned;
 * y and status must not overlap an input or each other. */
int sacc_selective_scan_f32(const SaccScanShape* shape, const SaccScanInputs* inputs, float* y, SaccScanStatus* status,
                            cudaStream_t stream);

/* The same operator with FP16 activations: u, delta, b, c and y are IEEE
 * binary16 bit patterns (2-byte aligned), a and d stay FP32.  Checks,
 * arithmetic and status bits are those of sacc_selective_scan_f32 on the
 * inputs widened to FP32 (a NaN or infinity in an FP16 input sets its input
 * bit), and y is that call's output rounded to nearest FP16; an output of
 * magnitude 65520 or more, which FP16 cannot hold, is SACC_SCAN_OUTPUT_RANGE.
 * On failure every y element is the FP16 quiet NaN 0x7E00. */
typedef struct SaccScanInputsF16 {
    const uint16_t *u, *delta;
    const float* a;
    const uint16_t *b, *c;
    const float* d;
} SaccScanInputsF16;
int sacc_selective_scan_f16(const SaccScanShape* shape, const SaccScanInputsF16* inputs, uint16_t* y, SaccScanStatus* status,
                            cudaStream_t stream);

/* Cross-Scan (x (batch, channels, height, width) <-> tokens (4 batch,
 * height*width, channels), direction-major rows; direction 0 identity, 1 flip
 * H and W, 2 flip W, 3 flip H).  Merge averages ((y0+y1)+y2)+y3 times 0.25. */
typedef struct SaccCrossScanShape {
    uint64_t batch, channels, height, width;
} SaccCrossScanShape;
int sacc_cross_scan_expand_f32(const SaccCrossScanShape* shape, const float* x, float* tokens, SaccScanStatus* status,
                               cudaStream_t stream);
int sacc_cross_scan_merge_f32(const SaccCrossScanShape* shape, const float* y, float* out, SaccScanStatus* status,
                              cudaStream_t stream);

/* Message of the last failed call on this thread ("" if none). */
const char* sacc_last_error(void);

/* Build identity: nvcc version, flags, target architectures, one key=value per line. */
const char* sacc_scan_identity(void);

/* Diagnostics (no counterpart in the reference): every wait of a kernel on an
 * asynchronous copy has an iteration limit; when one runs out, the kernel sets
 * a bit in the library's device fault word and leaves.  Reads that word into
 * *out (synchronous with the device), clearing it when `clear` is non-zero.
 * 0 means no kernel has ever given up waiting. */
int sacc_scan_fault(uint32_t* out, int clear);
/* Diagnostics: enqueues one CTA that waits, with the scan kernels' own wait
 * helpers, on a hand-off flag nothing sets and on an mbarrier nothing arrives
 * at, `limit` polls each (1 .. 2^20); both waits run out, the kernel sets bit 0
 * of the fault word and returns, and the context stays usable.  For testing
 * the failure path without a GPU fault. */
int sacc_scan_wait_probe(uint32_t limit, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * Extended scan (no counterpart in the reference, whose contract has zero
 * initial state, no final state and FP32 only): the Mamba selective-scan
 * forward with bf16/fp16/fp32 activations and FP32 state.
 *
 * layout SACC_LAYOUT_BLD (reference order):
 *   u, delta, z, y (batch, length, channels); b (batch, length, groups, state);
 *   c (batch, length, groups, c_width)
 * layout SACC_LAYOUT_BDL (Mamba order):
 *   u, delta, z, y (batch, channels, length); b (batch, groups, state, length);
 *   c (batch, groups, c_width, length)
 * a (a_rows, state) FP32; d, delta_bias (channels) FP32, each optional.
 * Delta = softplus(delta + delta_bias) when delta_softplus, else delta + delta_bias.
 * y = (sum_n C_n h_n + D u) * silu(z) (gate only when z is given).
 * h0 / h_final (nseq, channels, state) FP32, each optional.
 * cu_seqlens (nseq + 1 int32, batch must be 1): sequence k is tokens
 * [cu_seqlens[k], cu_seqlens[k+1]) of the length axis and starts from h0[k]
 * (or zero); without cu_seqlens nseq = batch.  The entries are device data and
 * are not checked on the host: each is clamped to [0, length], and a
 * sequence whose end precedes its start is empty.
 * No status words: non-finite values propagate into y as IEEE arithmetic does.
 * Pointers of 16-bit tensors must be 16-byte aligned and channels * 2 bytes
 * (BLD) or length * 2 bytes (BDL) a multiple of 16, for the TMA staging.
 * ------------------------------------------------------------------------ */
#define SACC_DTYPE_F32 0
#define SACC_DTYPE_BF16 1
#define SACC_DTYPE_F16 2
#define SACC_LAYOUT_BLD 0
#define SACC_LAYOUT_BDL 1

typedef struct SaccScanExArgs {
    uint64_t batch, length, channels, state, groups, a_rows, c_width;
    int32_t layout, dtype, delta_softplus, nseq;
    const void *u, *delta, *b, *c, *z; /* activations, `dtype` */
    const float *a, *d, *delta_bias;   /* parameters, FP32 */
    const float* h0;                   /* optional (nseq, channels, state) */
    float* h_final;                    /* optional (nseq, channels, state) */
    const int32_t* cu_seqlens;         /* optional (nseq + 1) */
    void* y;                           /* output, `dtype` */
} SaccScanExArgs;

int sacc_selective_scan_ex(const SaccScanExArgs* args, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * Per-frame step (no counterpart in the reference): one token of every
 * sequence advances carried FP32 state in place,
 *   h[slot[i]] = exp(Delta_i A) h[slot[i]] + Delta_i B_i u_i,
 *   y_i = (sum_n C_i,n h_n + D u_i) * silu(z_i).
 * u, delta, z, y (nseq, channels); b (nseq, groups, state); c (nseq, groups,
 * c_width); a (a_rows, state), d, delta_bias (channels) FP32.
 * state: (slots, channels, state) FP32, 16-byte aligned, read and written.
 * slot (optional, nseq int32): state row of sequence i (a tracker's slot);
 * a negative slot skips the sequence and writes y_i = 0.  Without slot,
 * sequence i uses row i and slots must equal nseq.  Two sequences must not
 * name the same slot in one call.
 * ------------------------------------------------------------------------ */
typedef struct SaccScanStepArgs {
    uint64_t nseq, channels, state, groups, a_rows, c_width, slots;
    int32_t dtype, delta_softplus;
    const void *u, *delta, *z, *b, *c; /* `dtype` */
    const float *a, *d, *delta_bias;
    float* state_io;
    const int32_t* slot;
    void* y;
} SaccScanStepArgs;

int sacc_selective_scan_step(const SaccScanStepArgs* args, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * Projection GEMM on the tensor cores (no counterpart in the reference, whose
 * projections are TensorRT matrix-multiply layers, src/head_trt_network.cpp:
 * 192-230): C[m, n] = s[m] sum_k A[m, k] B[n, k] (+ bias[n]) (+ R[m, n]).
 * A (m x k, row stride lda) and B (n x k, row stride ldb) are bf16 or fp16
 * (in_dtype), K contiguous, 16-byte aligned, lda and ldb multiples of 8;
 * C and R are out_dtype (f32, bf16, f16) with row strides ldc / ldr; bias FP32.
 * FP32 accumulation in tensor memory.
 * ------------------------------------------------------------------------ */
typedef struct SaccGemmArgs {
    uint64_t m, n, k, lda, ldb, ldc, ldr;
    int32_t in_dtype, out_dtype;
    const void* a;
    const void* b;
    void* c;
    const float* bias;      /* optional (n) */
    const void* residual;   /* optional (m x n, ldr) */
    const float* row_scale; /* optional (m), s above; 1 when absent */
} SaccGemmArgs;

int sacc_gemm(const SaccGemmArgs* args, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * One Mamba block forward (the reference builds it from TensorRT layers
 * around its scan plugin, src/head_trt_network.cpp:181-233), with the
 * optional RMSNorm prologue of BASELINE configs 1 and 4:
 *   xn = rmsnorm(x) * norm_w; [x_in, z] = xn W_in^T; u = silu(conv1d(x_in) + conv_b);
 *   [dt, B, C] = u W_x^T; delta = dt W_dt^T; y = scan(u, delta + dt_bias, A, B, C, D) * silu(z);
 *   out = y W_out^T (+ x when residual).
 * Activations and projection weights bf16 or fp16 (dtype); x, out
 * (batch, length, d_model); w_in (2 d_inner, d_model); w_x (dt_rank + d_state +
 * c_width, d_inner) with c_width = d_state (also written 0) or 1 (one C per token
 * broadcast over the states, as in the reference head's x_proj 256 -> 16 + 16 + 1);
 * w_dt (d_inner, dt_rank); w_out (d_model, d_inner).  FP32: norm_w
 * (d_model, optional), conv_w (d_inner, d_conv), conv_b, dt_bias, d (d_inner),
 * a (d_inner, d_state) = -exp(A_log).  d_conv must be 4, d_state 16, d_inner
 * and d_model multiples of 128, dt_rank a multiple of 8.
 * Intermediates go to `workspace` (at least sacc_mamba_block_workspace bytes,
 * 256-byte aligned); the call allocates nothing.
 * ------------------------------------------------------------------------ */
typedef struct SaccMambaBlockArgs {
    uint64_t batch, length, d_model, d_inner, d_state, d_conv, dt_rank;
    int32_t dtype, residual;
    float eps;
    const void* x;
    const float* norm_w;
    const void* w_in;
    const float *conv_w, *conv_b;
    const void* w_x;
    const void* w_dt;
    const float *dt_bias, *a, *d;
    const void* w_out;
    void* out;
    int32_t c_width; /* C per token: 0 or d_state (full), or 1 */
} SaccMambaBlockArgs;

int sacc_mamba_block_workspace(const SaccMambaBlockArgs* args, size_t* bytes);
int sacc_mamba_block_forward(const SaccMambaBlockArgs* args, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * sacc_mamba_block_forward_noalloc -- no counterpart in the reference.
 *
 * The same block forward for callers that cannot allocate a workspace (a
 * plugin that the engine gives no workspace and that may not allocate inside
 * enqueue; a per-frame loop under a fixed memory budget).  The intermediates
 * go to one static device array of SACC_NOALLOC_SCRATCH_BYTES per device,
 * reserved when CUDA loads the library's module; the call allocates nothing.
 * Blocks whose sacc_mamba_block_workspace exceeds that size are rejected with
 * SACC_EINVAL.  The first call on a device looks up the array's address:
 * make it before any stream capture.  All calls on a device share the array
 * and it keeps the last call's contents: every intermediate is written before
 * it is read, and the scan's hand-off flags in it are cleared on the stream
 * before each use.  Calls that overlap on the GPU race on the array: order
 * them on one stream.
 * ------------------------------------------------------------------------ */
#define SACC_NOALLOC_SCRATCH_BYTES ((size_t)24 << 20)
int sacc_mamba_block_forward_noalloc(const SaccMambaBlockArgs* args, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * sacc_cross_scan_block_forward -- one Cross-Scan head level with the expand
 * and merge fused into the Mamba block.  Replaces the reference's steps 3-5 of
 * a head level (src/head_trt_network.cpp:200-232): the CrossScanExpand plugin
 * (cuda/selective_scan.cu:157-175, host :402-416), the block layers with the
 * residual on the expanded tokens, and the CrossScanMerge plugin (:177-192,
 * host :418-434):
 *   tokens_k = expand_k(x)            direction k: 0 identity, 1 flip H and W, 2 flip W, 3 flip H
 *   r_k = block(tokens_k) (+ tokens_k when block.residual)
 *   out = (((r_0 + r_1) + r_2) + r_3) / 4 at each map position
 * without materialising the (4 batch, H W, d_model) tokens: in_proj and
 * out_proj act on each token alone, so in_proj runs once per map position and
 * each direction reads its rows through the flip; the four directions' gated
 * scan outputs are averaged per position (the merge's order and overflow
 * rule) before one out_proj per position, and x is added as the maps are
 * written (a flip is an involution, so every direction's token at a position
 * is x there).  The
 * result equals the reference composition up to rounding (out_proj is linear).
 * block: as for sacc_mamba_block_forward with batch = images and length =
 * height * width; its x and out are not used.  x, out: (batch, d_model,
 * height, width) FP32 maps, 16-byte aligned, not overlapping.  At most 65535
 * images.  Workspace from sacc_cross_scan_block_workspace (256-byte aligned).
 * ------------------------------------------------------------------------ */
typedef struct SaccCrossScanBlockArgs {
    SaccMambaBlockArgs block;
    uint64_t height, width;
    const float* x;
    float* out;
} SaccCrossScanBlockArgs;

int sacc_cross_scan_block_workspace(const SaccCrossScanBlockArgs* args, size_t* bytes);
int sacc_cross_scan_block_forward(const SaccCrossScanBlockArgs* args, void* workspace, size_t workspace_bytes,
                                  cudaStream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SACC_SCAN_H */
