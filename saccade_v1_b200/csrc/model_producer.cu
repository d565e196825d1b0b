// model_producer.cu -- the detector producer's status aggregate (reference
// cuda/model_producer.cu:34-71): every element of the image and of the six
// raw tensors checked for NaN / Inf, the nine plugin statuses (three levels x
// expand / scan / merge) and both finite checks gated by role and retired,
// then the 8-byte aggregate written flags first, done last.
//
// The reference launches initialize (one thread), finite (256 x 7 CTAs) and
// aggregate (one thread).  Here the aggregate runs in the last CTA of the
// finite check to arrive (an arrival counter in the workspace, which the
// one-thread initialize clears): two launches.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <string>

#include "../../include/sacc_frame.h"
#include "internal.h"
#include "scan_common.cuh"

namespace sacc {
namespace {

constexpr unsigned kThreads = 256;

struct Workspace {
    SaccScanStatus input, output; // the two finite checks
    std::uint32_t arrivals, pad;
};

__global__ void producer_initialize_kernel(SaccProducerStatus* producer, Workspace* work) {
    pdl_wait();
    if (threadIdx.x || blockIdx.x) return;
    *producer = SaccProducerStatus{};
    *work = Workspace{};
}

// The bits a source may carry (reference :57-59): scan plugins (i % 3 == 1)
// input and range bits, Cross-Scan plugins their non-finite input bit, the
// finite checks their own bit.
__device__ __forceinline__ std::uint32_t allowed_bits(unsigned i) {
    if (i < SACC_MODEL_PRODUCER_PLUGINS)
        return i % 3 == 1 ? (SACC_SCAN_INPUT_FAILURES | SACC_SCAN_RANGE_FAILURES) : SACC_CROSS_SCAN_NONFINITE_INPUT;
    return i == SACC_MODEL_PRODUCER_PLUGINS ? SACC_FRAME_NONFINITE_INPUT : SACC_FRAME_NONFINITE_OUTPUT;
}

// blockIdx.y = tensor (0 = image, 1..6 = raw); blockIdx.x strides over it.
__global__ void __launch_bounds__(kThreads) producer_check_kernel(ProducerLaunch in, SaccProducerStatus* producer, Workspace* work) {
    pdl_wait();
    const unsigned tensor = blockIdx.y;
    const float* data = in.tensor[tensor];
    const unsigned long long count = in.count[tensor], stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
    bool bad = false;
    for (unsigned long long i = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride)
        bad = bad || !(fabsf(data[i]) <= FLT_MAX);
    bad = __syncthreads_or(bad);
    if (threadIdx.x) return;
    if (bad) atomicOr(tensor == 0 ? &work->input.flags : &work->output.flags,
                      tensor == 0 ? SACC_FRAME_NONFINITE_INPUT : SACC_FRAME_NONFINITE_OUTPUT);
    __threadfence();
    if (atomicAdd(&work->arrivals, 1u) != gridDim.x * gridDim.y - 1) return;
    __threadfence();
    // Last CTA: the aggregate (reference :51-71), every source inspected and
    // retired, including after the first failure.
    work->input.flags = atomicOr(&work->input.flags, 0u); // the other CTAs' ORs, read at L2
    work->output.flags = atomicOr(&work->output.flags, 0u);
    work->input.done = work->output.done = SACC_SCAN_DONE;
    std::uint32_t flags = 0;
    for (unsigned i = 0; i < SACC_MODEL_PRODUCER_PLUGINS + 2; ++i) {
        SaccScanStatus* source = i < SACC_MODEL_PRODUCER_PLUGINS ? in.plugin[i]
                                 : i == SACC_MODEL_PRODUCER_PLUGINS ? &work->input
                                                                    : &work->output;
        const std::uint32_t f = source->flags, d = source->done;
        if (f != 0) flags |= SACC_POSTPROCESS_NUMERIC;
        if (d != SACC_SCAN_DONE || (f & ~allowed_bits(i)) != 0) flags |= SACC_POSTPROCESS_PROTOCOL;
        source->flags = 0;
        source->done = 0;
    }
    work->arrivals = 0;
    producer->flags = flags;
    __threadfence();
    producer->done = SACC_PRODUCER_DONE;
}

} // namespace

std::size_t producer_workspace_bytes() { return sizeof(Workspace); }

cudaError_t launch_model_producer(const ProducerLaunch& p, SaccProducerStatus* producer, void* workspace, int sms, cudaStream_t s) {
    auto* work = static_cast<Workspace*>(workspace);
    cudaError_t e = launch_pdl_k(producer_initialize_kernel, dim3(1), dim3(1), 0, s, producer, work);
    if (e != cudaSuccess) return e;
    unsigned long long most = 0;
    for (unsigned long long c : p.count) most = c > most ? c : most;
    // Enough CTAs per tensor for the largest one at 8 elements a thread, at
    // most two per SM each.
    unsigned long long x = (most + kThreads * 8 - 1) / (kThreads * 8);
    const unsigned long long cap = static_cast<unsigned long long>(sms > 0 ? sms : 148) * 2;
    x = x == 0 ? 1 : x < cap ? x : cap;
    return launch_pdl_k(producer_check_kernel, dim3(static_cast<unsigned>(x), 7), dim3(kThreads), 0, s, p, producer, work);
}

cudaError_t load_producer_kernels(std::string& report) {
    const std::pair<const char*, const void*> kernels[] = {
        {"producer_initialize", reinterpret_cast<const void*>(producer_initialize_kernel)},
        {"producer_check", reinterpret_cast<const void*>(producer_check_kernel)}};
    for (const auto& [name, fn] : kernels) {
        cudaFuncAttributes attr{};
        const cudaError_t e = cudaFuncGetAttributes(&attr, fn);
        if (e != cudaSuccess) return e;
        report += std::string("kernel=") + name + " registers=" + std::to_string(attr.numRegs) +
                  " local_bytes=" + std::to_string(attr.localSizeBytes) + "\n";
    }
    return cudaSuccess;
}

} // namespace sacc
