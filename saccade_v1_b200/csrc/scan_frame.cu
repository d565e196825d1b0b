// scan_frame.cu -- the frame-end protocol that consumes the scan status words
// (reference cuda/scan_frame.cu, include/saccade/scan_frame_kernels.hpp).
//
// A frame stream keeps one control block in device memory.  Per frame:
// begin (frame number and epoch checks), gate (read every plugin status, map
// it to the frame's error bits, retire it to {0, 0}), a guarded publish of the
// payload into the working one of two result versions, commit (advance the
// committed version or latch the first failure) and the ResultPacket header.
// The reference runs these as five launches, four of them one thread; here the
// five are also one launch (`frame_step_kernel`): every CTA derives the gate's
// decision from the unchanged control block and statuses, copies its share of
// the payload, and the last CTA to arrive (an arrival counter in the control
// block) applies begin, gate, publish, commit and packet to the control block
// in the reference's order, so the state changes, records and packet bytes are
// those of the five calls.  The five single steps are kept for callers that
// interleave their own work between them.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <string>

#include "../../include/sacc_frame.h"
#include "internal.h"
#include "scan_common.cuh"

namespace sacc {
namespace {

using Control = SaccScanFrameControl;
using Record = SaccScanFrameRecord;

constexpr unsigned kThreads = 256;
constexpr std::uint32_t kKnownFlags = SACC_SCAN_INPUT_FAILURES | SACC_SCAN_RANGE_FAILURES | SACC_CROSS_SCAN_NONFINITE_INPUT |
                                      SACC_FRAME_NONFINITE_INPUT | SACC_FRAME_NONFINITE_OUTPUT;

// splitmix64's output function (Steele, Lea and Flood, "Fast splittable
// pseudorandom number generators", 2014): the per-element term of the payload
// digest, (index << 32 | bits) mixed, summed modulo 2^64 (order independent).
__host__ __device__ __forceinline__ std::uint64_t mix64(std::uint64_t x) {
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

// begin's protocol check (reference cuda/scan_frame.cu:45): the epoch must
// match and, before a failure is latched, frames must follow the committed one.
__device__ __forceinline__ std::uint32_t begin_bits(const Control* c, std::uint64_t epoch, std::int64_t frame) {
    return (epoch != c->epoch || (!c->fail_code && frame != c->committed + 1)) ? SACC_ERROR_PROTOCOL : 0u;
}

// The gate's error bits for the statuses as they are (reference :53-63): a
// missing completion or an unknown bit is PROTOCOL, any flag NUMERIC; no
// status at all is PROTOCOL.
__device__ __forceinline__ std::uint32_t gate_bits(const SaccScanStatusList& list) {
    std::uint32_t bits = list.count == 0 ? SACC_ERROR_PROTOCOL : 0u;
    for (unsigned i = 0; i < list.count; ++i) {
        const std::uint32_t flags = list.status[i]->flags, done = list.status[i]->done;
        if (done != SACC_SCAN_DONE) bits |= SACC_ERROR_PROTOCOL;
        if (flags) bits |= SACC_ERROR_NUMERIC;
        if (flags & ~kKnownFlags) bits |= SACC_ERROR_PROTOCOL;
    }
    return bits;
}

__device__ __forceinline__ Record* frame_record(const Control* c, Record* records, std::int64_t capacity) {
    return records && c->current >= 0 && c->current < capacity ? records + c->current : nullptr;
}

// begin: the state changes of reference :38-46.
__device__ void apply_begin(Control* c, std::uint64_t epoch, std::int64_t frame) {
    const std::uint32_t bits = begin_bits(c, epoch, frame);
    c->current = frame;
    c->working_slot = 1u - c->committed_slot;
    c->frame_status = bits;
    c->run_stage = 0;
    c->published = 0;
}

// gate: reference :48-68 (reads, records and retires every status).
__device__ void apply_gate(Control* c, const SaccScanStatusList& list, Record* records, std::int64_t capacity) {
    Record* record = frame_record(c, records, capacity);
    if (record) *record = Record{};
    for (unsigned i = 0; i < list.count; ++i) {
        SaccScanStatus* s = list.status[i];
        const std::uint32_t flags = s->flags, done = s->done;
        if (done != SACC_SCAN_DONE) c->frame_status |= SACC_ERROR_PROTOCOL;
        if (flags) c->frame_status |= SACC_ERROR_NUMERIC;
        if (flags & ~kKnownFlags) c->frame_status |= SACC_ERROR_PROTOCOL;
        c->scan_flags |= flags;
        s->flags = 0;
        s->done = 0; // retired: only the next producer write makes it valid again
        if (record) {
            record->flags[i] = flags;
            record->done[i] = done;
        }
    }
    if (list.count == 0) c->frame_status |= SACC_ERROR_PROTOCOL;
    if (record) record->frame_status = c->frame_status;
    c->run_stage = !c->fail_code && !c->frame_status;
}

// commit: reference :91-104.
__device__ void apply_commit(Control* c) {
    if (!c->fail_code) {
        if (!c->frame_status && !c->published) c->frame_status |= SACC_ERROR_PROTOCOL;
        if (c->frame_status) {
            c->fail_frame = c->current;
            c->fail_code = c->frame_status;
        } else {
            c->committed = c->current;
            c->committed_slot = c->working_slot;
        }
    }
    c->run_stage = 0;
}

__device__ __forceinline__ void put_le(unsigned char* p, std::uint64_t v, int n) {
    for (int i = 0; i < n; ++i) p[i] = static_cast<unsigned char>(v >> (8 * i));
}

// ResultPacket v1 (reference :112-127): zero rows, the 64-byte header fields
// little endian, the rest of the 80-byte header zero.  All threads of the CTA.
__device__ void write_packet(const Control* c, unsigned char* out) {
    for (unsigned i = threadIdx.x; i < SACC_PACKET_BYTES; i += blockDim.x) out[i] = 0;
    __syncthreads();
    if (threadIdx.x) return;
    out[0] = 'S'; out[1] = 'C'; out[2] = 'R'; out[3] = 'P';
    put_le(out + 4, 1, 2);
    put_le(out + 6, SACC_PACKET_HEADER_BYTES, 2);
    put_le(out + 8, SACC_PACKET_BYTES, 4);
    put_le(out + 12, SACC_PACKET_CAPACITY, 4);
    put_le(out + 16, c->epoch, 8);
    put_le(out + 24, static_cast<std::uint64_t>(c->current), 8);
    put_le(out + 32, static_cast<std::uint64_t>(c->committed), 8);
    put_le(out + 40, static_cast<std::uint64_t>(c->fail_frame), 8);
    const std::uint32_t status = !c->fail_code ? 0u : (c->current == c->fail_frame ? 1u : 2u);
    put_le(out + 48, status, 4);
    put_le(out + 56, status == 1 ? c->fail_code : 0u, 4);
    put_le(out + 60, c->fail_code, 4);
}

// Grid-stride copy of the payload with the digest of the copied bits; returns
// the CTA's digest sum in thread 0.
__device__ std::uint64_t copy_digest(const float* payload, unsigned long long count, float* out) {
    __shared__ std::uint64_t part[kThreads / 32];
    std::uint64_t digest = 0;
    const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
    for (unsigned long long i = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
        const float v = payload[i];
        out[i] = v;
        digest += mix64((static_cast<std::uint64_t>(i) << 32) | __float_as_uint(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) digest += __shfl_down_sync(0xffffffffu, digest, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = digest;
    __syncthreads();
    std::uint64_t sum = 0;
    if (threadIdx.x == 0)
        for (unsigned w = 0; w < blockDim.x / 32; ++w) sum += part[w];
    return sum;
}

struct StepParams {
    SaccScanStatusList list;
    const float* payload;
    unsigned long long count;
    float* results;
    std::int64_t* result_frames;
    Record* records;
    std::int64_t capacity;
    unsigned char* packet;
    std::uint64_t epoch;
    std::int64_t frame;
};

// One frame in one launch.  Nothing in the control block or the statuses
// changes until every CTA has arrived, so each CTA's reading of the gate is
// the one the last CTA applies.
__global__ void __launch_bounds__(kThreads) frame_step_kernel(Control* ctl, StepParams p) {
    pdl_wait();
    __shared__ std::uint32_t s_run, s_slot, s_last;
    if (threadIdx.x == 0) {
        const std::uint32_t bits = begin_bits(ctl, p.epoch, p.frame) | gate_bits(p.list);
        s_run = !ctl->fail_code && !bits;
        s_slot = 1u - ctl->committed_slot;
    }
    __syncthreads();
    std::uint64_t digest = 0;
    if (s_run) digest = copy_digest(p.payload, p.count, p.results + static_cast<unsigned long long>(s_slot) * p.count);
    if (threadIdx.x == 0) {
        if (digest) atomicAdd(reinterpret_cast<unsigned long long*>(&ctl->digest_sum), static_cast<unsigned long long>(digest));
        __threadfence();
        s_last = atomicAdd(&ctl->arrivals, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) {
        // Other CTAs' additions were made at L2: read and reset atomically.
        const std::uint64_t total = atomicExch(reinterpret_cast<unsigned long long*>(&ctl->digest_sum), 0ull);
        atomicExch(&ctl->arrivals, 0u);
        apply_begin(ctl, p.epoch, p.frame);
        apply_gate(ctl, p.list, p.records, p.capacity);
        if (ctl->run_stage) {
            // publish's bookkeeping (reference :84-88)
            Record* record = frame_record(ctl, p.records, p.capacity);
            if (record) record->digest += total;
            p.result_frames[ctl->working_slot] = ctl->current;
            ctl->published = 1;
            if (record) record->published = 1;
        }
        apply_commit(ctl);
    }
    if (p.packet) {
        __syncthreads();
        write_packet(ctl, p.packet);
    }
}

// ------------------------------------------------------------ single steps

__global__ void initialize_kernel(Control* ctl, std::uint64_t epoch, std::int64_t* result_frames) {
    pdl_wait();
    if (threadIdx.x || blockIdx.x) return;
    *ctl = Control{};
    ctl->epoch = epoch;
    ctl->current = ctl->committed = ctl->fail_frame = -1;
    ctl->committed_slot = 1;
    result_frames[0] = result_frames[1] = -1;
}

__global__ void begin_kernel(Control* ctl, std::uint64_t epoch, std::int64_t frame) {
    pdl_wait();
    if (threadIdx.x || blockIdx.x) return;
    apply_begin(ctl, epoch, frame);
}

__global__ void gate_kernel(Control* ctl, SaccScanStatusList list, Record* records, std::int64_t capacity) {
    pdl_wait();
    if (threadIdx.x || blockIdx.x) return;
    apply_gate(ctl, list, records, capacity);
}

__global__ void __launch_bounds__(kThreads) publish_kernel(Control* ctl, const float* payload, unsigned long long count, float* results,
                                                            std::int64_t* result_frames, Record* records, std::int64_t capacity) {
    pdl_wait();
    if (!ctl->run_stage) return; // fixed by the gate; this grid never writes it
    const std::uint64_t digest = copy_digest(payload, count, results + static_cast<unsigned long long>(ctl->working_slot) * count);
    if (threadIdx.x) return;
    Record* record = frame_record(ctl, records, capacity);
    if (record && digest) atomicAdd(reinterpret_cast<unsigned long long*>(&record->digest), static_cast<unsigned long long>(digest));
    if (blockIdx.x == 0) {
        result_frames[ctl->working_slot] = ctl->current;
        ctl->published = 1;
        if (record) record->published = 1;
    }
}

__global__ void commit_kernel(Control* ctl) {
    pdl_wait();
    if (threadIdx.x || blockIdx.x) return;
    apply_commit(ctl);
}

__global__ void __launch_bounds__(kThreads) packet_kernel(const Control* ctl, unsigned char* out) {
    pdl_wait();
    write_packet(ctl, out);
}

// Finite check into a status cleared by the caller: CTAs with a NaN or an
// infinity OR the flag in, and the status's done word counts the CTAs that
// have finished; the last one turns it into SACC_SCAN_DONE (a count below the
// grid size is never the done value), so no second launch is needed.
__global__ void __launch_bounds__(kThreads) check_finite_kernel(const float* data, unsigned long long count, SaccScanStatus* status,
                                                                 std::uint32_t flag) {
    pdl_wait();
    bool bad = false;
    const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
    for (unsigned long long i = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride)
        bad = bad || !isfinite(data[i]);
    bad = __syncthreads_or(bad);
    if (threadIdx.x) return;
    if (bad) atomicOr(&status->flags, flag);
    __threadfence();
    if (atomicAdd(&status->done, 1u) == gridDim.x - 1) atomicExch(&status->done, SACC_SCAN_DONE);
}

// A busy wait bounded by `cycles` SM clocks (at most ~2.2 s at 1.97 GHz).
__global__ void delay_kernel(unsigned cycles) {
    pdl_wait();
    const long long start = clock64();
    while (clock64() - start < static_cast<long long>(cycles)) {
    }
}

unsigned grid_for(unsigned long long count, int sms) {
    const unsigned long long blocks = (count + kThreads - 1) / kThreads, cap = static_cast<unsigned long long>(sms > 0 ? sms : 148) * 4;
    return static_cast<unsigned>(blocks == 0 ? 1 : blocks < cap ? blocks : cap);
}

} // namespace

cudaError_t launch_frame_initialize(SaccScanFrameControl* ctl, std::uint64_t epoch, std::int64_t* result_frames, cudaStream_t s) {
    return launch_pdl_k(initialize_kernel, dim3(1), dim3(1), 0, s, ctl, epoch, result_frames);
}

cudaError_t launch_frame_begin(SaccScanFrameControl* ctl, std::uint64_t epoch, std::int64_t frame, cudaStream_t s) {
    return launch_pdl_k(begin_kernel, dim3(1), dim3(1), 0, s, ctl, epoch, frame);
}

cudaError_t launch_frame_gate(SaccScanFrameControl* ctl, const SaccScanStatusList& list, SaccScanFrameRecord* records,
                              std::int64_t capacity, cudaStream_t s) {
    return launch_pdl_k(gate_kernel, dim3(1), dim3(1), 0, s, ctl, list, records, capacity);
}

cudaError_t launch_frame_publish(SaccScanFrameControl* ctl, const float* payload, unsigned long long count, float* results,
                                 std::int64_t* result_frames, SaccScanFrameRecord* records, std::int64_t capacity, int sms,
                                 cudaStream_t s) {
    return launch_pdl_k(publish_kernel, dim3(grid_for(count, sms)), dim3(kThreads), 0, s, ctl, payload, count, results,
                        result_frames, records, capacity);
}

cudaError_t launch_frame_commit(SaccScanFrameControl* ctl, cudaStream_t s) {
    return launch_pdl_k(commit_kernel, dim3(1), dim3(1), 0, s, ctl);
}

cudaError_t launch_frame_packet(const SaccScanFrameControl* ctl, unsigned char* packet, cudaStream_t s) {
    return launch_pdl_k(packet_kernel, dim3(1), dim3(kThreads), 0, s, ctl, packet);
}

cudaError_t launch_frame_step(SaccScanFrameControl* ctl, const FrameStep& f, int sms, cudaStream_t s) {
    StepParams p{f.list, f.payload, f.count, f.results, f.result_frames, f.records, f.capacity, f.packet, f.epoch, f.frame};
    return launch_pdl_k(frame_step_kernel, dim3(grid_for(f.count, sms)), dim3(kThreads), 0, s, ctl, p);
}

cudaError_t launch_frame_check_finite(const float* data, unsigned long long count, SaccScanStatus* status, std::uint32_t flag,
                                      int sms, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(status, 0, sizeof(SaccScanStatus), s);
    if (e != cudaSuccess) return e;
    return launch_pdl_k(check_finite_kernel, dim3(grid_for(count, sms)), dim3(kThreads), 0, s, data, count, status, flag);
}

cudaError_t launch_frame_delay(unsigned cycles, cudaStream_t s) { return launch_pdl_k(delay_kernel, dim3(1), dim3(1), 0, s, cycles); }

std::uint64_t frame_digest(const float* payload, std::size_t count) {
    std::uint64_t digest = 0;
    for (std::size_t i = 0; i < count; ++i) {
        std::uint32_t bits = 0;
        std::memcpy(&bits, payload + i, sizeof bits);
        digest += mix64((static_cast<std::uint64_t>(i) << 32) | bits);
    }
    return digest;
}

cudaError_t load_frame_kernels(std::string& report) {
    const std::pair<const char*, const void*> kernels[] = {
        {"frame_step", reinterpret_cast<const void*>(frame_step_kernel)},
        {"frame_initialize", reinterpret_cast<const void*>(initialize_kernel)},
        {"frame_begin", reinterpret_cast<const void*>(begin_kernel)},
        {"frame_gate", reinterpret_cast<const void*>(gate_kernel)},
        {"frame_publish", reinterpret_cast<const void*>(publish_kernel)},
        {"frame_commit", reinterpret_cast<const void*>(commit_kernel)},
        {"frame_packet", reinterpret_cast<const void*>(packet_kernel)},
        {"frame_check_finite", reinterpret_cast<const void*>(check_finite_kernel)},
        {"frame_delay", reinterpret_cast<const void*>(delay_kernel)}};
    for (const auto& [name, fn] : kernels) {
        cudaFuncAttributes attr{};
        const cudaError_t e = cudaFuncGetAttributes(&attr, fn); // loads the kernel under lazy loading
        if (e != cudaSuccess) return e;
        report += std::string("kernel=") + name + " registers=" + std::to_string(attr.numRegs) +
                  " local_bytes=" + std::to_string(attr.localSizeBytes) + "\n";
    }
    return cudaSuccess;
}

} // namespace sacc
