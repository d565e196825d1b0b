// ref_frame_shim.cpp -- C entry points around the reference's own frame
// protocol and model-producer kernels, for the GPU parity tests.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file with nvcc
// together with the reference's cuda/scan_frame.cu, cuda/model_producer.cu
// and src/postprocess.cpp, taken from where they lie in the reference checkout
// (never copied), into oracle/_ref/libref_frame.so.  The GPU tests run the
// reference kernels and the library's kernels on the same device buffers'
// copies and compare every byte they leave.
//
// Wrapped interfaces: include/saccade/scan_frame_kernels.hpp:49-77 and
// include/saccade/model_producer_cuda.hpp:23-61 (exceptions become -1 with
// the message in ref_frame_error()).
#include "saccade/model_producer_cuda.hpp"
#include "saccade/scan_frame_kernels.hpp"

#include <cstdint>
#include <cstdio>
#include <exception>
#include <string>

namespace {
thread_local std::string g_message;

template <typename F>
int call(F&& f) {
    try {
        f();
        g_message.clear();
        return 0;
    } catch (const std::exception& e) {
        g_message = e.what();
        return -1;
    }
}
} // namespace

extern "C" {

const char* ref_frame_error(void) { return g_message.c_str(); }
size_t ref_frame_control_bytes(void) { return sizeof(saccade::ScanFrameControl); }
size_t ref_frame_record_bytes(void) { return sizeof(saccade::ScanFrameRecord); }

int ref_frame_load(void) { return call([] { (void)saccade::scan_frame_load_kernels(); (void)saccade::model_producer_cuda_load_kernels(); }); }

int ref_frame_initialize(void* ctl, uint64_t epoch, int64_t* result_frames, cudaStream_t s) {
    return call([&] { saccade::scan_frame_initialize(static_cast<saccade::ScanFrameControl*>(ctl), epoch, result_frames, s); });
}

int ref_frame_begin(void* ctl, uint64_t epoch, int64_t frame, cudaStream_t s) {
    return call([&] { saccade::scan_frame_begin(static_cast<saccade::ScanFrameControl*>(ctl), epoch, frame, s); });
}

int ref_frame_gate(void* ctl, void* const* statuses, unsigned count, void* records, int64_t capacity, cudaStream_t s) {
    return call([&] {
        saccade::ScanStatusList list{};
        for (unsigned i = 0; i < count && i < saccade::kScanFrameMaxStatuses; ++i)
            list.status[i] = static_cast<saccade::ScanStatus*>(statuses[i]);
        list.count = count;
        saccade::scan_frame_gate(static_cast<saccade::ScanFrameControl*>(ctl), list, static_cast<saccade::ScanFrameRecord*>(records),
                                 capacity, s);
    });
}

int ref_frame_publish(void* ctl, const float* payload, size_t count, float* results, int64_t* result_frames, void* records,
                      int64_t capacity, cudaStream_t s) {
    return call([&] {
        saccade::scan_frame_publish(static_cast<saccade::ScanFrameControl*>(ctl), payload, count, results, result_frames,
                                    static_cast<saccade::ScanFrameRecord*>(records), capacity, s);
    });
}

int ref_frame_commit(void* ctl, cudaStream_t s) {
    return call([&] { saccade::scan_frame_commit(static_cast<saccade::ScanFrameControl*>(ctl), s); });
}

int ref_frame_packet(const void* ctl, unsigned char* out, cudaStream_t s) {
    return call([&] { saccade::scan_frame_packet(static_cast<const saccade::ScanFrameControl*>(ctl), out, s); });
}

int ref_frame_check_finite(const float* data, size_t count, void* status, uint32_t flag, cudaStream_t s) {
    return call([&] { saccade::scan_frame_check_finite(data, count, static_cast<saccade::ScanStatus*>(status), flag, s); });
}

uint64_t ref_frame_digest(const float* payload, size_t count) { return saccade::scan_frame_digest(payload, count); }

size_t ref_producer_workspace_bytes(void) { return saccade::model_producer_workspace_bytes(); }

int ref_model_producer(const float* images, size_t image_elements, const float* const* cls, const float* const* reg,
                       const size_t* cls_elements, const size_t* reg_elements, void* const* plugins, void* producer,
                       void* workspace, size_t workspace_bytes, cudaStream_t s, int profile) {
    return call([&] {
        saccade::PostprocessRawView raw{};
        saccade::ModelProducerPlugins statuses{};
        for (int l = 0; l < 3; ++l) {
            raw.cls[l] = cls[l];
            raw.reg[l] = reg[l];
            raw.cls_elements[l] = cls_elements[l];
            raw.reg_elements[l] = reg_elements[l];
        }
        for (unsigned i = 0; i < saccade::kModelProducerPlugins; ++i) statuses[i] = static_cast<saccade::ScanStatus*>(plugins[i]);
        saccade::model_producer_cuda(images, image_elements, raw, statuses, static_cast<saccade::PostprocessProducerStatus*>(producer),
                                     workspace, workspace_bytes, s,
                                     profile == 1 ? saccade::ModelProfile::Hr1280x768 : saccade::ModelProfile::T01_640x640);
    });
}

} // extern "C"
