/* sacc_frame.h -- consumers of the scan status words: the frame-end protocol
 * that gates a frame's payload on its plugins' statuses, and the model
 * producer's status aggregate.  C ABI of libsacc_scan.so; the status words
 * themselves (SaccScanStatus, SACC_SCAN_*) are declared in sacc_scan.h.
 *
 * Each entry replaces, with the same semantics:
 *   SaccScanFrameControl / Record / StatusList
 *                                 include/saccade/scan_frame_kernels.hpp:20-47
 *   sacc_scan_frame_load_kernels  scan_frame_load_kernels,  cuda/scan_frame.cu:144-158
 *   sacc_scan_frame_initialize    scan_frame_initialize,    cuda/scan_frame.cu:160-163 (kernel :29-36)
 *   sacc_scan_frame_begin         scan_frame_begin,         cuda/scan_frame.cu:164-167 (kernel :38-46)
 *   sacc_scan_frame_gate          scan_frame_gate,          cuda/scan_frame.cu:168-172 (kernel :48-68)
 *   sacc_scan_frame_publish       scan_frame_publish,       cuda/scan_frame.cu:173-179 (kernel :70-89)
 *   sacc_scan_frame_commit        scan_frame_commit,        cuda/scan_frame.cu:180-183 (kernel :91-104)
 *   sacc_scan_frame_packet        scan_frame_packet,        cuda/scan_frame.cu:184-187 (kernel :112-127)
 *   sacc_scan_frame_check_finite  scan_frame_check_finite,  cuda/scan_frame.cu:188-195 (kernels :129-138)
 *   sacc_scan_frame_delay         scan_frame_delay,         cuda/scan_frame.cu:196-199
 *   sacc_scan_frame_digest        scan_frame_digest,        cuda/scan_frame.cu:201-209
 *   sacc_model_producer_*         model_producer_cuda*,     cuda/model_producer.cu:117-196,
 *                                 include/saccade/model_producer_cuda.hpp:10-61
 * plus one entry without a reference counterpart:
 *   sacc_scan_frame_step          begin + gate + publish + commit + packet of
 *                                 one frame as ONE launch (same state changes,
 *                                 records and packet bytes as the five calls).
 *
 * Every call is asynchronous on the caller's stream, allocates nothing and
 * never synchronizes; rejections return SACC_EINVAL before any GPU work
 * (sacc_last_error() gives the message). */
#ifndef SACC_FRAME_H
#define SACC_FRAME_H

#include <stddef.h>
#include <stdint.h>

#include "sacc_scan.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------- frame protocol */

#define SACC_FRAME_MAX_STATUSES 16u
/* Status flags of the frame's own finite checks (known to the gate). */
#define SACC_FRAME_NONFINITE_INPUT (1u << 20)
#define SACC_FRAME_NONFINITE_OUTPUT (1u << 21)
/* Frame error bits (include/saccade/protocol.hpp:20-23). */
#define SACC_ERROR_PROTOCOL (1u << 0)
#define SACC_ERROR_NUMERIC (1u << 3)
/* ResultPacket v1 sizes (include/saccade/protocol.hpp:15-18). */
#define SACC_PACKET_CAPACITY 256u
#define SACC_PACKET_HEADER_BYTES 80u
#define SACC_PACKET_ROW_BYTES 48u
#define SACC_PACKET_BYTES (SACC_PACKET_HEADER_BYTES + SACC_PACKET_CAPACITY * SACC_PACKET_ROW_BYTES)

/* Device-resident control block of one frame stream; not a wire ABI.  The
 * first eleven fields are the reference's; `arrivals` and `digest_sum` are the
 * fused step's scratch (zero between calls). */
typedef struct SaccScanFrameControl {
    uint64_t epoch;
    int64_t current, committed, fail_frame;
    uint32_t committed_slot, working_slot, frame_status, fail_code, run_stage, published;
    uint32_t scan_flags; /* OR of every flags word the gate read (diagnostic) */
    uint32_t arrivals;
    uint64_t digest_sum;
} SaccScanFrameControl;

/* What the gate read and the publish copied for one frame (diagnostic). */
typedef struct SaccScanFrameRecord {
    uint32_t flags[SACC_FRAME_MAX_STATUSES];
    uint32_t done[SACC_FRAME_MAX_STATUSES];
    uint32_t frame_status; /* after the gate */
    uint32_t published;    /* 1 when the guarded publish copied the payload */
    uint64_t digest;       /* order-independent digest of the copied payload bits */
} SaccScanFrameRecord;

/* Device pointers to one engine slot's status outputs (host struct). */
typedef struct SaccScanStatusList {
    SaccScanStatus* status[SACC_FRAME_MAX_STATUSES];
    unsigned count;
} SaccScanStatusList;

int sacc_scan_frame_load_kernels(char* report, size_t report_bytes);
/* Resets the control block for `epoch`: nothing committed (committed = -1,
 * committed_slot = 1), no failure; result_frames[0..1] = -1. */
int sacc_scan_frame_initialize(SaccScanFrameControl* control, uint64_t epoch, int64_t* result_frames, cudaStream_t stream);
/* Starts `frame`: PROTOCOL unless the epoch matches and (before a failure)
 * frame == committed + 1. */
int sacc_scan_frame_begin(SaccScanFrameControl* control, uint64_t epoch, int64_t frame, cudaStream_t stream);
/* Reads every status (flags != 0 -> NUMERIC; done != SACC_SCAN_DONE or unknown
 * flag bits or no status at all -> PROTOCOL), retires each to {0, 0}, records
 * what it read in records[frame] when 0 <= frame < capacity, and decides
 * whether the publish runs.  At most SACC_FRAME_MAX_STATUSES statuses. */
int sacc_scan_frame_gate(SaccScanFrameControl* control, const SaccScanStatusList* statuses, SaccScanFrameRecord* records,
                         int64_t capacity, cudaStream_t stream);
/* When the gate passed: copies `count` floats into results + working_slot *
 * count, sets result_frames[working_slot] = frame and adds the digest to the
 * frame's record. */
int sacc_scan_frame_publish(SaccScanFrameControl* control, const float* payload, size_t count, float* results,
                            int64_t* result_frames, SaccScanFrameRecord* records, int64_t capacity, cudaStream_t stream);
/* A passing, published frame becomes the committed version; the first failing
 * frame latches fail_frame / fail_code. */
int sacc_scan_frame_commit(SaccScanFrameControl* control, cudaStream_t stream);
/* The ResultPacket v1 bytes (SACC_PACKET_BYTES; header only, zero rows). */
int sacc_scan_frame_packet(const SaccScanFrameControl* control, unsigned char* packet, cudaStream_t stream);
/* begin + gate + publish + commit (+ packet when `packet` is not NULL) of one
 * frame in one launch.  Needs a control block set by
 * sacc_scan_frame_initialize. */
int sacc_scan_frame_step(SaccScanFrameControl* control, uint64_t epoch, int64_t frame, const SaccScanStatusList* statuses,
                         const float* payload, size_t count, float* results, int64_t* result_frames,
                         SaccScanFrameRecord* records, int64_t capacity, unsigned char* packet, cudaStream_t stream);
/* Clears `status`, ORs `flag` into it when any of the `count` floats is NaN or
 * infinite, then marks it done (a memset and one kernel). */
int sacc_scan_frame_check_finite(const float* data, size_t count, SaccScanStatus* status, uint32_t flag, cudaStream_t stream);
/* A one-thread busy wait of `cycles` SM clocks (stress of slot ownership). */
int sacc_scan_frame_delay(unsigned cycles, cudaStream_t stream);
/* Host twin of the publish digest. */
uint64_t sacc_scan_frame_digest(const float* payload, size_t count);

/* ---------------------------------------------------- model producer status */

#define SACC_MODEL_PRODUCER_PLUGINS 9u         /* P3, P4, P5 x (expand, scan, merge) */
#define SACC_PRODUCER_DONE 0x34525046u         /* "FPR4" */
#define SACC_POSTPROCESS_NUMERIC (1u << 0)
#define SACC_POSTPROCESS_UPSTREAM (1u << 1)
#define SACC_POSTPROCESS_PROTOCOL (1u << 2)
#define SACC_PROFILE_T01_640X640 0              /* include/saccade/model_profile.hpp:37 */
#define SACC_PROFILE_HR_1280X768 1              /* include/saccade/model_profile.hpp:38 */

typedef struct SaccProducerStatus {
    uint32_t flags, done;
} SaccProducerStatus;

/* NCHW FP32 detector outputs, one pointer / element count per level
 * (cls: 80 x H x W, reg: 4 x H x W of the profile's three levels). */
typedef struct SaccRawView {
    const float* cls[3];
    const float* reg[3];
    size_t cls_elements[3];
    size_t reg_elements[3];
} SaccRawView;

size_t sacc_model_producer_workspace_bytes(void);
int sacc_model_producer_load_kernels(char* report, size_t report_bytes);
/* Checks every image and raw element for NaN / Inf, gates the nine plugin
 * statuses (scan plugins, i % 3 == 1, may carry input and range bits; the
 * Cross-Scan plugins only SACC_CROSS_SCAN_NONFINITE_INPUT) and both finite
 * checks, retires them to {0, 0}, then writes producer->flags and only then
 * producer->done = SACC_PRODUCER_DONE.  Any source flags -> NUMERIC; a
 * missing done or a bit outside the source's role -> PROTOCOL.  All 18 ranges
 * must be disjoint device memory of the current device. */
int sacc_model_producer_cuda(const float* images, size_t image_elements, const SaccRawView* raw,
                             SaccScanStatus* const plugins[SACC_MODEL_PRODUCER_PLUGINS], SaccProducerStatus* producer,
                             void* workspace, size_t workspace_bytes, cudaStream_t stream, int profile);

#ifdef __cplusplus
}
#endif

#endif /* SACC_FRAME_H */
