/* sacc_shard.h -- batch-sharded selective scan over the GPUs of one process,
 * for C and C++ hosts (no counterpart in the reference, which runs one head
 * per GPU; the sharding follows its batch-independence contract: every
 * (batch, channel) lane is its own recurrence, src/selective_scan.cpp:61-109).
 *
 * One host process drives `ndev` GPUs.  Every shard is a contiguous slice of
 * the batch (tracks, sequences) on its own device; the scan path has no
 * collective: each device scans its slice with the same kernels as
 * sacc_selective_scan_ex.  Only the optional output assembly crosses devices,
 * as one NCCL all-gather over NVLink (ncclAllGather inside
 * ncclGroupStart/ncclGroupEnd, one communicator per device from
 * ncclCommInitAll).  NCCL (libnccl.so.2) is loaded when the first group is
 * created; the rest of the library does not need it.
 *
 * Same return codes and sacc_last_error() text as sacc_scan.h.
 * ------------------------------------------------------------------------ */
#ifndef SACC_SHARD_H
#define SACC_SHARD_H

#include <stddef.h>
#include <stdint.h>

#include "sacc_scan.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Contiguous split of `total` rows over `world` shards, as
 * saccade_v1_b200/shard.py splits them: shard `rank` gets rows
 * [*row0, *row0 + *rows); the first total % world shards get one row more. */
int sacc_shard_rows(uint64_t total, int world, int rank, uint64_t* row0, uint64_t* rows);

typedef struct SaccShardGroup SaccShardGroup; /* opaque */

/* A group of `ndev` devices (CUDA ordinals devices[0..ndev-1], distinct) with
 * one NCCL communicator each.  Collective across the devices: call once, from
 * one host thread.  The caller's current device is restored. */
int sacc_shard_group_create(int ndev, const int* devices, SaccShardGroup** group);

/* Frees the communicators (after the work enqueued on them has completed:
 * synchronise the streams first). */
int sacc_shard_group_destroy(SaccShardGroup* group);

/* One batch-sharded scan: args[i] describes shard i entirely on device
 * devices[i] (its tensors live there; its batch is the shard's rows),
 * enqueued on streams[i] (an explicit stream of that device).  Every shard is
 * validated first, with sacc_selective_scan_ex's rules; if any is rejected
 * (SACC_EINVAL, the message names the shard) nothing is enqueued on any
 * device.  With gather non-null, every device i also receives the
 * concatenation of all shards' y, in shard order, in gather[i] (a device
 * buffer of ndev * shard_y_bytes bytes on device i), by one NCCL all-gather
 * on the same streams; every shard's y must then hold exactly shard_y_bytes
 * bytes (equal shards).  Returns once everything is enqueued: no host
 * synchronisation. */
int sacc_scan_sharded_forward(SaccShardGroup* group, const SaccScanExArgs* args, const cudaStream_t* streams,
                              void* const* gather, size_t shard_y_bytes);

#ifdef __cplusplus
}
#endif

#endif /* SACC_SHARD_H */
