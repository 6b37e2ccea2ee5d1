/*
 * b200_shard.h - the gather step of kv-head-sharded attention across the GPUs of one node, as one
 * kernel of peer stores over NVLink.
 *
 * The reference runs every node on one device (rust/src/device.rs:85-170: one MLX GPU stream);
 * this build shards the paged-attention path by kv head: rank r of N owns kv heads
 * [r*KV/N, (r+1)*KV/N) and the q heads that read them, so append and attention need no
 * cross-rank traffic, and rank r's output is [rows, H/N*d].  The consumer wants [rows, H*d] on
 * every rank: an all-gather plus a head permute.  b200_shard_gather does both at once: every rank
 * stores its slice straight into every rank's [rows, H*d] output at column offset r*H/N*d (plain
 * 16-byte peer stores over NVLink; no multicast, no NVLS), between two barriers on flag words in
 * peer memory:
 *   - entry: a rank writes its slice into a peer's output only after that peer has reached the
 *     same call (so the peer's previous output has been consumed: its stream runs the consumer
 *     before this call);
 *   - exit: the call completes on a rank only after every rank's slice has landed there.
 * Every wait is bounded (1 s by %globaltimer); a timeout sets B200 status bit 1 << 5 in
 * `status` and the call completes without the data, so a rank that never arrives cannot hang
 * the others.  The kernel needs no host synchronisation, so a CUDA graph can capture it.
 *
 * Set-up (once per output shape): each rank allocates its output and flag buffers with
 * b200_ep_device_alloc (whole allocations: an IPC handle names an allocation), zeroes the flag
 * and state words, exchanges b200_ipc_get_handle() handles with the other ranks (any host
 * channel; torch.distributed in the Python binding) and opens the peers' handles with
 * b200_ipc_open_handle().  All ranks call b200_shard_gather the same number of times, in the
 * same order, with the same rows / slice_bytes.
 */
#ifndef B200_SHARD_H
#define B200_SHARD_H

#include <stddef.h>
#include <stdint.h>

#include "b200_paged.h"

#ifdef __cplusplus
extern "C" {
#endif

#define B200_SHARD_MAX_RANKS 8

typedef struct B200ShardGatherParams {
  int32_t world;            /* ranks, 1..B200_SHARD_MAX_RANKS                                   */
  int32_t rank;             /* this rank                                                        */
  int32_t rows;             /* rows of every output (tokens)                                    */
  int32_t slice_bytes;      /* bytes of one row's slice on one rank (H/N * d * element size),
                               a multiple of 16                                                 */
  const void* local;        /* this rank's [rows, slice_bytes] output, 16-byte aligned           */
  void* outputs[B200_SHARD_MAX_RANKS]; /* every rank's [rows, world * slice_bytes] output:
                               this rank's own buffer at [rank], opened peer handles elsewhere  */
  uint32_t* flags[B200_SHARD_MAX_RANKS]; /* every rank's 2 * world flag words (zero at set-up),
                               the same way                                                      */
  uint32_t* state;          /* this rank's 2 device words (zero at set-up): call count, CTA count */
  int32_t* status;          /* this rank's device status word (B200 status bits), or NULL        */
  int32_t num_sms;          /* 0 = query the device                                              */
} B200ShardGatherParams;

/* sizeof(B200ShardGatherParams), for binding layout checks. */
B200_API int b200_shard_gather_params_size(void);

/* One gather (see above), enqueued on `stream`.  B200_ERR_INVALID_ARGUMENT for bad geometry or
 * missing pointers. */
B200_API int b200_shard_gather(const B200ShardGatherParams* p, void* stream);

/* CUDA IPC of device allocations for the set-up: the handle size in bytes, the handle of an
 * allocation made by b200_ep_device_alloc (its base pointer), a peer's handle opened on
 * `device` (peer access enabled lazily), and closing an opened handle. */
B200_API int b200_ipc_handle_size(void);
B200_API int b200_ipc_get_handle(const void* base, void* handle);
B200_API int b200_ipc_open_handle(int32_t device, const void* handle, void** ptr);
B200_API int b200_ipc_close_handle(int32_t device, void* ptr);

#ifdef __cplusplus
}
#endif

#endif /* B200_SHARD_H */
