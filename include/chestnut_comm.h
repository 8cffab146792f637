/* Clip-end result gather over NCCL (libcncomm.so), one process per GPU.
 *
 * Clips are the only axis the frame path shards on: each rank runs its own
 * clips with no per-frame exchange, and once, at clip end, every rank's
 * per-clip results are all-gathered (NCCL over NVLink / NVSwitch).  The
 * reference has no multi-GPU path; this is the gather at the end of the
 * clip-parallel form of its per-clip loop (video_check.py:50-66).
 *
 * The library is separate from libchestnut.so so that the frame engine does
 * not load NCCL.  Every call returns a status (0 = success, negative =
 * error; cn_comm_last_error() explains the last failure on this thread) and
 * never aborts the process.  A rank that does not arrive makes init or a
 * gather return CN_COMM_ERR_TIMEOUT after timeout_ms instead of hanging: the
 * communicator is then aborted and must be destroyed.
 */
#ifndef CHESTNUT_COMM_H
#define CHESTNUT_COMM_H
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CN_COMM_ID_BYTES 128
#define CN_COMM_ERR_ARG (-2)
#define CN_COMM_ERR_CUDA (-3)
#define CN_COMM_ERR_NCCL (-4)
#define CN_COMM_ERR_TIMEOUT (-5)

typedef struct cn_comm cn_comm;

const char* cn_comm_last_error(void);
/* NCCL version the library runs with (e.g. 22809). */
int cn_comm_nccl_version(int* version);
/* A fresh rendezvous id (rank 0 makes it; the host hands the bytes to every rank). */
int cn_comm_unique_id(void* id /* CN_COMM_ID_BYTES */);
/* Join the communicator of nranks processes; device = this rank's GPU.  Waits at
 * most timeout_ms for the other ranks. */
int cn_comm_init(cn_comm** out, int device, int nranks, int rank, const void* id, int timeout_ms);
/* recv[r * count + i] = rank r's send[i] on every rank (host buffers, f64).
 * Synchronous: returns once recv holds the gathered values. */
int cn_comm_allgather_f64(cn_comm* c, const double* send, double* recv, size_t count, int timeout_ms);
int cn_comm_destroy(cn_comm* c);

#ifdef __cplusplus
}
#endif
#endif
