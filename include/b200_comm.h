/*
 * Tensor-parallel exchange over NVLink peer memory: the B200 counterpart of
 * the reference runtime's TCP mesh comm_t (board/tp/tp_llama.cpp:377-526).
 *
 * One communicator per rank (one process per GPU). Each rank owns a window of
 * device memory that every peer maps through CUDA IPC; the handles travel
 * over whatever out-of-band channel the caller has (the reference's own mesh,
 * torch.distributed, a file): export this rank's blob, gather all ranks'
 * blobs in rank order, import them.
 *
 * Collectives run as kernels on a CUDA stream and may be captured in a CUDA
 * graph (the epoch that pairs the ranks' calls lives in device memory). Every
 * rank must make the same calls in the same order, as with the reference's
 * comm_t. Each wait on a peer is bounded (1 s); a wait that runs out sets
 * the value 2 in the status word (b200_comm_status) and the call's output is
 * then not valid. All functions return 0 or a negative errno value; b200_last_error()
 * says why.
 */
#ifndef B200_COMM_H
#define B200_COMM_H

#include <stdint.h>

#ifndef B200_API
#define B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b200_comm b200_comm_t;

/* Replaces comm_t::open (tp_llama.cpp:409-448), minus the sockets: allocate
 * this rank's window on `device` for collectives of up to max_floats floats.
 * nranks <= 8. */
B200_API int b200_comm_create(b200_comm_t **c, int rank, int nranks, int device, int max_floats);
/* Size of the blob b200_comm_export writes. */
B200_API int b200_comm_handle_bytes(void);
B200_API int b200_comm_export(b200_comm_t *c, void *handle);
/* `handles`: nranks blobs of b200_comm_handle_bytes() bytes, in rank order. */
B200_API int b200_comm_import(b200_comm_t *c, const void *handles);

/* Replaces comm_t::allreduce_sum (tp_llama.cpp:504-525): in place, every
 * element becomes p0 + p1 + ... + p{n-1} summed left to right in rank order,
 * the same bits on every rank. v holds len floats (len <= max_floats), on
 * `stream` (a cudaStream_t; NULL: legacy default). */
B200_API int b200_allreduce_sum(b200_comm_t *c, uint64_t v, int len, void *stream);

/* Replaces comm_t::allgather (tp_llama.cpp:482-490): out (nranks * bytes)
 * receives every rank's `bytes` bytes from `in`, in rank order. bytes <= 256
 * and a multiple of 4. */
B200_API int b200_allgather(b200_comm_t *c, uint64_t in, uint64_t out, int bytes, void *stream);

/* The greedy candidate exchange of sample_token (tp_llama.cpp:894-925) for
 * temperature 0: every rank passes its shard's pick (int32 global index,
 * float32 value) at `in`; `out` receives the winner over all ranks -- largest
 * value, lowest index on a tie -- on every rank. */
B200_API int b200_allgather_pick(b200_comm_t *c, uint64_t in, uint64_t out, void *stream);

/* Status word of this communicator: 2 = a wait for a peer ran out.
 * Reading clears it. */
B200_API int b200_comm_status(b200_comm_t *c, unsigned *status);
B200_API int b200_comm_destroy(b200_comm_t *c);

#ifdef __cplusplus
}
#endif
#endif
