/*
 * jstorch_dist.h -- C ABI of the multi-GPU (one process per GPU) GEMM path,
 * library jstorch_b200/libjstorch_dist.so (NCCL over NVLink / NVSwitch).
 *
 * No counterpart in the reference, which is single-GPU only.  These entry
 * points shard the reference's launch_matmul (native/ops/matmul.cu:28) by row
 * blocks of A and launch_bmm (:40) by batch index across the GPUs of a box.
 */
#ifndef JSTORCH_DIST_H
#define JSTORCH_DIST_H

#include "jstorch_gemm.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct jst_comm jst_comm;

#define JST_COMM_ID_BYTES 128

/* Fill `id` with a new communicator id (call on one rank, share the bytes). */
int jst_comm_get_unique_id(unsigned char id[JST_COMM_ID_BYTES]);

/*
 * Create this rank's communicator on the current device.  Non-blocking NCCL
 * initialisation polled against a host deadline of `timeout_s` seconds: if a
 * peer never joins, the call aborts the communicator and returns
 * JST_ERR_TIMEOUT instead of hanging.  The same deadline bounds every later
 * collective of the communicator.
 */
int jst_comm_init(jst_comm** comm, int nranks, int rank, const unsigned char id[JST_COMM_ID_BYTES],
                  double timeout_s);
/*
 * Wait on the host for `stream` to drain, bounded by the communicator's
 * deadline; on expiry (a collective waiting for a rank that is gone) abort the
 * communicator and return JST_ERR_TIMEOUT.  Use instead of
 * cudaStreamSynchronize after sharded calls.
 */
int jst_comm_sync(jst_comm* comm, jst_stream_t stream);
int jst_comm_rank(const jst_comm* comm);
int jst_comm_size(const jst_comm* comm);
/*
 * Timeline of the last row-sharded call (no counterpart in the reference):
 * jst_comm_trace(comm, 1) turns event recording on; after the call and a
 * jst_comm_sync, jst_comm_trace_read fills up to max_entries labels (each up
 * to 31 chars + NUL, 32 bytes apart in `labels`) and millisecond offsets from
 * the call's entry, and returns the number of entries.
 */
int jst_comm_trace(jst_comm* comm, int on);
int jst_comm_trace_read(jst_comm* comm, char* labels, double* ms, int max_entries);
/* Destroy (or, after an error, abort) the communicator and free its streams. */
int jst_comm_destroy(jst_comm* comm);

/*
 * Multicast-backed buffer: `bytes` of device memory on every rank of the
 * communicator, bound to one NVLink-switch multicast object, so that a single
 * store through the multicast address lands in every rank's copy.  Collective:
 * every rank calls it in the same order with the same size.  Needs a device
 * with multicast support (CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED) and all
 * ranks on one node; otherwise returns JST_ERR_UNSUPPORTED.  *local receives
 * this rank's ordinary device pointer to its copy.
 */
typedef struct jst_symm jst_symm;
int jst_symm_alloc(jst_comm* comm, size_t bytes, jst_symm** out, void** local);
/* Collective release (all ranks, after their last use). */
int jst_symm_free(jst_symm* buf);

/*
 * Register `bytes` of this rank's device memory at `ptr` with every rank
 * (collective; CUDA IPC handles are exchanged through the communicator).  A
 * row-sharded GEMM whose C_full lies in a registered buffer delivers each row
 * block with copy-engine writes straight into the other ranks' buffers
 * (no all-gather kernel, no SMs taken from the GEMM) and ends with one
 * barrier.  The memory must come from cudaMalloc (directly or through a
 * caching allocator) and stay allocated until jst_comm_deregister.
 */
typedef struct jst_reg jst_reg;
int jst_comm_register(jst_comm* comm, void* ptr, size_t bytes, jst_reg** out);
/* Collective: all ranks, after their last use of the buffer. */
int jst_comm_deregister(jst_reg* reg);

/*
 * Row-sharded C = A * B over all ranks (every rank receives the full C).
 *   A_local   [M_local, K] row-major on this rank: row block i (chunk_rows rows,
 *             i = 0 .. M_local/chunk_rows - 1) holds global rows
 *             (i * nranks + rank) * chunk_rows + [0, chunk_rows).  With
 *             chunk_rows == M_local this is plain row-block sharding (rank r
 *             owns rows [r*M_local, (r+1)*M_local)).
 *   B         [K, N], valid on `root`; broadcast in place to every rank.
 *   C_full    [M_local * nranks, N] on every rank.
 * Each row block is multiplied with the 3 x TF32 tensor-core kernel straight
 * into its place in C_full; its in-place all-gather runs on a second stream
 * while the next block is computed.  When C_full lies in a registered buffer
 * (jst_comm_register) each block is instead copied by the copy engines into
 * every other rank's buffer.  When C_full lies in a jst_symm buffer the
 * all-gather is fused into the GEMM instead: the kernel's epilogue stores each
 * tile once through the multicast address and the switch delivers it to every
 * rank (no collective for C, one barrier at the end).  Asynchronous on `stream`.
 * M_local must be a multiple of chunk_rows and equal on all ranks.
 */
int jst_gemm_rowsharded(jst_comm* comm, const float* A_local, int M_local, int K, float* B, int N, int root,
                        float* C_full, int chunk_rows, jst_stream_t stream);

/*
 * Batch-sharded C[b] = A[b] * B[b]: this rank holds batches
 * [rank * batch_local, (rank + 1) * batch_local) of A and B (packed, as
 * launch_bmm), computes them into their place in C_full [batch_local * nranks,
 * M, N] and all-gathers C_full in place.  Asynchronous on `stream`.
 */
int jst_bmm_batchsharded(jst_comm* comm, const float* A_local, const float* B_local, int batch_local, int M, int K,
                         int N, float* C_full, jst_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* JSTORCH_DIST_H */
