/*
 * ecq_comm.h -- the tensor-parallel exchange of a batch-1 decode step, fused
 * into the kernels on either side of it: the row-parallel fused GEMV pushes
 * its fp32 partial y straight into every peer GPU's receive buffer over
 * NVLink (plain peer stores into CUDA-IPC-mapped memory, no multicast), each
 * value stored together with its epoch in one 8-byte word; the next kernel
 * (residual add + RMSNorm) polls those words with a bounded wait and sums the
 * partials in rank order. It replaces the NCCL all-reduce
 * (sum) that closes every row-parallel layer of the tensor-parallel step
 * (the reference's model glue lives in its MLX fork; the layer structure is
 * experiments/real_model_test.py:18-113).
 *
 * Every rank allocates one exchange buffer (ecq_comm_alloc), publishes its
 * CUDA IPC handle to the others (any host transport), opens theirs
 * (ecq_ipc_open) and fills an ecq_tp_comm with the device addresses. All
 * ranks must then issue the same sequence of ecq_gemv_tp / consumer calls.
 */
#ifndef ECQ_COMM_H
#define ECQ_COMM_H

#include <stdint.h>

#include "ecq.h"

#ifdef __cplusplus
extern "C" {
#endif

#define ECQ_TP_MAX_RANKS 8
#define ECQ_IPC_HANDLE_BYTES 64

/* Exchange-buffer layout (bytes from its base): [0, 4) this rank's epoch
 * counter; [256, ...) slots[2][world][n_max], u64, written by the ranks:
 * fp32 value bits | (epoch + 1) << 32. Index [e & 1] alternates with the
 * epoch e; a slot is valid for epoch e once its high half reads e + 1. The
 * consumers run as one thread-block cluster of 8 CTAs of 256 threads, each
 * CTA a contiguous chunk of the elements; they combine through distributed
 * shared memory and the cluster barrier, and rank 0 advances the epoch after
 * every CTA has read its slots. */
typedef struct ecq_tp_comm {
    uint32_t world;   /* ranks, 1..ECQ_TP_MAX_RANKS */
    uint32_t rank;    /* this rank */
    uint32_t n_max;   /* partial length the buffers hold */
    uint32_t reserved;
    void *local;                          /* this rank's exchange buffer */
    void *peers[ECQ_TP_MAX_RANKS];        /* every rank's buffer, mapped here (peers[rank] == local) */
} ecq_tp_comm;

/* Size of one exchange buffer for partials of up to n_max values. */
int64_t ecq_comm_buffer_bytes(uint32_t n_max, uint32_t world);

/* Allocate and zero an exchange buffer on the current device (cudaMalloc, so
 * that it can be exported whole); ecq_comm_free releases it. */
int32_t ecq_comm_alloc(int64_t bytes, void **d_buf);
int32_t ecq_comm_free(void *d_buf);

/* CUDA IPC: export a cudaMalloc'd buffer, open a peer's export here (with
 * lazy peer access), close an opened mapping. */
int32_t ecq_ipc_get_handle(const void *d_buf, void *handle_out /* ECQ_IPC_HANDLE_BYTES */);
int32_t ecq_ipc_open(const void *handle /* ECQ_IPC_HANDLE_BYTES */, void **d_mapped);
int32_t ecq_ipc_close(void *d_mapped);

/* The fused GEMV of a row-parallel layer at batch 1 (x [cols], scales as for
 * ecq_gemv): instead of writing y, each row's fp32 sum goes to
 * slots[e & 1][rank][row] on every rank as (value, e + 1) in one 8-byte store
 * (e = this rank's epoch). rows <= n_max. The workspace is ecq_gemv_workspace_bytes(m, 1) bytes. */
int32_t ecq_gemv_tp(const ecq_matrix_view *m, const void *x_f16, const void *scales_f16, const ecq_tp_comm *comm,
                    void *workspace, int64_t workspace_bytes, uint32_t *d_status, void *stream);

/* The consumer: wait (bounded, ~1 s; ECQ_STATUS_TIMEOUT on expiry) until
 * every rank's slots [e & 1][r][0..n) read e + 1 (e = this rank's epoch), then
 * d = sum over ranks of their values (rank order, fp32, rounded once to fp16),
 * h_out = h + d and y = rmsnorm(h_out) * w as ecq_add_rmsnorm_f16 does for
 * one row (the sum of squares is added over the CTAs' chunks in a fixed
 * order), and advance the epoch. n <= n_max, n <= 98048. After a timeout
 * the ranks' epochs may disagree: the results are unusable and every rank
 * must rebuild its exchange buffer before the next exchange. */
int32_t ecq_tp_add_rmsnorm_f16(const void *h, const ecq_tp_comm *comm, const void *w, void *h_out, void *y, int32_t n,
                               float eps, uint32_t *d_status, void *stream);

/* The plain consumer: y[0..n) = sum over ranks of this rank's epoch-e slots
 * (rank order, fp32, rounded once to fp16), waiting as above, then advance
 * the epoch. ecq_gemv_tp followed by this is a column-sharded GEMV with its
 * all-reduce fused in. n <= n_max. */
int32_t ecq_tp_sum_f16(const ecq_tp_comm *comm, void *y, int32_t n, uint32_t *d_status, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ECQ_COMM_H */
