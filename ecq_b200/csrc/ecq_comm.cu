// ecq_comm.cu -- the tensor-parallel exchange's host plumbing (exchange
// buffers, CUDA IPC) and its consumer kernel. The producer side is the fused
// GEMV's TP mode (ecq_gemv_tp, ecq_device.cu). Layout and protocol:
// include/ecq_comm.h.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>

#include "ecq_comm.h"
#include "ecq_kernels.cuh"

namespace {

using ecq_dev::launch_pdl;
using ecq_dev::pdl_launch_dependents;
using ecq_dev::pdl_wait;

constexpr uint64_t kFlagWaitNs = 1000ull * 1000ull * 1000ull;  // 1 s

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* addr) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
    return v;
}

// Sum over ranks of slot i of epoch half `slot` (want = e + 1 in the high
// halves): every rank's word is loaded first and only then checked, so an
// element costs one round trip to memory, not one per rank; a word not yet
// written is polled again until it is or the wait gives up (bounded, shared
// flag, status bit).
__device__ __forceinline__ float sum_ranks(const uint64_t* slot, const ecq_tp_comm& c, int i, uint32_t want,
                                           uint64_t t0, uint32_t* gave_up, uint32_t* status) {
    uint64_t v[ECQ_TP_MAX_RANKS];
#pragma unroll
    for (int r = 0; r < ECQ_TP_MAX_RANKS; ++r)
        if (r < static_cast<int>(c.world)) v[r] = ld_relaxed_sys_u64(slot + static_cast<size_t>(r) * c.n_max + i);
    float d = 0.f;
#pragma unroll
    for (int r = 0; r < ECQ_TP_MAX_RANKS; ++r) {
        if (r < static_cast<int>(c.world)) {
            while (static_cast<uint32_t>(v[r] >> 32) != want) {
                if (*reinterpret_cast<volatile uint32_t*>(gave_up)) break;
                if (global_timer_ns() - t0 > kFlagWaitNs) {
                    *gave_up = 1u;
                    atomicOr(status, ECQ_STATUS_TIMEOUT);
                    break;
                }
                v[r] = ld_relaxed_sys_u64(slot + static_cast<size_t>(r) * c.n_max + i);
            }
            d += __uint_as_float(static_cast<uint32_t>(v[r]));
        }
    }
    return d;
}

using ecq_dev::cluster_rank;
using ecq_dev::cluster_size;
using ecq_dev::cluster_sync;
using ecq_dev::launch_pdl_cluster;
using ecq_dev::ld_cluster_f32;

// The consumers run as ONE thread-block cluster of kCluster CTAs: CTA rank r
// owns the r-th contiguous chunk of the n elements. Cross-CTA steps use the
// hardware cluster barrier and distributed shared memory, not global atomics
// or spin waits: the RMSNorm's sum of squares is each CTA's partial in its
// shared memory, read by every CTA in rank order (deterministic), and after a
// final barrier -- every CTA has read its slots and every partial -- rank 0
// advances the epoch.
constexpr int kCluster = 8;
constexpr int kConsumerThreads = 256;

__global__ void __launch_bounds__(kConsumerThreads) tp_add_rmsnorm_kernel(const __half* h, ecq_tp_comm c,
                                                                          const __half* __restrict__ w, __half* h_out,
                                                                          __half* __restrict__ y, int n, float eps,
                                                                          uint32_t* __restrict__ status) {
    extern __shared__ float buf[];  // this CTA's chunk + 32 warp partials
    __shared__ uint32_t s_epoch, s_gave_up;
    __shared__ float s_part;
    uint32_t* epoch = static_cast<uint32_t*>(c.local);
    const uint32_t cr = cluster_rank(), cn = cluster_size();
    const int chunk = (n + static_cast<int>(cn) - 1) / static_cast<int>(cn);
    const int i0 = static_cast<int>(cr) * chunk;
    const int i1 = min(n, i0 + chunk);
    pdl_launch_dependents();
    pdl_wait();  // h and this rank's epoch come from the kernels before this one
    if (threadIdx.x == 0) {
        s_epoch = *reinterpret_cast<volatile uint32_t*>(epoch);
        s_gave_up = 0u;
    }
    __syncthreads();
    const uint32_t e = s_epoch;
    const uint64_t* slot = reinterpret_cast<const uint64_t*>(static_cast<const uint8_t*>(c.local) + 256u) +
                           static_cast<size_t>(e & 1u) * c.world * c.n_max;
    const uint64_t t0 = global_timer_ns();
    float ss = 0.f;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const float d = sum_ranks(slot, c, i, e + 1u, t0, &s_gave_up, status);
        const float v = __half2float(__float2half_rn(__half2float(h[i]) + __half2float(__float2half_rn(d))));
        buf[i - i0] = v;
        h_out[i] = __float2half_rn(v);
        ss += v * v;
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    float* red = buf + chunk;
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) s_part = v;
    }
    cluster_sync();  // every CTA's partial sum of squares is in its shared memory
    float tot = 0.f;
    for (uint32_t r = 0; r < cn; ++r) tot += ld_cluster_f32(&s_part, r);
    const float rs = rsqrtf(tot / n + eps);
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x)
        y[i] = __hmul(__float2half_rn(buf[i - i0] * rs), w[i]);
    cluster_sync();  // every slot and every partial has been read
    if (cr == 0 && threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(epoch) = e + 1u;
}

// y[i] = sum over ranks of this rank's epoch-e slots (rank order, fp32,
// rounded once to fp16), waiting for each slot as above; one cluster, rank 0
// advances the epoch after the final barrier. The plain all-reduce that
// closes a column-sharded GEMV.
__global__ void __launch_bounds__(kConsumerThreads) tp_sum_kernel(ecq_tp_comm c, __half* __restrict__ y, int n,
                                                                  uint32_t* __restrict__ status) {
    __shared__ uint32_t s_epoch, s_gave_up;
    uint32_t* epoch = static_cast<uint32_t*>(c.local);
    const uint32_t cr = cluster_rank(), cn = cluster_size();
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) {
        s_epoch = *reinterpret_cast<volatile uint32_t*>(epoch);
        s_gave_up = 0u;
    }
    __syncthreads();
    const uint32_t e = s_epoch;
    const uint64_t* slot = reinterpret_cast<const uint64_t*>(static_cast<const uint8_t*>(c.local) + 256u) +
                           static_cast<size_t>(e & 1u) * c.world * c.n_max;
    const uint64_t t0 = global_timer_ns();
    for (int i = static_cast<int>(cr * blockDim.x + threadIdx.x); i < n; i += static_cast<int>(cn * blockDim.x)) {
        const float d = sum_ranks(slot, c, i, e + 1u, t0, &s_gave_up, status);
        y[i] = __float2half_rn(d);
    }
    cluster_sync();  // every slot of every CTA has been read
    if (cr == 0 && threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(epoch) = e + 1u;
}

bool comm_ok(const ecq_tp_comm* c) {
    if (!c || c->world < 1 || c->world > ECQ_TP_MAX_RANKS || c->rank >= c->world || !c->local) return false;
    for (uint32_t q = 0; q < c->world; ++q)
        if (!c->peers[q]) return false;
    return c->peers[c->rank] == c->local;
}

static_assert(sizeof(cudaIpcMemHandle_t) == ECQ_IPC_HANDLE_BYTES, "CUDA IPC handle size");

}  // namespace

extern "C" {

int64_t ecq_comm_buffer_bytes(uint32_t n_max, uint32_t world) {
    if (n_max == 0 || world < 1 || world > ECQ_TP_MAX_RANKS) return ECQ_ERR_ARG;
    return 256 + 2ll * world * n_max * static_cast<int64_t>(sizeof(uint64_t));
}

int32_t ecq_comm_alloc(int64_t bytes, void** d_buf) {
    if (!d_buf || bytes <= 0) return ECQ_ERR_ARG;
    *d_buf = nullptr;
    if (cudaMalloc(d_buf, static_cast<size_t>(bytes)) != cudaSuccess) return ECQ_ERR_CUDA;
    if (cudaMemset(*d_buf, 0, static_cast<size_t>(bytes)) != cudaSuccess) {
        cudaFree(*d_buf);
        *d_buf = nullptr;
        return ECQ_ERR_CUDA;
    }
    return ECQ_OK;
}

int32_t ecq_comm_free(void* d_buf) {
    if (!d_buf) return ECQ_ERR_ARG;
    return cudaFree(d_buf) == cudaSuccess ? ECQ_OK : ECQ_ERR_CUDA;
}

int32_t ecq_ipc_get_handle(const void* d_buf, void* handle_out) {
    if (!d_buf || !handle_out) return ECQ_ERR_ARG;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, const_cast<void*>(d_buf)) != cudaSuccess) return ECQ_ERR_CUDA;
    memcpy(handle_out, &h, sizeof(h));
    return ECQ_OK;
}

int32_t ecq_ipc_open(const void* handle, void** d_mapped) {
    if (!handle || !d_mapped) return ECQ_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *d_mapped = nullptr;
    if (cudaIpcOpenMemHandle(d_mapped, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return ECQ_ERR_CUDA;
    return ECQ_OK;
}

int32_t ecq_ipc_close(void* d_mapped) {
    if (!d_mapped) return ECQ_ERR_ARG;
    return cudaIpcCloseMemHandle(d_mapped) == cudaSuccess ? ECQ_OK : ECQ_ERR_CUDA;
}

int32_t ecq_tp_add_rmsnorm_f16(const void* h, const ecq_tp_comm* comm, const void* w, void* h_out, void* y, int32_t n,
                               float eps, uint32_t* d_status, void* stream) {
    if (!h || !w || !h_out || !y || !d_status || !comm_ok(comm) || n < 1 || n > kCluster * 12256 ||
        static_cast<uint32_t>(n) > comm->n_max)
        return ECQ_ERR_ARG;
    const int chunk = (n + kCluster - 1) / kCluster;
    if (!ecq_dev::ensure_smem_limit(reinterpret_cast<const void*>(tp_add_rmsnorm_kernel), (chunk + 32) * 4))
        return ECQ_ERR_CUDA;
    const cudaError_t rc = launch_pdl_cluster(tp_add_rmsnorm_kernel, dim3(kCluster), dim3(kConsumerThreads),
                                              (chunk + 32) * sizeof(float), static_cast<cudaStream_t>(stream),
                                              kCluster, static_cast<const __half*>(h), *comm,
                                      static_cast<const __half*>(w), static_cast<__half*>(h_out),
                                      static_cast<__half*>(y), n, eps, d_status);
    if (rc != cudaSuccess) {
        cudaGetLastError();
        return ECQ_ERR_CUDA;
    }
    return ECQ_OK;
}

int32_t ecq_tp_sum_f16(const ecq_tp_comm* comm, void* y, int32_t n, uint32_t* d_status, void* stream) {
    if (!y || !d_status || !comm_ok(comm) || n < 1 || static_cast<uint32_t>(n) > comm->n_max) return ECQ_ERR_ARG;
    const cudaError_t rc = launch_pdl_cluster(tp_sum_kernel, dim3(kCluster), dim3(kConsumerThreads), 0,
                                              static_cast<cudaStream_t>(stream), kCluster, *comm,
                                              static_cast<__half*>(y), n, d_status);
    if (rc != cudaSuccess) {
        cudaGetLastError();
        return ECQ_ERR_CUDA;
    }
    return ECQ_OK;
}

}  // extern "C"
