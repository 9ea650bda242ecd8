// ecq_glue.cu -- the element-wise steps between the fused GEMVs of a
// transformer decode step, one kernel each, so a batch-1 step launches a
// handful of kernels per layer instead of dozens of framework ops:
//   ecq_add_rmsnorm_f16  h += d; y = rmsnorm(h) * w          (one CTA per row)
//   ecq_rope_kv_f16      rotate q and k, store k and v into the KV cache slot
//   ecq_silu_mul_f16     m = silu(gate) * up                  (gate|up packed)
// fp16 in/out, fp32 arithmetic.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ecq_glue.h"
#include "ecq_kernels.cuh"

namespace {

using ecq_dev::launch_pdl;
using ecq_dev::pdl_launch_dependents;
using ecq_dev::pdl_wait;

__global__ void add_rmsnorm_kernel(const __half* __restrict__ h, const __half* __restrict__ d,
                                   const __half* __restrict__ w, __half* __restrict__ h_out, __half* __restrict__ y,
                                   int n, float eps) {
    extern __shared__ float buf[];  // n floats + 32 partials
    pdl_launch_dependents();
    pdl_wait();  // h and d come from the kernels before this one
    const size_t row = blockIdx.x;
    h += row * n;
    if (d) d += row * n;
    h_out += row * n;
    y += row * n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = __half2float(h[i]);
        if (d) v = __half2float(__float2half_rn(v + __half2float(d[i])));  // the residual is stored in fp16
        buf[i] = v;
        ss += v * v;
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    float* part = buf + n;
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) part[0] = rsqrtf(v / n + eps);
    }
    __syncthreads();
    const float r = part[0];
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = buf[i];
        if (d) h_out[i] = __float2half_rn(v);
        y[i] = __hmul(__float2half_rn(v * r), w[i]);
    }
}

// One row on one thread-block cluster of kRowCluster CTAs: CTA rank r takes
// the r-th chunk of the row; the sum of squares is each CTA's partial in its
// shared memory, read by every CTA in rank order after the cluster barrier
// (deterministic, no global atomics).
constexpr int kRowCluster = 8;
constexpr int kRowThreads = 256;

__global__ void __launch_bounds__(kRowThreads) add_rmsnorm_row_cluster_kernel(
    const __half* h, const __half* __restrict__ d, const __half* __restrict__ w, __half* h_out,
    __half* __restrict__ y, int n, float eps) {
    extern __shared__ float buf[];  // this CTA's chunk + 32 warp partials (h_out may be h)
    __shared__ float s_part;
    const uint32_t cr = ecq_dev::cluster_rank(), cn = ecq_dev::cluster_size();
    const int chunk = (n + static_cast<int>(cn) - 1) / static_cast<int>(cn);
    const int i0 = static_cast<int>(cr) * chunk;
    const int i1 = min(n, i0 + chunk);
    pdl_launch_dependents();
    pdl_wait();  // h and d come from the kernels before this one
    float ss = 0.f;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        float v = __half2float(h[i]);
        if (d) v = __half2float(__float2half_rn(v + __half2float(d[i])));  // the residual is stored in fp16
        buf[i - i0] = v;
        ss += v * v;
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    float* part = buf + chunk;
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) s_part = v;
    }
    ecq_dev::cluster_sync();
    float tot = 0.f;
    for (uint32_t r = 0; r < cn; ++r) tot += ecq_dev::ld_cluster_f32(&s_part, r);
    const float rs = rsqrtf(tot / n + eps);
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const float v = buf[i - i0];
        if (d) h_out[i] = __float2half_rn(v);
        y[i] = __hmul(__float2half_rn(v * rs), w[i]);
    }
    ecq_dev::cluster_sync();  // no CTA leaves while another reads its partial
}

// q, k: [heads, dim] (dim even); pairs (2i, 2i+1) rotate by angle index i.
__global__ void rope_kv_kernel(__half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
                               __half* __restrict__ kc, __half* __restrict__ vc, const __half* __restrict__ cs,
                               const __half* __restrict__ sn, int heads, int dim, int64_t cache_head_stride) {
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x;
    const int half_dim = dim / 2;
    for (int i = threadIdx.x; i < half_dim; i += blockDim.x) {
        const float c = __half2float(cs[i]), s = __half2float(sn[i]);
        const size_t o = static_cast<size_t>(h) * dim + 2 * i;
        const float q0 = __half2float(q[o]), q1 = __half2float(q[o + 1]);
        q[o] = __float2half_rn(q0 * c - q1 * s);
        q[o + 1] = __float2half_rn(q0 * s + q1 * c);
        const float k0 = __half2float(k[o]), k1 = __half2float(k[o + 1]);
        __half* kd = kc + h * cache_head_stride + 2 * i;
        kd[0] = __float2half_rn(k0 * c - k1 * s);
        kd[1] = __float2half_rn(k0 * s + k1 * c);
        __half* vd = vc + h * cache_head_stride + 2 * i;
        vd[0] = v[o];
        vd[1] = v[o + 1];
    }
}

__global__ void silu_mul_kernel(const __half* __restrict__ gu, __half* __restrict__ m, int f, int64_t rows) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t n = static_cast<int64_t>(f) * rows;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / f, c = i - r * f;
        const float g = __half2float(gu[r * 2 * f + c]);
        const float u = __half2float(gu[r * 2 * f + f + c]);
        m[i] = __float2half_rn(__half2float(__float2half_rn(g / (1.f + __expf(-g)))) * u);
    }
}

}  // namespace

extern "C" {

int32_t ecq_add_rmsnorm_f16(const void* h, const void* d, const void* w, void* h_out, void* y, int32_t rows,
                            int32_t n, float eps, void* stream) {
    if (!h || !w || !y || rows < 1 || n < 1 || (d && !h_out) || n > 12256) return -1;
    if (rows == 1 && n >= 1024) {
        // one row: spread over a cluster of CTAs instead of one CTA
        const int chunk = (n + kRowCluster - 1) / kRowCluster;
        const cudaError_t rc = ecq_dev::launch_pdl_cluster(
            add_rmsnorm_row_cluster_kernel, dim3(kRowCluster), dim3(kRowThreads), (chunk + 32) * sizeof(float),
            static_cast<cudaStream_t>(stream), kRowCluster, static_cast<const __half*>(h),
            static_cast<const __half*>(d), static_cast<const __half*>(w), static_cast<__half*>(h_out),
            static_cast<__half*>(y), n, eps);
        return rc == cudaSuccess ? 0 : (cudaGetLastError(), -6);
    }
    const int threads = n >= 1024 ? 1024 : ((n + 31) / 32) * 32;
    const cudaError_t rc = launch_pdl(add_rmsnorm_kernel, dim3(rows), dim3(threads), (n + 32) * sizeof(float),
                                      static_cast<cudaStream_t>(stream), static_cast<const __half*>(h),
                                      static_cast<const __half*>(d), static_cast<const __half*>(w),
                                      static_cast<__half*>(h_out), static_cast<__half*>(y), n, eps);
    return rc == cudaSuccess ? 0 : (cudaGetLastError(), -6);
}

int32_t ecq_rope_kv_f16(void* q, const void* k, const void* v, void* k_cache, void* v_cache, const void* cos_t,
                        const void* sin_t, int32_t heads, int32_t dim, int64_t cache_head_stride, void* stream) {
    if (!q || !k || !v || !k_cache || !v_cache || !cos_t || !sin_t || heads < 1 || dim < 2 || (dim & 1)) return -1;
    const cudaError_t rc = launch_pdl(rope_kv_kernel, dim3(heads), dim3(64), 0, static_cast<cudaStream_t>(stream),
                                      static_cast<__half*>(q), static_cast<const __half*>(k),
                                      static_cast<const __half*>(v), static_cast<__half*>(k_cache),
                                      static_cast<__half*>(v_cache), static_cast<const __half*>(cos_t),
                                      static_cast<const __half*>(sin_t), heads, dim, cache_head_stride);
    return rc == cudaSuccess ? 0 : (cudaGetLastError(), -6);
}

int32_t ecq_silu_mul_f16(const void* gate_up, void* m, int32_t f, int32_t rows, void* stream) {
    if (!gate_up || !m || f < 1 || rows < 1) return -1;
    const int64_t n = static_cast<int64_t>(f) * rows;
    const int blocks = static_cast<int>((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
    const cudaError_t rc = launch_pdl(silu_mul_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                                      static_cast<const __half*>(gate_up), static_cast<__half*>(m), f, n / f);
    return rc == cudaSuccess ? 0 : (cudaGetLastError(), -6);
}

}  // extern "C"
