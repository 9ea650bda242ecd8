// ecq_attention.cu -- batch-1 decode attention over an fp16 KV cache for the
// few heads a tensor-parallel rank holds.
//
// att[h] = softmax(q[h] . K[h]^T / sqrt(D)) . V[h] for one query token,
// heads h < H, keys t < T, head_dim D = 128. One kernel, split over keys:
//   * grid (H, S): CTA (h, s) takes a contiguous chunk of the T keys; each of
//     its 4 warps walks every 4th key of the chunk, 8 keys per step. Lane l
//     holds q[4l .. 4l+3] (fp32, pre-scaled by log2(e)/sqrt(D)), loads 4 fp16
//     of each key's K and V row (8 bytes; a warp reads the 256-byte row in
//     one coalesced request), sums the dot product over the warp, and keeps an
//     online softmax (running max m, sum l, output o[4]) in fp32 with exp2.
//   * the 4 warps merge in shared memory; the CTA writes its (m, l, o[D]) to
//     the workspace and counts itself in the head's counter. The CTA that
//     counts last merges the S partials in a fixed order (deterministic) and
//     writes att[h] in fp16, then clears the counter for the next call.
// The arithmetic follows flash-decoding (fp32 softmax and accumulation over
// fp16 K/V); results agree with cuDNN's SDPA to fp16 rounding.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ecq_glue.h"
#include "ecq_kernels.cuh"

namespace {

using ecq_dev::launch_pdl;
using ecq_dev::pdl_launch_dependents;
using ecq_dev::pdl_wait;

constexpr int kD = 128;
constexpr int kWarps = 4;
constexpr int kKeysPerStep = 8;
constexpr int kMaxSplits = 128;
constexpr int kStride = kD + 4;  // per partial: m, l, 2 pad, o[kD] (o 16-byte aligned)

__device__ __forceinline__ uint2 ldg8(const __half* p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ void h4(uint2 v, float (&f)[4]) {
    const float2 a = __half22float2(*reinterpret_cast<__half2*>(&v.x));
    const float2 b = __half22float2(*reinterpret_cast<__half2*>(&v.y));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
}

// workspace per (head, split): m, l, 2 pad, o[kD] as floats; then one u32 counter per head
__global__ void __launch_bounds__(kWarps * 32) decode_attention_kernel(const __half* __restrict__ q,
                                                                      const __half* __restrict__ kc,
                                                                      const __half* __restrict__ vc,
                                                                      __half* __restrict__ out, float* ws,
                                                                      int T, int S, int64_t head_stride,
                                                                      float qscale) {
    __shared__ float sm_m[kWarps], sm_l[kWarps];
    __shared__ float sm_o[kWarps][kD];
    __shared__ uint32_t s_last;
    const int h = blockIdx.x, s = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int chunk = (T + S - 1) / S;
    const int t0 = s * chunk, t1 = min(T, t0 + chunk);
    const int H = gridDim.x;
    float* part = ws + (static_cast<size_t>(h) * S + s) * kStride;
    uint32_t* counter = reinterpret_cast<uint32_t*>(ws + static_cast<size_t>(H) * S * kStride) + h;

    pdl_launch_dependents();
    pdl_wait();  // q and the new token's K/V come from the kernels before this one
    float qv[4];
    h4(ldg8(q + static_cast<size_t>(h) * kD + 4 * lane), qv);
#pragma unroll
    for (int i = 0; i < 4; ++i) qv[i] *= qscale;
    const __half* kh = kc + static_cast<size_t>(h) * head_stride + 4 * lane;
    const __half* vh = vc + static_cast<size_t>(h) * head_stride + 4 * lane;

    float m = -INFINITY, l = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int tb = t0 + warp; tb < t1; tb += kWarps * kKeysPerStep) {
        uint2 kr[kKeysPerStep], vr[kKeysPerStep];
#pragma unroll
        for (int j = 0; j < kKeysPerStep; ++j) {
            const int t = tb + j * kWarps;
            if (t < t1) {
                kr[j] = ldg8(kh + static_cast<size_t>(t) * kD);
                vr[j] = ldg8(vh + static_cast<size_t>(t) * kD);
            } else {
                kr[j] = make_uint2(0u, 0u);
                vr[j] = make_uint2(0u, 0u);
            }
        }
        float sc[kKeysPerStep];
#pragma unroll
        for (int j = 0; j < kKeysPerStep; ++j) {
            float kf[4];
            h4(kr[j], kf);
            float d = qv[0] * kf[0] + qv[1] * kf[1] + qv[2] * kf[2] + qv[3] * kf[3];
#pragma unroll
            for (int off = 16; off; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
            sc[j] = (tb + j * kWarps < t1) ? d : -INFINITY;
        }
        float mx = m;
#pragma unroll
        for (int j = 0; j < kKeysPerStep; ++j) mx = fmaxf(mx, sc[j]);
        const float alpha = exp2f(m - mx);  // m = -inf on the first step: alpha = 0
        l *= alpha;
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] *= alpha;
#pragma unroll
        for (int j = 0; j < kKeysPerStep; ++j) {
            const float pj = exp2f(sc[j] - mx);
            float vf[4];
            h4(vr[j], vf);
            l += pj;
#pragma unroll
            for (int i = 0; i < 4; ++i) o[i] = fmaf(pj, vf[i], o[i]);
        }
        m = mx;
    }
    // merge the 4 warps of this CTA
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) sm_o[warp][4 * lane + i] = o[i];
    __syncthreads();
    if (warp == 0) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w]);
        float L = 0.f, O[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float a = (sm_m[w] == -INFINITY) ? 0.f : exp2f(sm_m[w] - M);
            L = fmaf(a, sm_l[w], L);
#pragma unroll
            for (int i = 0; i < 4; ++i) O[i] = fmaf(a, sm_o[w][4 * lane + i], O[i]);
        }
        if (lane == 0) {
            part[0] = M;
            part[1] = L;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) part[4 + 4 * lane + i] = O[i];
        __threadfence();
        __syncwarp();
        if (lane == 0) s_last = (atomicAdd(counter, 1u) == static_cast<uint32_t>(S - 1)) ? 1u : 0u;
        __syncwarp();
        if (__shfl_sync(0xffffffffu, s_last, 0)) {
            // the last split of this head merges all S partials in a fixed
            // order: lane j loads the (m, l) of splits j, j + 32, ... at once,
            // the weights are summed by a fixed butterfly, and the outputs
            // stream in split order
            __threadfence();
            const float* hp = ws + static_cast<size_t>(h) * S * kStride;
            float mk[kMaxSplits / 32], lk[kMaxSplits / 32];
            float MM = -INFINITY;
#pragma unroll
            for (int u = 0; u < kMaxSplits / 32; ++u) {
                const int k = lane + 32 * u;
                mk[u] = k < S ? __ldcg(hp + static_cast<size_t>(k) * kStride) : -INFINITY;
                lk[u] = k < S ? __ldcg(hp + static_cast<size_t>(k) * kStride + 1) : 0.f;
                MM = fmaxf(MM, mk[u]);
            }
#pragma unroll
            for (int off = 16; off; off >>= 1) MM = fmaxf(MM, __shfl_xor_sync(0xffffffffu, MM, off));
            float ak[kMaxSplits / 32];
            float LL = 0.f;
#pragma unroll
            for (int u = 0; u < kMaxSplits / 32; ++u) {
                ak[u] = (mk[u] == -INFINITY) ? 0.f : exp2f(mk[u] - MM);
                LL = fmaf(ak[u], lk[u], LL);
            }
#pragma unroll
            for (int off = 16; off; off >>= 1) LL += __shfl_xor_sync(0xffffffffu, LL, off);
            float OO[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int u = 0; u < kMaxSplits / 32; ++u) {
                if (32 * u >= S) break;
#pragma unroll 4
                for (int j = 0; j < 32; ++j) {
                    const int k = 32 * u + j;
                    const float a = __shfl_sync(0xffffffffu, ak[u], j);
                    if (k < S) {
                        const float4 ov =
                            __ldcg(reinterpret_cast<const float4*>(hp + static_cast<size_t>(k) * kStride + 4) + lane);
                        OO[0] = fmaf(a, ov.x, OO[0]);
                        OO[1] = fmaf(a, ov.y, OO[1]);
                        OO[2] = fmaf(a, ov.z, OO[2]);
                        OO[3] = fmaf(a, ov.w, OO[3]);
                    }
                }
            }
            const float inv = 1.f / LL;
            __half2* dst = reinterpret_cast<__half2*>(out + static_cast<size_t>(h) * kD + 4 * lane);
            dst[0] = __floats2half2_rn(OO[0] * inv, OO[1] * inv);
            dst[1] = __floats2half2_rn(OO[2] * inv, OO[3] * inv);
            if (lane == 0) *counter = 0u;
        }
    }
}

}  // namespace

extern "C" {

int64_t ecq_decode_attention_workspace_bytes(int32_t heads, int32_t splits) {
    if (heads < 1 || splits < 1) return -1;
    return static_cast<int64_t>(heads) * splits * kStride * 4 + static_cast<int64_t>(heads) * 4;
}

int32_t ecq_decode_attention_splits(int32_t heads, int32_t keys) {
    if (heads < 1 || keys < 1) return -1;
    // about two CTAs per SM over all heads, at least 32 keys per split, and
    // no more splits than the merge handles
    int s = (2 * ecq_dev::sm_count_cached() + heads - 1) / heads;
    const int max_s = (keys + 31) / 32;
    if (s > max_s) s = max_s;
    if (s > kMaxSplits) s = kMaxSplits;
    return s < 1 ? 1 : s;
}

int32_t ecq_decode_attention_f16(const void* q, const void* k_cache, const void* v_cache, void* out, int32_t heads,
                                 int32_t head_dim, int32_t keys, int64_t head_stride, int32_t splits, void* workspace,
                                 int64_t workspace_bytes, void* stream) {
    if (!q || !k_cache || !v_cache || !out || !workspace || heads < 1 || keys < 1 || splits < 1) return -1;
    if (head_dim != kD || head_stride < static_cast<int64_t>(keys) * kD) return -8;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
         reinterpret_cast<uintptr_t>(out)) & 7u)
        return -1;
    if (splits > kMaxSplits) return -1;
    if (workspace_bytes < ecq_decode_attention_workspace_bytes(heads, splits)) return -9;
    const float qscale = 1.4426950408889634f / sqrtf(static_cast<float>(head_dim));
    const cudaError_t rc = launch_pdl(decode_attention_kernel, dim3(heads, splits), dim3(kWarps * 32), 0,
                                      static_cast<cudaStream_t>(stream), static_cast<const __half*>(q),
                                      static_cast<const __half*>(k_cache), static_cast<const __half*>(v_cache),
                                      static_cast<__half*>(out), static_cast<float*>(workspace), keys, splits,
                                      head_stride, qscale);
    return rc == cudaSuccess ? 0 : (cudaGetLastError(), -6);
}

}  // extern "C"
