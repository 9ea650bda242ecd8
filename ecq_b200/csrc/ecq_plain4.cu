// ecq_plain4.cu -- the plain (not entropy-coded) 4-bit GEMV for sm_100a.
//
// Two roles:
//   * the in-run control beside the fused rANS GEMV: the same shapes, scales
//     and x, with the weights stored as plain packed nibbles, so the bench
//     shows how the entropy-coded path compares with an HBM-bound 4-bit GEMV
//     on the same GPU (the reference's analogue is the nibble-LUT kernel
//     fused_memory_bench, src/metal_interleaved.py:555-683);
//   * the consumer of the CACHED strategy, which decodes each matrix once to
//     packed 4-bit (DecodeOnceStrategy, src/decode_strategies.py:43-73: "store
//     as 4-bit") and then runs this GEMV per call.
//
// Layout: q is [rows, cols/2] bytes, row-major; byte i of a row holds column
// 2i in its low nibble and column 2i+1 in its high nibble (the reference's
// nibble order: `w & 0xF` first). w[r, c] = (q[r, c] - 8) * scales[r, c / g].
//
// Kernel: CTAs of 8 warps; each warp owns R consecutive rows and walks them
// in 16-byte chunks (32 columns), lane l taking chunks l, l + 32, ... with
// streaming 128-bit loads, U chunks per row in flight. x is staged once per
// CTA in shared memory, pre-paired for the nibble extraction below; scales
// are read through L1. Dequantisation is exact in fp16: a nibble ORed into
// the mantissa of 1024.0 (0x6400) gives 1024 + q (low nibble of a byte) or
// 1024 + 16q (high nibble); subtracting 1032 or 1152 leaves q - 8 or
// 16(q - 8) exactly. Products are summed over 8 terms in fp16 (HFMA2), then
// in fp32 per 32-column chunk with the group scale; the warp sum runs in a
// fixed order, so y is deterministic.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ecq.h"
#include "ecq_kernels.cuh"

namespace {

using namespace ecq_dev;

__device__ __forceinline__ uint4 ldg_stream16(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
// (v & mask) | 0x64006400: two nibbles into the mantissas of two fp16 1024.0
__device__ __forceinline__ uint32_t nib2(uint32_t v, uint32_t mask) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(v), "r"(mask), "r"(0x64006400u));
    return d;
}
__device__ __forceinline__ __half2 as_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// The 8 weights of one 32-bit word (columns 8w..8w+7), as q - 8 (pairs A, C)
// and 16(q - 8) (pairs B, D): A = (c0, c4), B = (c1, c5), C = (c2, c6),
// D = (c3, c7).
struct Word8 {
    __half2 a, b, c, d;
};
__device__ __forceinline__ Word8 unpack8(uint32_t v) {
    const __half2 lo_bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
    const __half2 hi_bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    const uint32_t v8 = v >> 8;
    Word8 w;
    w.a = __hsub2(as_h2(nib2(v, 0x000F000Fu)), lo_bias);
    w.b = __hsub2(as_h2(nib2(v, 0x00F000F0u)), hi_bias);
    w.c = __hsub2(as_h2(nib2(v8, 0x000F000Fu)), lo_bias);
    w.d = __hsub2(as_h2(nib2(v8, 0x00F000F0u)), hi_bias);
    return w;
}

// x of one 32-bit weight word, paired to match Word8: (x0, x4), (x1, x5),
// (x2, x6), (x3, x7). Shared memory holds 4 planes of cols/32 uint4: plane j
// entry k is the pairs of word 4k + j (consecutive lanes read consecutive
// 16-byte entries: no bank conflicts).
__device__ __forceinline__ uint4 pair_x8(uint4 v) {
    uint4 o;
    o.x = prmt(v.x, v.z, 0x5410u);
    o.y = prmt(v.x, v.z, 0x7632u);
    o.z = prmt(v.y, v.w, 0x5410u);
    o.w = prmt(v.y, v.w, 0x7632u);
    return o;
}

// sum over one chunk's 4 words: acc0 collects the A/C pairs, acc1 the B/D
// pairs (16x scaled); 8 fp16 products per accumulator half
__device__ __forceinline__ float chunk_dot(const Word8 (&w)[4], const uint4 (&xp)[4]) {
    __half2 acc0 = __float2half2_rn(0.f), acc1 = __float2half2_rn(0.f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        acc0 = __hfma2(w[j].a, as_h2(xp[j].x), acc0);
        acc1 = __hfma2(w[j].b, as_h2(xp[j].y), acc1);
        acc0 = __hfma2(w[j].c, as_h2(xp[j].z), acc0);
        acc1 = __hfma2(w[j].d, as_h2(xp[j].w), acc1);
    }
    const float2 f0 = __half22float2(acc0);
    const float2 f1 = __half22float2(acc1);
    return (f0.x + f0.y) + 0.0625f * (f1.x + f1.y);
}

// W warps per CTA, R rows per warp, U chunks per row in flight, B tokens per
// launch. The loads of the next U chunks of every row (weights and their
// group scales) are issued before the current ones are used, so each lane
// keeps R * U 16-byte weight loads in flight.
template <int W, int R, int U, int B>
__global__ void __launch_bounds__(W * 32) plain4_gemv_kernel(const uint8_t* __restrict__ q,
                                                            const __half* __restrict__ scales,
                                                            const __half* __restrict__ x, __half* __restrict__ y,
                                                            uint32_t rows, uint32_t cols, uint32_t ng,
                                                            uint32_t gshift) {
    extern __shared__ uint4 xs[];  // B tokens x 4 planes x nch
    const uint32_t nch = cols >> 5;
    const uint32_t nw = cols >> 3;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const uint32_t row0 = (blockIdx.x * W + warp) * R;

    // q, x and the scales may all be written by the kernel before this one
    // in the stream (the CACHED strategy decodes q right before its first
    // GEMV): wait for it before touching any of them
    pdl_launch_dependents();
    pdl_wait();
    const uint4* qrow[R];
    const __half* srow[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const uint32_t row = min(row0 + r, rows - 1);
        qrow[r] = reinterpret_cast<const uint4*>(q + static_cast<size_t>(row) * (cols >> 1));
        srow[r] = scales + static_cast<size_t>(row) * ng;
    }
    const bool live = row0 < rows;
    uint4 wv[U][R];
    __half sv[U][R];
    auto fetch = [&](int u, uint32_t k) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (k < nch && live) {
                wv[u][r] = ldg_stream16(qrow[r] + k);
                sv[u][r] = __ldg(srow[r] + (k << 5 >> gshift));
            }
        }
    };
#pragma unroll
    for (int u = 0; u < U; ++u) fetch(u, lane + 32u * u);  // in flight while x is staged
    for (uint32_t i = threadIdx.x; i < B * nw; i += blockDim.x) {
        const uint32_t b = i / nw, w = i - b * nw;
        const uint4 v = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(b) * cols + 8u * w);
        xs[(b * 4 + (w & 3)) * nch + (w >> 2)] = pair_x8(v);
    }
    __syncthreads();
    if (!live) return;

    float acc[R][B];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int b = 0; b < B; ++b) acc[r][b] = 0.f;

    for (uint32_t k0 = lane; k0 < nch; k0 += 32u * U) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t k = k0 + 32u * u;
            if (k < nch) {
                uint4 xp[B][4];
#pragma unroll
                for (int b = 0; b < B; ++b)
#pragma unroll
                    for (int j = 0; j < 4; ++j) xp[b][j] = xs[(b * 4 + j) * nch + k];
                Word8 w[R][4];
                float s[R];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    w[r][0] = unpack8(wv[u][r].x);
                    w[r][1] = unpack8(wv[u][r].y);
                    w[r][2] = unpack8(wv[u][r].z);
                    w[r][3] = unpack8(wv[u][r].w);
                    s[r] = __half2float(sv[u][r]);
                }
                fetch(u, k + 32u * U);  // the next pass's chunk u, loaded while this one computes
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int b = 0; b < B; ++b) acc[r][b] = fmaf(s[r], chunk_dot(w[r], xp[b]), acc[r][b]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float v = acc[r][b];
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && row0 + r < rows) y[static_cast<size_t>(b) * rows + row0 + r] = __float2half_rn(v);
        }
}

using Plain4Fn = void (*)(const uint8_t*, const __half*, const __half*, __half*, uint32_t, uint32_t, uint32_t,
                          uint32_t);

struct Plain4Shape {
    Plain4Fn fn;
    int warps, rows_per_warp;
};

// Launch shape (one token), measured on the Llama-7B sweep shapes: 8-warp
// CTAs with one row per warp for up to 8191 rows, 4-warp CTAs with two rows
// per warp above; 4 chunks of each row in flight per lane. Token batches
// take one row per warp.
Plain4Shape pick_plain4(int B, uint32_t rows) {
    if (B == 1) {
        if (rows >= 8192) return {plain4_gemv_kernel<4, 2, 4, 1>, 4, 2};
        return {plain4_gemv_kernel<8, 1, 4, 1>, 8, 1};
    }
    if (B == 2) return {plain4_gemv_kernel<4, 1, 4, 2>, 4, 1};
    if (B == 3) return {plain4_gemv_kernel<4, 1, 2, 3>, 4, 1};
    return {plain4_gemv_kernel<4, 1, 2, 4>, 4, 1};
}

}  // namespace

extern "C" int32_t ecq_plain4_gemv(const void* q_packed, const void* scales_f16, const void* x_f16, void* y_f16,
                                   uint32_t rows, uint32_t cols, uint32_t group_size, uint32_t batch,
                                   void* stream) {
    if (!q_packed || !scales_f16 || !x_f16 || !y_f16 || rows == 0 || cols == 0 || batch == 0) return ECQ_ERR_ARG;
    if (cols % 32 || group_size < 32 || (group_size & (group_size - 1))) return ECQ_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(q_packed) | reinterpret_cast<uintptr_t>(x_f16)) & 15u) return ECQ_ERR_ARG;
    uint32_t gshift = 0;
    while ((1u << gshift) < group_size) ++gshift;
    const uint32_t ng = (cols + group_size - 1) / group_size;
    const auto* q = static_cast<const uint8_t*>(q_packed);
    const auto* sc = static_cast<const __half*>(scales_f16);
    const auto* x = static_cast<const __half*>(x_f16);
    auto* y = static_cast<__half*>(y_f16);
    // x takes 16 bytes of shared memory per 8 columns per token
    const uint32_t fit = static_cast<uint32_t>(kMaxSmem) / (cols * 2u);
    if (fit == 0) return ECQ_ERR_UNSUPPORTED;
    // up to 4 tokens per launch share one pass over the weights
    for (uint32_t b0 = 0; b0 < batch;) {
        const int B = static_cast<int>(min(min(4u, fit), batch - b0));
        const size_t smem = static_cast<size_t>(B) * cols * 2u;
        const Plain4Shape ps = pick_plain4(B, rows);
        if (!ensure_smem_limit(reinterpret_cast<const void*>(ps.fn), kMaxSmem)) return ECQ_ERR_CUDA;
        const uint32_t per_cta = static_cast<uint32_t>(ps.warps * ps.rows_per_warp);
        const dim3 grid((rows + per_cta - 1) / per_cta);
        if (launch_pdl(ps.fn, grid, dim3(ps.warps * 32), smem, static_cast<cudaStream_t>(stream), q, sc,
                       x + static_cast<size_t>(b0) * cols, y + static_cast<size_t>(b0) * rows, rows, cols, ng,
                       gshift) != cudaSuccess) {
            cudaGetLastError();
            return ECQ_ERR_CUDA;
        }
        b0 += static_cast<uint32_t>(B);
    }
    return ECQ_OK;
}
