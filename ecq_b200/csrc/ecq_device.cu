// ecq_device.cu -- sm_100a kernels of libecq and their C-ABI launchers.
//
// Kernels
//   decode_interleaved_exact  one thread per stream of ONE reference tile
//                             (any stream count), the reference decoder's
//                             exact semantics including its guards
//                             (drxddy/ecq src/interleaved_rans.py:156-217).
//   matrix_kernel<...>        persistent, one CTA per SM. Each warp owns a
//                             contiguous run of 32-stream tiles of a packed
//                             matrix; lane j decodes stream j of the tile.
//                             The 16384-entry packed decode table lives in
//                             shared memory (one bulk copy per CTA); tile
//                             bytes are double-buffered into shared memory
//                             with cp.async.bulk + mbarrier. Two consumers:
//                             the fused dequant+GEMV (fp32 accumulation, no
//                             decoded weight ever leaves registers) and the
//                             symbol store (CACHED mode).
//
// Decode step (one symbol, per lane), the reference's arithmetic
// (src/rans.py:145-181):
//   slot = x & 16383; e = table[slot]  ->  sym, freq, bias = slot - cumfreq
//   x = freq * (x >> 14) + bias
//   while x < 2^23: x = (x << 8) | next byte          (at most twice)
// The fast kernels read bytes without the reference's "ptr < stream_len"
// guard; a stream that would have hit it cannot end in the state the
// encoder started from, so the end-of-stream check (state == 2^23 and
// exactly stream_len bytes consumed) flags it (ECQ_STATUS_CORRUPT). For
// intact streams the two decoders are therefore identical.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "ecq.h"

namespace {

constexpr uint32_t kL = ECQ_RANS_L;
constexpr int kTableBytes = ECQ_TABLE_ENTRIES * 4;
constexpr int kMaxSmem = 227 * 1024;
constexpr uint64_t kWaitLimitNs = 200ull * 1000ull * 1000ull;  // 0.2 s per bounded wait

// ---------------------------------------------------------------------------
// PTX helpers (mbarrier + bulk copy; no multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false after kWaitLimitNs without the phase completing.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Exact reference-semantics decode of one interleaved tile (any S).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) decode_interleaved_exact(const uint8_t* __restrict__ data,
                                                                 const uint32_t* __restrict__ lengths,
                                                                 uint32_t S, uint64_t n,
                                                                 const uint32_t* __restrict__ gtable,
                                                                 uint32_t flags, uint8_t* __restrict__ out,
                                                                 uint32_t* __restrict__ status) {
    extern __shared__ __align__(16) uint32_t table[];
    for (int i = threadIdx.x; i < ECQ_TABLE_ENTRIES; i += blockDim.x) table[i] = gtable[i];
    __syncthreads();
    const uint64_t j = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= S) return;
    const uint64_t count = (j < n) ? (n - 1 - j) / S + 1 : 0;
    const uint32_t len = lengths[j];
    if (len < 4) {
        // src/interleaved_rans.py:178-179: the stream is skipped, its outputs stay 0
        for (uint64_t i = 0; i < count; ++i) out[j + i * S] = 0;
        if (count) atomicOr(status, ECQ_STATUS_CORRUPT);
        return;
    }
    const bool constant = flags & ECQ_FLAG_CONSTANT;
    const uint32_t csym = (flags >> ECQ_FLAG_CONSTANT_SYM_SHIFT) & 15u;
    uint32_t x = (static_cast<uint32_t>(data[j]) << 24) | (static_cast<uint32_t>(data[j + S]) << 16) |
                 (static_cast<uint32_t>(data[j + 2 * S]) << 8) | static_cast<uint32_t>(data[j + 3 * S]);
    uint32_t ptr = 4;
    for (uint64_t i = 0; i < count; ++i) {
        uint32_t sym;
        if (constant) {
            sym = csym;  // freq 16384, cumfreq 0: the state is unchanged
        } else {
            const uint32_t e = table[x & 16383u];
            sym = e & 15u;
            x = ((e >> 4) & 16383u) * (x >> 14) + (e >> 18);
        }
        out[j + i * S] = static_cast<uint8_t>(sym);
        while (x < kL && ptr < len) {
            x = (x << 8) | data[j + static_cast<uint64_t>(ptr) * S];
            ++ptr;
        }
    }
    if (x != kL || ptr != len) atomicOr(status, ECQ_STATUS_CORRUPT);
}

// ---------------------------------------------------------------------------
// Persistent packed-matrix kernel
// ---------------------------------------------------------------------------
struct MatrixParams {
    const uint8_t* data;
    const uint32_t* tile_offset;
    const uint16_t* stream_len;
    const uint32_t* dec_table;
    const __half* x;       // [cols]
    const __half* scales;  // [rows, ng]
    __half* y;             // [rows]
    uint8_t* sym_out;      // [rows, cols] (decode mode)
    float* partials;       // [n_tiles, 8]
    uint32_t* slab_count;  // [n_slabs]
    uint32_t* status;
    uint32_t rows, cols, ng, group_size;
    uint32_t n_ktiles, n_tiles;
    uint32_t buf_bytes;
    uint32_t flags;
};

constexpr int kTileRows = 8;

// One decode step on lane state (x, a); a is the shared-memory address of
// the lane's next stream byte (byte p of lane j at tile_base + 32p + j).
__device__ __forceinline__ uint32_t decode_step(uint32_t& x, uint32_t& a, const uint32_t* __restrict__ table,
                                                const uint8_t* __restrict__ smem_base) {
    const uint32_t e = table[x & 16383u];
    x = (e >> 18) + ((e >> 4) & 16383u) * (x >> 14);
    if (x < kL) {
        x = (x << 8) | smem_base[a];
        a += 32;
        if (x < kL) {
            x = (x << 8) | smem_base[a];
            a += 32;
        }
    }
    return e & 15u;
}

__device__ __forceinline__ float sym_minus8(uint32_t sym) {
    // exact float(sym - 8) for sym < 16: (2^23 + sym) - (2^23 + 8)
    return __int_as_float(0x4B000000u | sym) - 8388616.0f;
}

// Reduce v[0..7] over the 32 lanes; lane l ends with the total of row
// 4*bit4(l) + 2*bit3(l) + bit2(l). Fixed order, so results are deterministic.
__device__ __forceinline__ float transpose_reduce8(float (&v)[8], int lane) {
    const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = b16 ? v[i] : v[i + 4];
        const float keep = b16 ? v[i + 4] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = b8 ? v[i] : v[i + 2];
        const float keep = b8 ? v[i + 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    {
        const float send = b4 ? v[0] : v[1];
        const float keep = b4 ? v[1] : v[0];
        v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
    return v[0];
}

__device__ __forceinline__ int reduce_row_of_lane(int lane) {
    return ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
}

template <int MPL, int GPL, bool GEMV, bool CONSTANT>
__device__ __forceinline__ void process_tile(const MatrixParams& p, uint32_t t, uint32_t buf, const uint32_t* table,
                                             const uint8_t* smem_base, int lane) {
    constexpr int NSG = MPL / GPL;                      // group segments per tile row
    constexpr int NSC = (kTileRows * NSG + 31) / 32;    // scales held per lane
    const uint32_t slab = t / p.n_ktiles;
    const uint32_t kt = t - slab * p.n_ktiles;
    const uint32_t r0 = slab * kTileRows;
    const uint32_t rows_here = min(static_cast<uint32_t>(kTileRows), p.rows - r0);
    const uint32_t c0 = kt * (MPL * 32);
    const uint32_t len = p.stream_len[t * 32 + lane];

    uint32_t a = buf + lane;
    uint32_t x = (static_cast<uint32_t>(smem_base[a]) << 24) | (static_cast<uint32_t>(smem_base[a + 32]) << 16) |
                 (static_cast<uint32_t>(smem_base[a + 64]) << 8) | static_cast<uint32_t>(smem_base[a + 96]);
    a += 128;
    const uint32_t csym = (p.flags >> ECQ_FLAG_CONSTANT_SYM_SHIFT) & 15u;

    float xr[MPL];
    float sc[NSC];
    float acc[kTileRows];
    if constexpr (GEMV) {
#pragma unroll
        for (int m = 0; m < MPL; ++m) xr[m] = __half2float(p.x[c0 + 32 * m + lane]);
#pragma unroll
        for (int i = 0; i < NSC; ++i) {
            const int idx = lane + 32 * i;
            const int r = idx / NSG, sg = idx - (idx / NSG) * NSG;
            float s = 0.f;
            if (r < static_cast<int>(rows_here))
                s = __half2float(p.scales[static_cast<size_t>(r0 + r) * p.ng + (c0 + sg * GPL * 32) / p.group_size]);
            sc[i] = s;
        }
#pragma unroll
        for (int r = 0; r < kTileRows; ++r) acc[r] = 0.f;
    }

#pragma unroll
    for (int r = 0; r < kTileRows; ++r) {
        if (r < static_cast<int>(rows_here)) {
#pragma unroll
            for (int sg = 0; sg < NSG; ++sg) {
                float part = 0.f;
#pragma unroll
                for (int mm = 0; mm < GPL; ++mm) {
                    const int m = sg * GPL + mm;
                    uint32_t sym;
                    if constexpr (CONSTANT) {
                        sym = csym;
                    } else {
                        sym = decode_step(x, a, table, smem_base);
                    }
                    if constexpr (GEMV) {
                        part = fmaf(sym_minus8(sym), xr[m], part);
                    } else {
                        p.sym_out[static_cast<size_t>(r0 + r) * p.cols + c0 + 32 * m + lane] = static_cast<uint8_t>(sym);
                    }
                }
                if constexpr (GEMV) {
                    constexpr int idx0 = 0;
                    (void)idx0;
                    const int idx = r * NSG + sg;  // compile-time after unrolling
                    const float s = __shfl_sync(0xffffffffu, sc[idx >> 5], idx & 31);
                    acc[r] = fmaf(s, part, acc[r]);
                }
            }
        }
    }
    if constexpr (!CONSTANT) {
        if (x != kL || (a - buf - lane) != len * 32u) atomicOr(p.status, ECQ_STATUS_CORRUPT);
    } else {
        if (len != 4u) atomicOr(p.status, ECQ_STATUS_CORRUPT);
    }

    if constexpr (GEMV) {
        const float v = transpose_reduce8(acc, lane);
        if ((lane & 3) == 0) p.partials[static_cast<size_t>(t) * kTileRows + reduce_row_of_lane(lane)] = v;
        __threadfence();
        __syncwarp();
        uint32_t old = 0;
        if (lane == 0) old = atomicAdd(p.slab_count + slab, 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == p.n_ktiles - 1) {
            // last tile of this row slab: sum the slab's partials in fixed order
            __threadfence();
            const int row = lane & 7, kp = lane >> 3;
            const float* base = p.partials + static_cast<size_t>(slab) * p.n_ktiles * kTileRows;
            float s = 0.f;
            for (uint32_t k = kp; k < p.n_ktiles; k += 4) s += __ldcg(base + static_cast<size_t>(k) * kTileRows + row);
            s += __shfl_xor_sync(0xffffffffu, s, 8);
            s += __shfl_xor_sync(0xffffffffu, s, 16);
            if (kp == 0 && row < static_cast<int>(rows_here)) p.y[r0 + row] = __float2half_rn(s);
            if (lane == 0) p.slab_count[slab] = 0u;
        }
    }
}

template <int MPL, int GPL, bool GEMV>
__global__ void __launch_bounds__(1024, 1) matrix_kernel(MatrixParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int W = blockDim.x >> 5;
    const uint32_t bufs = smem_addr(smem);
    const uint32_t* table = reinterpret_cast<const uint32_t*>(smem + 2 * W * p.buf_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * W * p.buf_bytes + kTableBytes);
    const uint32_t table_bar = smem_addr(bars + 2 * W);
    const bool constant = p.flags & ECQ_FLAG_CONSTANT;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2 * W + 1; ++i) mbar_init(smem_addr(bars + i), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        mbar_expect_tx(table_bar, kTableBytes);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            bulk_copy_g2s(smem_addr(table) + i * (kTableBytes / 4),
                          reinterpret_cast<const uint8_t*>(p.dec_table) + i * (kTableBytes / 4), kTableBytes / 4,
                          table_bar);
    }

    // contiguous run of tiles for this warp
    const uint64_t GW = static_cast<uint64_t>(gridDim.x) * W;
    const uint64_t gw = static_cast<uint64_t>(blockIdx.x) * W + warp;
    const uint32_t t_begin = static_cast<uint32_t>(gw * p.n_tiles / GW);
    const uint32_t t_end = static_cast<uint32_t>((gw + 1) * p.n_tiles / GW);
    const uint32_t my_bar0 = smem_addr(bars + 2 * warp);
    const uint32_t my_buf0 = bufs + 2 * warp * p.buf_bytes;

    auto issue = [&](uint32_t t, int stage) {
        const uint32_t off = p.tile_offset[t];
        uint32_t bytes = p.tile_offset[t + 1] - off;
        if (bytes > p.buf_bytes || (off & 15u) || (bytes & 15u)) {
            // never copy past the stage buffer: the tile decodes from stale
            // bytes instead and fails its end-of-stream check
            atomicOr(p.status, ECQ_STATUS_BADARG);
            bytes = 0;
        }
        const uint32_t bar = my_bar0 + 8 * stage;
        mbar_expect_tx(bar, bytes);
        if (bytes) bulk_copy_g2s(my_buf0 + stage * p.buf_bytes, p.data + off, bytes, bar);
    };

    if (lane == 0 && t_begin < t_end) issue(t_begin, 0);
    bool ok = mbar_wait(table_bar, 0);
    if (!ok && lane == 0) atomicOr(p.status, ECQ_STATUS_TIMEOUT);

    uint32_t phase0 = 0, phase1 = 0;
    for (uint32_t t = t_begin; ok && t < t_end; ++t) {
        const int stage = (t - t_begin) & 1;
        if (t + 1 < t_end) {
            __syncwarp();
            if (lane == 0) {
                fence_proxy_async();
                issue(t + 1, stage ^ 1);
            }
        }
        const uint32_t parity = stage ? phase1 : phase0;
        if (!mbar_wait(my_bar0 + 8 * stage, parity)) {
            if (lane == 0) atomicOr(p.status, ECQ_STATUS_TIMEOUT);
            ok = false;
            break;
        }
        if (stage) phase1 ^= 1; else phase0 ^= 1;
        const uint32_t buf = 2 * warp * p.buf_bytes + stage * p.buf_bytes;  // offset within smem
        if (constant)
            process_tile<MPL, GPL, GEMV, true>(p, t, buf, table, smem, lane);
        else
            process_tile<MPL, GPL, GEMV, false>(p, t, buf, table, smem, lane);
    }
    // never leave a bulk copy in flight when exiting after a timeout
    if (!ok && t_begin < t_end) {
        mbar_wait(my_bar0, phase0);
        mbar_wait(my_bar0 + 8, phase1);
    }
}

// ---------------------------------------------------------------------------
// launch plumbing
// ---------------------------------------------------------------------------
using KernelFn = void (*)(MatrixParams);

template <bool GEMV>
KernelFn pick_kernel(int mpl, int gpl) {
#define ECQ_CASE(M_, G_) \
    if (mpl == M_ && gpl == G_) return matrix_kernel<M_, G_, GEMV>;
    ECQ_CASE(4, 1) ECQ_CASE(4, 2) ECQ_CASE(4, 4)
    ECQ_CASE(8, 1) ECQ_CASE(8, 2) ECQ_CASE(8, 4) ECQ_CASE(8, 8)
    ECQ_CASE(16, 1) ECQ_CASE(16, 2) ECQ_CASE(16, 4) ECQ_CASE(16, 8) ECQ_CASE(16, 16)
#undef ECQ_CASE
    return nullptr;
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device),
// outside any stream capture that may follow.
bool ensure_smem_limit(const void* fn, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({fn, dev})) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
    done.insert({fn, dev});
    return true;
}

int sm_count_cached() {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 1;
    }
    return sms;
}

struct LaunchShape {
    int mpl, gpl, warps, ctas;
    uint32_t buf_bytes;
    size_t smem;
};

int32_t shape_for(const ecq_matrix_view* m, bool gemv, LaunchShape* ls) {
    if (!m) return ECQ_ERR_ARG;
    if (m->tile_rows != kTileRows) return ECQ_ERR_UNSUPPORTED;
    if (m->tile_cols % 32 || m->tile_cols == 0 || m->cols % m->tile_cols) return ECQ_ERR_SHAPE;
    const int mpl = static_cast<int>(m->tile_cols / 32);
    int gpl = mpl;
    if (gemv) {
        const uint32_t g = m->group_size;
        if (g == 0 || g % 32) return ECQ_ERR_UNSUPPORTED;
        if (g < m->tile_cols) {
            if (m->tile_cols % g) return ECQ_ERR_UNSUPPORTED;
            gpl = static_cast<int>(g / 32);
        } else if (g % m->tile_cols) {
            return ECQ_ERR_UNSUPPORTED;
        }
    }
    if (!(gemv ? pick_kernel<true>(mpl, gpl) : pick_kernel<false>(mpl, gpl))) return ECQ_ERR_UNSUPPORTED;
    const uint32_t slabs = (m->rows + kTileRows - 1) / kTileRows;
    if (m->n_tiles != slabs * (m->cols / m->tile_cols)) return ECQ_ERR_SHAPE;
    uint32_t buf = (m->max_tile_bytes + 127u) & ~127u;
    if (buf < 128) buf = 128;
    const int bar_bytes = 8 * (2 * 32 + 1);
    int warps = static_cast<int>((kMaxSmem - kTableBytes - bar_bytes) / (2 * static_cast<int64_t>(buf)));
    if (warps > 32) warps = 32;
    if (warps < 1) return ECQ_ERR_UNSUPPORTED;
    ls->mpl = mpl;
    ls->gpl = gpl;
    ls->warps = warps;
    ls->ctas = sm_count_cached();
    ls->buf_bytes = buf;
    ls->smem = static_cast<size_t>(2 * warps) * buf + kTableBytes + 8 * (2 * warps + 1);
    return ECQ_OK;
}

int32_t launch_matrix(const ecq_matrix_view* m, bool gemv, const __half* x, const __half* scales, __half* y,
                      uint8_t* sym_out, void* workspace, uint32_t* status, cudaStream_t stream) {
    LaunchShape ls;
    int32_t rc = shape_for(m, gemv, &ls);
    if (rc != ECQ_OK) return rc;
    MatrixParams p{};
    p.data = m->data;
    p.tile_offset = m->tile_offset;
    p.stream_len = m->stream_len;
    p.dec_table = m->dec_table;
    p.x = x;
    p.scales = scales;
    p.y = y;
    p.sym_out = sym_out;
    p.status = status;
    p.rows = m->rows;
    p.cols = m->cols;
    p.group_size = m->group_size ? m->group_size : 32;
    p.ng = (m->cols + p.group_size - 1) / p.group_size;
    p.n_ktiles = m->cols / m->tile_cols;
    p.n_tiles = m->n_tiles;
    p.buf_bytes = ls.buf_bytes;
    p.flags = m->flags;
    if (gemv) {
        p.partials = static_cast<float*>(workspace);
        p.slab_count = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) +
                                                   static_cast<size_t>(m->n_tiles) * kTileRows * sizeof(float));
    }
    KernelFn fn = gemv ? pick_kernel<true>(ls.mpl, ls.gpl) : pick_kernel<false>(ls.mpl, ls.gpl);
    if (!ensure_smem_limit(reinterpret_cast<const void*>(fn), kMaxSmem)) return ECQ_ERR_CUDA;
    fn<<<ls.ctas, ls.warps * 32, ls.smem, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? ECQ_OK : ECQ_ERR_CUDA;
}

bool view_ok(const ecq_matrix_view* m) {
    return m && m->data && m->tile_offset && m->stream_len && m->dec_table && m->rows && m->cols && m->n_tiles;
}

}  // namespace

extern "C" {

int32_t ecq_decode_interleaved(const uint8_t* d_data, const uint32_t* d_lengths, uint32_t n_streams,
                               uint64_t n_symbols, uint32_t max_len, const uint32_t* d_dec_table,
                               uint32_t decode_flags, uint8_t* d_out, uint32_t* d_status, void* stream) {
    if (n_streams == 0 || !d_lengths || !d_dec_table || !d_status) return ECQ_ERR_ARG;
    if (n_symbols == 0) return ECQ_OK;
    if (!d_out || (max_len > 0 && !d_data)) return ECQ_ERR_ARG;
    const int threads = 256;
    const unsigned blocks = (n_streams + threads - 1) / threads;
    if (!ensure_smem_limit(reinterpret_cast<const void*>(decode_interleaved_exact), kTableBytes))
        return ECQ_ERR_CUDA;
    decode_interleaved_exact<<<blocks, threads, kTableBytes, static_cast<cudaStream_t>(stream)>>>(
        d_data, d_lengths, n_streams, n_symbols, d_dec_table, decode_flags, d_out, d_status);
    return cudaGetLastError() == cudaSuccess ? ECQ_OK : ECQ_ERR_CUDA;
}

int32_t ecq_matrix_decode(const ecq_matrix_view* m, uint8_t* d_out, uint32_t* d_status, void* stream) {
    if (!view_ok(m) || !d_out || !d_status) return ECQ_ERR_ARG;
    return launch_matrix(m, false, nullptr, nullptr, nullptr, d_out, nullptr, d_status,
                         static_cast<cudaStream_t>(stream));
}

int64_t ecq_gemv_workspace_bytes(const ecq_matrix_view* m, uint32_t batch) {
    (void)batch;
    if (!m || !m->rows || !m->n_tiles) return ECQ_ERR_ARG;
    const int64_t slabs = (m->rows + kTileRows - 1) / kTileRows;
    return static_cast<int64_t>(m->n_tiles) * kTileRows * 4 + slabs * 4;
}

int32_t ecq_gemv(const ecq_matrix_view* m, const void* x_f16, const void* scales_f16, void* y_f16, uint32_t batch,
                 void* workspace, int64_t workspace_bytes, uint32_t* d_status, void* stream) {
    if (!view_ok(m) || !x_f16 || !scales_f16 || !y_f16 || !d_status || batch == 0) return ECQ_ERR_ARG;
    if (!workspace || workspace_bytes < ecq_gemv_workspace_bytes(m, batch)) return ECQ_ERR_WORKSPACE;
    const __half* x = static_cast<const __half*>(x_f16);
    __half* y = static_cast<__half*>(y_f16);
    for (uint32_t b = 0; b < batch; ++b) {
        int32_t rc = launch_matrix(m, true, x + static_cast<size_t>(b) * m->cols, static_cast<const __half*>(scales_f16),
                                   y + static_cast<size_t>(b) * m->rows, nullptr, workspace, d_status,
                                   static_cast<cudaStream_t>(stream));
        if (rc != ECQ_OK) return rc;
    }
    return ECQ_OK;
}

int32_t ecq_device_info(int32_t* sm_count, int32_t* gemv_ctas, int32_t* gemv_warps_per_cta,
                        const ecq_matrix_view* m) {
    if (sm_count) *sm_count = sm_count_cached();
    if (m) {
        LaunchShape ls;
        int32_t rc = shape_for(m, true, &ls);
        if (rc != ECQ_OK) return rc;
        if (gemv_ctas) *gemv_ctas = ls.ctas;
        if (gemv_warps_per_cta) *gemv_warps_per_cta = ls.warps;
    }
    return ECQ_OK;
}

}  // extern "C"
