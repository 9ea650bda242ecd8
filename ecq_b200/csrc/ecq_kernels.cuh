// ecq_kernels.cuh -- device helpers shared by the libecq kernels: codec
// constants, mbarrier / bulk-copy PTX wrappers with bounded waits, the
// branch-free rANS decode step over the packed shared-memory decode table,
// the exact (sym - 8) weight trick, packed f32x2 arithmetic, and the host-side
// launch helpers (shared-memory limit, SM count).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <set>
#include <utility>

#include "ecq.h"

namespace ecq_dev {

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
// 32-bit shared-window byte load, kept ordered after the mbarrier waits.
__device__ __forceinline__ uint32_t lds_u8(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint16_t lds_u16(uint32_t addr) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

constexpr int kTileRows = 8;
// {-(2^23 + 8*2^14), -(2^23 + 8*2^14)} as f32x2
constexpr uint64_t kNegBias2 = 0xCB020000CB020000ull;

// (sym - 8) * 2^14 as an exact float, from a packed entry: the entry's sym
// field (bits 14..17) ORed into the mantissa of 2^23 gives 2^23 + sym*2^14.
constexpr float kWeightBias = 8519680.0f;  // 2^23 + 8 * 2^14
__device__ __forceinline__ uint32_t entry_weight_bits(uint32_t e) { return (e & 0x3C000u) | 0x4B000000u; }
__device__ __forceinline__ float entry_weight(uint32_t e) { return __int_as_float(entry_weight_bits(e)) - kWeightBias; }

// packed f32x2 arithmetic (sm_100): two fp32 lanes in one 64-bit register pair
__device__ __forceinline__ uint64_t pack2(uint32_t lo, uint32_t hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
    return d;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
    uint32_t a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(a), "=r"(b) : "l"(v));
    lo = __uint_as_float(a);
    hi = __uint_as_float(b);
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// One decode step for this lane. tb is the shared-window address of the
// packed decode table, a that of the lane's next unread stream byte (byte p
// of lane j of a tile at tile_base + 32p + j), and b0, b1 the bytes at a and
// a + 32, loaded ahead (stream_cursor_init sets them up). Returns the table
// entry.
//
// Renormalisation shifts in 0, 1 or 2 of the read-ahead bytes with one
// funnel shift. After a decode step of an intact stream 2^9 <= x < 2^31,
// and the reference's byte loop reads one byte iff x < 2^23 and a second iff
// x < 2^15: the shift is clz(2x) & 24 bits (clz(2x) = clz(x) - 1 lies in
// [0,7], [8,15] or [16,21] for the three cases). A damaged stream can leave
// x below 2^9; the shift is then at most 24 bits (3 bytes, the read-ahead
// bound the callers pad for), the state is wrong from there on, and the
// end-of-stream check flags the tile.
//
// Only lanes that shifted bytes in reload b0 and b1 (predicated loads at the
// new a): most steps consume no byte, and a lane whose load is predicated
// off takes no part in the shared-memory access, so the two byte loads cost
// far fewer bank wavefronts than loads by every lane. The reload is issued
// at the end of the step and consumed by the next step's funnel shift, after
// that step's table lookup, so its latency stays off the decode chain.
__device__ __forceinline__ uint32_t decode_step(uint32_t& x, uint32_t& a, uint32_t& b0, uint32_t& b1, uint32_t tb) {
    uint32_t e;
    asm volatile(
        "{\n\t"
        ".reg .u32 sl, q, f, bi, nx, sh;\n\t"
        ".reg .pred rl;\n\t"
        "and.b32 sl, %0, 16383;\n\t"          // slot
        "mad.lo.u32 sl, sl, 4, %5;\n\t"
        "ld.shared.u32 %2, [sl];\n\t"         // e = table[slot]
        "shr.u32 q, %0, 14;\n\t"
        "shr.u32 f, %2, 18;\n\t"
        "and.b32 bi, %2, 16383;\n\t"
        "mad.lo.u32 %0, f, q, bi;\n\t"        // x = freq * (x >> 14) + slot - cumfreq
        "prmt.b32 nx, %4, %3, 0x4011;\n\t"    // b0 << 24 | b1 << 16
        "shl.b32 sh, %0, 1;\n\t"             // x < 2^31 here, so clz(2x) = clz(x) - 1
        "clz.b32 sh, sh;\n\t"
        "and.b32 sh, sh, 24;\n\t"           // 0, 8 or 16: x >= 2^23, >= 2^15, < 2^15
        "shf.l.wrap.b32 %0, nx, %0, sh;\n\t"  // x = (x << sh) | (nx >> (32 - sh))
        "mad.lo.u32 %1, sh, 4, %1;\n\t"       // 32 bytes per consumed byte
        "setp.ne.u32 rl, sh, 0;\n\t"
        "@rl ld.shared.u8 %3, [%1];\n\t"      // refill the read-ahead bytes
        "@rl ld.shared.u8 %4, [%1+32];\n\t"
        "}"
        : "+r"(x), "+r"(a), "=r"(e), "+r"(b0), "+r"(b1)
        : "r"(tb));
    return e;
}

// Start decoding the lane's stream of a tile staged at shared address buf:
// the 4-byte initial state (big-endian, 32 bytes apart), then the two
// read-ahead bytes decode_step expects.
__device__ __forceinline__ void stream_cursor_init(uint32_t buf, int lane, uint32_t& x, uint32_t& a, uint32_t& b0,
                                                   uint32_t& b1) {
    a = buf + lane;
    x = (lds_u8(a) << 24) | (lds_u8(a + 32) << 16) | (lds_u8(a + 64) << 8) | lds_u8(a + 96);
    a += 128;
    b0 = lds_u8(a);
    b1 = lds_u8(a + 32);
}

template <int MPL>
__host__ __device__ constexpr uint32_t overrun_pad() {
    // a lane reads at most 4 + 3 bytes per symbol of a tile, 32 lanes apart,
    // plus one byte row of read-ahead (the refill after its last step)
    return (32u * (5u + 3u * kTileRows * MPL) + 127u) & ~127u;
}

// Programmatic dependent launch. A kernel launched with launch_pdl may start
// while the kernel before it in the stream is still running: it does the work
// that needs nothing from that kernel first (barrier set-up, decode-table and
// tile copies) and calls pdl_wait() before it touches anything the earlier
// kernel may write or read (activations, outputs, workspaces). pdl_wait()
// returns once the earlier kernel has completed and its writes are visible.
// pdl_launch_dependents() lets the next such kernel start early; it may be
// called at entry, because the next kernel waits for this one's completion
// before touching its data, and it only runs once every CTA of this grid has
// been scheduled.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... Params, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same as one thread-block cluster of `cluster` CTAs along x (grid.x a
// multiple of it), with programmatic dependent launch.
template <typename... Params, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t stream, unsigned cluster, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Thread-block clusters: this CTA's rank, the cluster barrier (every thread
// of every CTA of the cluster; release/acquire orders shared-memory writes
// before it with reads after it), and a float read from another CTA's shared
// memory (distributed shared memory).
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t n;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
    return n;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local)), r;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
    return v;
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device),
// outside any stream capture that may follow.
inline bool ensure_smem_limit(const void* fn, int bytes) {
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

inline int sm_count_cached() {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 1;
    }
    return sms;
}

}  // namespace ecq_dev
