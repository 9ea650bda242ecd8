// ecq_matmul.cu -- batched-token fused rANS decode + dequant + GEMM on the
// sm_100a tensor cores: y[B, rows] = x[B, cols] . W^T, W the packed
// rANS-coded matrix, B <= 128 tokens per launch. No decoded weight is
// written to HBM: each tile is decoded straight into the shared-memory
// operand of tcgen05.mma.
//
// One persistent CTA per SM walks a contiguous run of work items. An item is
// (row block, K-tile): NW row slabs of 8 rows (N = 8*NW weight rows) by one
// tile width C (128 or 256 columns). Roles:
//   decode warps 0..NW-1   warp w decodes slab (block*NW + w)'s tile of the
//                          item with the GEMV kernel's branch-free rANS step
//                          (tile bytes staged by cp.async.bulk), dequantises
//                          each symbol to fp16 ((sym - 8) * scale, one
//                          rounding) and stores it into the W block in the
//                          tensor core's K-major, no-swizzle layout.
//   loader warps NW..NW+3  one per TMEM lane quadrant: copy the item's x
//                          columns into tensor memory (tcgen05.st; token rows
//                          are TMEM lanes, two fp16 per column, two stages);
//                          lane 0 of the first one issues the MMAs and their
//                          commits. When a row block's run in this CTA ends
//                          they read the fp32 accumulator (tcgen05.ld) and
//                          add it, as 64-bit fixed point (2^-32 units), into
//                          the workspace. Integer addition is associative,
//                          so the sums do not depend on the order in which
//                          the CTAs sharing a row block finish.
// matmul_finish_kernel then converts the sums to fp16 y (a tiled transpose)
// and clears the workspace for the next call.
// MMA: tcgen05.mma.cta_group::1.kind::f16 with A = x (TMEM, M = 128 token
// rows), B = W block (shared-memory descriptor, N = 8*NW rows, K-major),
// D fp32 in TMEM; C/16 instructions of K = 16 per item.
//
// K order: the MMA sums over K, so the W block and x may share any order of
// the columns. Within each 64-column block, column 64q + 32u + j sits at K
// position 64q + 2j + u, so that the two symbols lane j decodes for columns
// j + 64q and j + 64q + 32 are adjacent: one 32-bit store.
// W block: element (n, p) -- n = 8g + r the weight row in the block, p the K
// position -- at byte (p/8)*LBO + 128g + 16r + 2(p%8): 8x8 core matrices of
// 128 contiguous bytes, the NW row groups of one core column adjacent
// (SBO = 128), core columns LBO = 128*NW + 16 bytes apart. The extra 16
// bytes put the eight core columns one warp stores to at once in different
// banks.
//
// Tensor memory (512 columns, the whole SM's): [0, 256) accumulator, D row m
// (token) in lane m, column n; [256, 256 + C) two x stages of C/2 columns.
//
// Shared memory: [stream buffers NW x 2][decode table 64 KB][W block]
// [mbarriers][tmem address, flag]. The stream buffers come first, so the
// read-ahead of a damaged stream past the last buffer lands in the table
// (reads only).
//
// Every wait is bounded (0.2 s): on a timeout the kernel sets
// ECQ_STATUS_TIMEOUT, all roles leave their loops, wait for what they have in
// flight and the TMEM allocation is released before the CTA exits.
#include <algorithm>

#include "ecq_kernels.cuh"

namespace {

using namespace ecq_dev;

constexpr int kLoaderWarps = 4;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCol = 0;
constexpr uint32_t kXCol = 256;
constexpr uint32_t kMaxBatch = 128;

struct MatmulParams {
    const uint8_t* data;
    const uint32_t* tile_offset;
    const uint16_t* stream_len;
    const uint32_t* dec_table;
    const __half* x;       // [batch, cols]
    const __half* scales;  // [rows, ng]
    __half* y;             // [batch, rows]
    unsigned long long* acc;  // [rows, batch] partial sums, 64-bit fixed point (2^-32); zero between calls
    uint32_t* status;
    uint32_t rows, cols, ng, group_size;
    uint32_t n_ktiles, n_slabs, n_blocks, n_items;
    uint32_t buf_bytes, flags, batch;
};

// ---------------------------------------------------------------------------
// tcgen05 wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] . B[smem]^T, kind::f16, one CTA
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive on the mbarrier once every MMA this thread issued so far has completed
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];" : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]) : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// K-major, no-swizzle shared-memory matrix descriptor (sm_100 layout: start,
// leading byte offset = K-direction core stride, stride byte offset = 8-row
// group stride, all in 16-byte units; bit 46 = descriptor version 1).
__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void sts_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
// barrier over the 4 loader warps (named barrier 1), returning whether any
// loader thread passed `v` true
__device__ __forceinline__ bool loader_sync_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v))
        : "memory");
    return r != 0;
}

// Decode tile t (bytes at shared address buf) into this warp's 8 rows of the
// W block; wlane is this lane's address of its first column pair in row 0.
// Lane j's symbols m = 2q and 2q+1 of a row (columns j + 64q and
// j + 64q + 32) are stored as one half2 at K position 64q + 2j. When wait_bar
// is set, the MMAs of the previous item still read the W block: the first
// two rows are held in registers and the warp waits (bounded) before its
// first store. Returns false if that wait timed out.
template <int MPL, int GPL, int NW, bool CONSTANT>
__device__ __forceinline__ bool decode_tile_to_w(const MatmulParams& p, uint32_t t, uint32_t slab, uint32_t kt,
                                                 uint32_t buf, uint32_t tb, uint32_t wlane, int lane,
                                                 uint32_t wait_bar, uint32_t wait_parity) {
    constexpr int NSG = MPL / GPL;
    constexpr int NP = MPL / 2;  // column pairs per lane and row
    constexpr uint32_t LBO = NW * 128 + 16;
    const uint32_t r0 = slab * kTileRows;
    const int rows_here = static_cast<int>(min(static_cast<uint32_t>(kTileRows), p.rows - r0));
    const uint32_t c0 = kt * (MPL * 32);
    const uint32_t len = p.stream_len[t * 32 + lane];
    uint32_t x, a, b0, b1;  // rANS state, next stream byte's shared-window address, read-ahead bytes
    stream_cursor_init(buf, lane, x, a, b0, b1);
    const uint32_t cent = ((p.flags >> ECQ_FLAG_CONSTANT_SYM_SHIFT) & 15u) << 14;
    // lane l < NSG loads the scale of the tile row's group l; its column index is fixed per tile
    const __half* srow = p.scales + static_cast<size_t>(r0) * p.ng + (c0 + (lane < NSG ? lane : 0) * GPL * 32) / p.group_size;
    float sc = lane < NSG ? __half2float(srow[0]) * 6.103515625e-05f : 0.f;  // scale * 2^-14
    bool waiting = wait_bar != 0u;
    bool ok = true;
    uint32_t hold[NP];
#pragma unroll
    for (int q = 0; q < NP; ++q) hold[q] = 0u;
#pragma unroll
    for (int r = 0; r < kTileRows; ++r) {
        if (r >= rows_here) break;
        float sn = 0.f;
        if (lane < NSG && r + 1 < rows_here) sn = __half2float(srow[static_cast<size_t>(r + 1) * p.ng]) * 6.103515625e-05f;
        float g[NSG], nb[NSG];
#pragma unroll
        for (int sg = 0; sg < NSG; ++sg) {
            g[sg] = __shfl_sync(0xffffffffu, sc, sg);
            nb[sg] = g[sg] * -kWeightBias;  // exact: 520 * scale
        }
        uint32_t h[NP];
#pragma unroll
        for (int q = 0; q < NP; ++q) {
            uint32_t e0, e1;
            if constexpr (CONSTANT) {
                e0 = e1 = cent;
            } else {
                e0 = decode_step(x, a, b0, b1, tb);
                e1 = decode_step(x, a, b0, b1, tb);
            }
            // (sym - 8) * scale = (2^23 + sym*2^14) * g - (2^23 + 8*2^14) * g, exact in fp32; one rounding to fp16
            const int s0 = (2 * q) / GPL, s1 = (2 * q + 1) / GPL;  // compile-time once unrolled
            const float f0 = fmaf(__uint_as_float(entry_weight_bits(e0)), g[s0], nb[s0]);
            const float f1 = fmaf(__uint_as_float(entry_weight_bits(e1)), g[s1], nb[s1]);
            const __half2 hv = __floats2half2_rn(f0, f1);
            h[q] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        sc = sn;
        if (waiting) {
            if (r == 0 && rows_here > 1) {
#pragma unroll
                for (int q = 0; q < NP; ++q) hold[q] = h[q];
                continue;
            }
            ok = mbar_wait(wait_bar, wait_parity);
            waiting = false;
            if (r == 1) {
#pragma unroll
                for (int q = 0; q < NP; ++q) sts_u32(wlane + q * 8 * LBO, hold[q]);
            }
        }
        const uint32_t wr = wlane + 16u * r;
#pragma unroll
        for (int q = 0; q < NP; ++q) sts_u32(wr + q * 8 * LBO, h[q]);
    }
    if constexpr (!CONSTANT) {
        if (x != kL || (a - buf - lane) != len * 32u) atomicOr(p.status, ECQ_STATUS_CORRUPT);
    } else {
        if (len != 4u) atomicOr(p.status, ECQ_STATUS_CORRUPT);
    }
    return ok;
}

template <int MPL, int GPL, int NW>
__global__ void __launch_bounds__((NW + kLoaderWarps) * 32, 1) matmul_kernel(MatmulParams p) {
    constexpr int C = MPL * 32;                   // K columns per item
    constexpr int N = NW * 8;                     // weight rows per item (MMA N)
    constexpr uint32_t LBO = NW * 128 + 16;       // W block core-column stride
    constexpr uint32_t W_BYTES = (C / 8) * LBO;
    constexpr uint32_t XCOLS = C / 2;             // TMEM columns per x stage
    constexpr int KSTEPS = C / 16;
    static_assert(NW % 4 == 0 && N % 32 == 0 && N <= 256, "N must be a multiple of 32 up to 256");
    static_assert(kXCol + 2 * XCOLS <= kTmemCols, "x stages exceed tensor memory");
    // instruction descriptor: D f32, A and B f16, both K-major, N >> 3, M = 128 >> 4
    constexpr uint32_t IDESC = (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | ((128u >> 4) << 24);

    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const uint32_t sbase = smem_addr(smem);
    const uint32_t bufs_bytes = NW * 2 * p.buf_bytes;
    const uint32_t tb = sbase + bufs_bytes;  // decode table
    const uint32_t wbuf = tb + kTableBytes;  // W block
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + bufs_bytes + kTableBytes + W_BYTES);
    const uint32_t bar0 = smem_addr(bars);  // [0, 2NW): stream stages of each decode warp
    const uint32_t table_bar = bar0 + 8 * (2 * NW);
    const uint32_t w_full = table_bar + 8;      // NW*32 arrivals: the W block of an item is written
    const uint32_t mma_done0 = w_full + 8;      // two: the MMAs of an item (x stage k&1) completed
    const uint32_t acc_full = mma_done0 + 16;   // the accumulator of a row block's run is final
    volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(bars + 2 * NW + 5);  // [0] tmem [1] abort

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2 * NW + 1; ++i) mbar_init(bar0 + 8 * i, 1);
        mbar_init(w_full, NW * 32);
        mbar_init(mma_done0, 1);
        mbar_init(mma_done0 + 8, 1);
        mbar_init(acc_full, 1);
        misc[1] = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == NW) {
        tmem_alloc(smem_addr(const_cast<uint32_t*>(misc)), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];

    const uint32_t i_begin = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * p.n_items / gridDim.x);
    const uint32_t i_end = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * p.n_items / gridDim.x);

    if (warp < NW) {
        // ------------------------------------------------------------ decode warps
        if (threadIdx.x == 0) {
            mbar_expect_tx(table_bar, kTableBytes);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                bulk_copy_g2s(tb + i * (kTableBytes / 4), reinterpret_cast<const uint8_t*>(p.dec_table) + i * (kTableBytes / 4),
                              kTableBytes / 4, table_bar);
        }
        const uint32_t my_bar0 = bar0 + 16 * warp;
        const uint32_t my_buf0 = sbase + 2 * warp * p.buf_bytes;
        const uint32_t wlane = wbuf + warp * 128 + (lane >> 2) * LBO + (lane & 3) * 4;
        const bool constant = p.flags & ECQ_FLAG_CONSTANT;
        // this warp's slab of an item; false past the last slab (its rows of
        // the W block are then left as they are: they only feed accumulator
        // columns that are never read)
        auto slab_of = [&](uint32_t item, uint32_t& slab, uint32_t& kt) {
            const uint32_t blk = item / p.n_ktiles;
            kt = item - blk * p.n_ktiles;
            slab = blk * NW + warp;
            return slab < p.n_slabs;
        };
        auto issue = [&](uint32_t t, int stage) {
            const uint32_t off = p.tile_offset[t];
            uint32_t bytes = p.tile_offset[t + 1] - off;
            if (bytes > p.buf_bytes || (off & 15u) || (bytes & 15u)) {
                atomicOr(p.status, ECQ_STATUS_BADARG);
                bytes = 0;
            }
            const uint32_t bar = my_bar0 + 8 * stage;
            mbar_expect_tx(bar, bytes);
            if (bytes) bulk_copy_g2s(my_buf0 + stage * p.buf_bytes, p.data + off, bytes, bar);
        };
        uint32_t slab, kt;
        bool any_issued = false;
        if (lane == 0 && i_begin < i_end && slab_of(i_begin, slab, kt)) issue(slab * p.n_ktiles + kt, 0);
        any_issued = i_begin < i_end && slab_of(i_begin, slab, kt);
        // every wait result is made warp-uniform: the loop body shuffles over all 32 lanes
        bool ok = __all_sync(0xffffffffu, mbar_wait(table_bar, 0));
        if (!ok) {
            if (lane == 0) atomicOr(p.status, ECQ_STATUS_TIMEOUT);
            misc[1] = 1u;
        }
        uint32_t phase0 = 0, phase1 = 0;
        for (uint32_t i = i_begin; ok && i < i_end; ++i) {
            if (__any_sync(0xffffffffu, misc[1] != 0u)) break;
            const uint32_t k = i - i_begin;
            const int stage = k & 1;  // the items with a slab are a prefix of the run
            if (slab_of(i, slab, kt)) {
                uint32_t s1, k1;
                if (i + 1 < i_end && slab_of(i + 1, s1, k1)) {
                    __syncwarp();
                    if (lane == 0) {
                        fence_proxy_async();
                        issue(s1 * p.n_ktiles + k1, stage ^ 1);
                    }
                }
                const uint32_t parity = stage ? phase1 : phase0;
                if (!__all_sync(0xffffffffu, mbar_wait(my_bar0 + 8 * stage, parity))) {
                    if (lane == 0) atomicOr(p.status, ECQ_STATUS_TIMEOUT);
                    misc[1] = 1u;
                    ok = false;
                    break;
                }
                if (stage) phase1 ^= 1; else phase0 ^= 1;
                uint32_t buf = my_buf0 + stage * p.buf_bytes;
                asm volatile("" : "+r"(buf)::"memory");  // keep this tile's byte loads after its wait
                const uint32_t wbar = k ? mma_done0 + 8 * ((k - 1) & 1) : 0u;
                const uint32_t wpar = k ? ((k - 1) >> 1) & 1 : 0u;
                const uint32_t t = slab * p.n_ktiles + kt;
                const bool wok = constant
                                     ? decode_tile_to_w<MPL, GPL, NW, true>(p, t, slab, kt, buf, tb, wlane, lane, wbar, wpar)
                                     : decode_tile_to_w<MPL, GPL, NW, false>(p, t, slab, kt, buf, tb, wlane, lane, wbar, wpar);
                if (!__all_sync(0xffffffffu, wok)) {
                    if (lane == 0) atomicOr(p.status, ECQ_STATUS_TIMEOUT);
                    misc[1] = 1u;
                    ok = false;
                    break;
                }
            } else if (k) {
                // no slab here, but this warp must not arrive for item k before
                // the whole CTA has arrived for item k-1 (whose MMAs then ran)
                if (!__all_sync(0xffffffffu, mbar_wait(mma_done0 + 8 * ((k - 1) & 1), ((k - 1) >> 1) & 1))) {
                    if (lane == 0) atomicOr(p.status, ECQ_STATUS_TIMEOUT);
                    misc[1] = 1u;
                    ok = false;
                    break;
                }
            }
            fence_proxy_async();  // this lane's W stores, before the tensor core reads them
            mbar_arrive(w_full);
        }
        // never leave a bulk copy in flight when leaving early
        if (!ok && any_issued) {
            mbar_wait(my_bar0, phase0);
            mbar_wait(my_bar0 + 8, phase1);
        }
    } else {
        // ------------------------------------------------------------ loader warps
        const uint32_t lw = warp - NW;  // == warp % 4: TMEM lanes [32 lw, 32 lw + 32)
        const uint32_t m = 32 * lw + lane;
        const bool has_row = m < p.batch;
        const uint4* xrow = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(has_row ? m : 0) * p.cols);
        const uint32_t lane_base = tmem + ((32 * lw) << 16);

        auto store_x = [&](uint32_t item, uint32_t stage) {
            const uint32_t kt = item % p.n_ktiles;
            const uint4* src = xrow + kt * (C / 8);
#pragma unroll 1
            for (uint32_t c = 0; c < XCOLS / 32; ++c) {
                uint32_t v[32];
                uint32_t u[32];  // x[64c .. 64c + 63] of this token row, two fp16 per word
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint4 w = has_row ? __ldg(src + c * 8 + j) : make_uint4(0u, 0u, 0u, 0u);
                    u[4 * j] = w.x;
                    u[4 * j + 1] = w.y;
                    u[4 * j + 2] = w.z;
                    u[4 * j + 3] = w.w;
                }
                // the W block's K order: column j holds x[64c + j] and x[64c + 32 + j]
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    v[j] = __byte_perm(u[j >> 1], u[16 + (j >> 1)], (j & 1) ? 0x7632 : 0x5410);
                tmem_st32(lane_base + kXCol + stage * XCOLS + 32 * c, v);
            }
            tmem_wait_st();
        };

        // accumulator of a finished run -> workspace (fire-and-forget 64-bit
        // adds; matmul_finish_kernel turns the sums into y after the kernel)
        auto epilogue = [&](uint32_t item, uint32_t run) {
            const bool got = __all_sync(0xffffffffu, mbar_wait(acc_full, run & 1));  // tcgen05.ld below is warp-wide
            if (!got && lane == 0) atomicOr(p.status, ECQ_STATUS_TIMEOUT);
            tc_fence_after();
            const uint32_t row0 = (item / p.n_ktiles) * N;
            if (got) {
#pragma unroll 1
                for (uint32_t c = 0; c < N / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld32(lane_base + kAccCol + 32 * c, v);
                    tmem_wait_ld();
                    if (has_row) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const uint32_t row = row0 + 32 * c + j;
                            if (row < p.rows)
                                atomicAdd(p.acc + static_cast<size_t>(row) * p.batch + m,
                                          static_cast<unsigned long long>(__float2ll_rn(__uint_as_float(v[j]) * 4294967296.0f)));
                        }
                    }
                }
            }
        };

        uint32_t issued = 0;  // items whose MMAs lane 0 of loader warp 0 issued
        uint32_t run = 0;
        if (i_begin < i_end) store_x(i_begin, 0);
        tc_fence_before();
        bool abort = loader_sync_any(misc[1] != 0u);
        for (uint32_t i = i_begin; !abort && i < i_end; ++i) {
            const uint32_t k = i - i_begin;
            const uint32_t stage = k & 1;
            const uint32_t kt = i % p.n_ktiles;
            const bool first = (i == i_begin) || kt == 0;
            const bool last = (i + 1 == i_end) || kt + 1 == p.n_ktiles;
            if (lw == 0) {
                if (lane == 0) {
                    if (mbar_wait(w_full, k & 1)) {
                        tc_fence_after();
#pragma unroll
                        for (int s = 0; s < KSTEPS; ++s) {
                            const uint64_t bdesc = smem_desc_kmajor(wbuf + 2u * s * LBO, LBO, 128u);
                            mma_ts(tmem + kAccCol, tmem + kXCol + stage * XCOLS + 8u * s, bdesc, IDESC,
                                   (first && s == 0) ? 0u : 1u);
                        }
                        mma_commit(mma_done0 + 8 * stage);
                        if (last) mma_commit(acc_full);
                        issued = k + 1;
                    } else {
                        atomicOr(p.status, ECQ_STATUS_TIMEOUT);
                        misc[1] = 1u;
                    }
                }
                __syncwarp();
            }
            if (i + 1 < i_end) {
                // stage (k+1)&1 was last read by the MMAs of item k-1
                bool free_ok = true;
                if (k >= 1) free_ok = __all_sync(0xffffffffu, mbar_wait(mma_done0 + 8 * ((k + 1) & 1), ((k - 1) >> 1) & 1));
                if (free_ok) {
                    store_x(i + 1, (k + 1) & 1);
                } else {
                    if (lane == 0) atomicOr(p.status, ECQ_STATUS_TIMEOUT);
                    misc[1] = 1u;
                }
            }
            if (last) {
                epilogue(i, run);
                ++run;
            }
            tc_fence_before();
            abort = loader_sync_any(misc[1] != 0u);
        }
        // every MMA issued has completed before the tensor memory is released
        if (lw == 0 && lane == 0 && issued)
            mbar_wait(mma_done0 + 8 * ((issued - 1) & 1), ((issued - 1) >> 1) & 1);
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == NW) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// y[b, r] = acc[r, b] * 2^-32 (fp16), acc cleared: a 32 x 32 tiled transpose
// so that both the workspace reads and the y writes are coalesced.
__global__ void __launch_bounds__(256) matmul_finish_kernel(unsigned long long* __restrict__ acc, __half* __restrict__ y,
                                                            uint32_t rows, uint32_t batch) {
    __shared__ float tile[32][33];
    const uint32_t r0 = blockIdx.x * 32, b0 = blockIdx.y * 32;
    const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
#pragma unroll
    for (uint32_t k = 0; k < 32; k += 8) {
        const uint32_t r = r0 + ty + k, b = b0 + tx;
        float v = 0.f;
        if (r < rows && b < batch) {
            unsigned long long* src = acc + static_cast<size_t>(r) * batch + b;
            v = __ll2float_rn(static_cast<long long>(__ldcg(src))) * 2.3283064365386963e-10f;
            __stcg(src, 0ull);
        }
        tile[ty + k][tx] = v;
    }
    __syncthreads();
#pragma unroll
    for (uint32_t k = 0; k < 32; k += 8) {
        const uint32_t b = b0 + ty + k, r = r0 + tx;
        if (r < rows && b < batch) y[static_cast<size_t>(b) * rows + r] = __float2half_rn(tile[tx][ty + k]);
    }
}

// ---------------------------------------------------------------------------
// launch plumbing
// ---------------------------------------------------------------------------
using MatmulFn = void (*)(MatmulParams);

template <int NW>
MatmulFn pick_matmul_nw(int mpl, int gpl) {
#define ECQ_MM_CASE(M_, G_) \
    if (mpl == M_ && gpl == G_) return matmul_kernel<M_, G_, NW>;
    ECQ_MM_CASE(4, 1) ECQ_MM_CASE(4, 2) ECQ_MM_CASE(4, 4)
    ECQ_MM_CASE(8, 1) ECQ_MM_CASE(8, 2) ECQ_MM_CASE(8, 4) ECQ_MM_CASE(8, 8)
#undef ECQ_MM_CASE
    return nullptr;
}

MatmulFn pick_matmul(int nw, int mpl, int gpl) {
    switch (nw) {
        case 28: return pick_matmul_nw<28>(mpl, gpl);
        case 20: return pick_matmul_nw<20>(mpl, gpl);
        case 12: return pick_matmul_nw<12>(mpl, gpl);
        default: return nullptr;
    }
}

constexpr int kNwChoices[] = {28, 20, 12};

size_t matmul_smem(int nw, int mpl, uint32_t buf) {
    const size_t w_bytes = static_cast<size_t>(mpl * 32 / 8) * (nw * 128 + 16);
    return static_cast<size_t>(nw) * 2 * buf + kTableBytes + w_bytes + 8 * (2 * nw + 5) + 16;
}

struct MatmulShape {
    int mpl, gpl, nw;
    uint32_t buf;
    size_t smem;
    uint32_t n_slabs, n_blocks, n_ktiles;
};

int32_t matmul_shape(const ecq_matrix_view* m, MatmulShape* s) {
    if (!m || !m->data || !m->tile_offset || !m->stream_len || !m->dec_table || !m->rows || !m->cols || !m->n_tiles)
        return ECQ_ERR_ARG;
    if (m->tile_rows != kTileRows) return ECQ_ERR_UNSUPPORTED;
    if (m->tile_cols != 128 && m->tile_cols != 256) return ECQ_ERR_UNSUPPORTED;
    if (m->cols % m->tile_cols) return ECQ_ERR_SHAPE;
    const int mpl = static_cast<int>(m->tile_cols / 32);
    const uint32_t g = m->group_size;
    int gpl = mpl;
    if (g == 0 || g % 32) return ECQ_ERR_UNSUPPORTED;
    if (g < m->tile_cols) {
        if (m->tile_cols % g) return ECQ_ERR_UNSUPPORTED;
        gpl = static_cast<int>(g / 32);
    } else if (g % m->tile_cols) {
        return ECQ_ERR_UNSUPPORTED;
    }
    const uint32_t slabs = (m->rows + kTileRows - 1) / kTileRows;
    if (m->n_tiles != slabs * (m->cols / m->tile_cols)) return ECQ_ERR_SHAPE;
    uint32_t buf = (m->max_tile_bytes + 127u) & ~127u;
    if (buf < 128) buf = 128;
    for (int nw : kNwChoices) {
        const size_t smem = matmul_smem(nw, mpl, buf);
        if (smem <= static_cast<size_t>(kMaxSmem) && pick_matmul(nw, mpl, gpl)) {
            s->mpl = mpl;
            s->gpl = gpl;
            s->nw = nw;
            s->buf = buf;
            s->smem = smem;
            s->n_slabs = slabs;
            s->n_blocks = (slabs + nw - 1) / nw;
            s->n_ktiles = m->cols / m->tile_cols;
            return ECQ_OK;
        }
    }
    return ECQ_ERR_UNSUPPORTED;
}

int64_t matmul_workspace(const ecq_matrix_view* m, uint32_t batch) {
    const uint64_t b = batch < kMaxBatch ? batch : kMaxBatch;
    return static_cast<int64_t>(static_cast<uint64_t>(m->rows) * b * 8);
}

}  // namespace

extern "C" {

int64_t ecq_matmul_workspace_bytes(const ecq_matrix_view* m, uint32_t batch) {
    MatmulShape s;
    const int32_t rc = matmul_shape(m, &s);
    if (rc != ECQ_OK) return rc;
    if (batch == 0) return ECQ_ERR_ARG;
    return matmul_workspace(m, batch);
}

int32_t ecq_matmul(const ecq_matrix_view* m, const void* x_f16, const void* scales_f16, void* y_f16, uint32_t batch,
                   void* workspace, int64_t workspace_bytes, uint32_t* d_status, void* stream) {
    if (!x_f16 || !scales_f16 || !y_f16 || !d_status || batch == 0) return ECQ_ERR_ARG;
    MatmulShape s;
    const int32_t rc = matmul_shape(m, &s);
    if (rc != ECQ_OK) return rc;
    if (!workspace || workspace_bytes < matmul_workspace(m, batch)) return ECQ_ERR_WORKSPACE;
    // x rows are read as 16-byte vectors
    if ((reinterpret_cast<uintptr_t>(x_f16) & 15u) || (m->cols & 7u)) return ECQ_ERR_UNSUPPORTED;
    MatmulFn fn = pick_matmul(s.nw, s.mpl, s.gpl);
    if (!fn || !ensure_smem_limit(reinterpret_cast<const void*>(fn), kMaxSmem)) return ECQ_ERR_CUDA;
    const uint32_t n_items = s.n_blocks * s.n_ktiles;
    const int ctas = static_cast<int>(std::min<uint32_t>(static_cast<uint32_t>(sm_count_cached()), n_items));
    for (uint32_t b0 = 0; b0 < batch; b0 += kMaxBatch) {
        MatmulParams p{};
        p.data = m->data;
        p.tile_offset = m->tile_offset;
        p.stream_len = m->stream_len;
        p.dec_table = m->dec_table;
        p.x = static_cast<const __half*>(x_f16) + static_cast<size_t>(b0) * m->cols;
        p.scales = static_cast<const __half*>(scales_f16);
        p.y = static_cast<__half*>(y_f16) + static_cast<size_t>(b0) * m->rows;
        p.acc = static_cast<unsigned long long*>(workspace);
        p.status = d_status;
        p.rows = m->rows;
        p.cols = m->cols;
        p.group_size = m->group_size;
        p.ng = (m->cols + m->group_size - 1) / m->group_size;
        p.n_ktiles = s.n_ktiles;
        p.n_slabs = s.n_slabs;
        p.n_blocks = s.n_blocks;
        p.n_items = n_items;
        p.buf_bytes = s.buf;
        p.flags = m->flags;
        p.batch = std::min(kMaxBatch, batch - b0);
        // the full shared-memory request keeps one CTA per SM: each CTA takes
        // all 512 TMEM columns, so a second resident CTA would only wait
        fn<<<ctas, (s.nw + kLoaderWarps) * 32, kMaxSmem, static_cast<cudaStream_t>(stream)>>>(p);
        if (cudaGetLastError() != cudaSuccess) return ECQ_ERR_CUDA;
        const dim3 fgrid((m->rows + 31) / 32, (p.batch + 31) / 32);
        matmul_finish_kernel<<<fgrid, 256, 0, static_cast<cudaStream_t>(stream)>>>(p.acc, p.y, m->rows, p.batch);
        if (cudaGetLastError() != cudaSuccess) return ECQ_ERR_CUDA;
    }
    return ECQ_OK;
}

}  // extern "C"
