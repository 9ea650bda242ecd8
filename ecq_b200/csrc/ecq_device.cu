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
#include <algorithm>

#include "ecq_comm.h"
#include "ecq_kernels.cuh"

namespace {

using namespace ecq_dev;

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
            sym = (e >> 14) & 15u;
            x = (e >> 18) * (x >> 14) + (e & 16383u);
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
    uint8_t* sym_out;      // [rows, cols] (decode mode: symbols)
    __half* w_out;         // [rows, cols] (decode mode: dequantised fp16 weights, when set)
    float* partials;       // [n_tiles, 8, nb] (GEMV modes)
    uint32_t* slab_count;  // [n_slabs] (GEMV modes; first in the workspace)
    uint32_t* status;
    uint32_t rows, cols, ng, group_size;
    uint32_t n_ktiles, n_tiles;
    uint32_t buf_bytes;
    uint32_t flags;
    uint32_t x_bytes;  // x staged in shared memory after the table (0: read x from global)
    uint32_t xs_bytes;  // batched GEMV: x of nb tokens staged as fp16 [cols][nb] after the table
    uint32_t nb, batch_here;  // batched GEMV: tokens per launch, of which the first batch_here are real
    // tensor-parallel push (ecq_gemv_tp; tp_world == 0 otherwise): y goes as
    // fp32 partials to every rank's exchange buffer instead of to p.y
    uint8_t* tp_peer[ECQ_TP_MAX_RANKS];
    uint32_t* tp_epoch;  // this rank's epoch counter
    uint32_t tp_world, tp_rank, tp_nmax;
    // fused epilogue of a batch-1 GEMV (ecq_gemv_fused; epi_kind 0 otherwise)
    uint32_t epi_kind;
    uint32_t epi_part_rows, epi_head_dim;
    int64_t epi_cache_stride;
    const __half* epi_cos;
    const __half* epi_sin;
    __half* epi_kc;
    __half* epi_vc;
};

// what matrix_kernel does with the decoded symbols
constexpr int kModeSymbols = 0;  // store uint8 symbols
constexpr int kModeGemv = 1;     // fused dequant + GEMV
constexpr int kModeWeights = 2;  // store dequantised fp16 weights
constexpr int kModePacked4 = 3;  // store symbols as packed nibbles (column 2i low, 2i+1 high)
constexpr int kModeGemvBatch = 4;  // fused dequant + GEMV for NB tokens, each tile decoded once
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

// Row-slab completion. A tile's 8 row sums go to the workspace and lane 0
// bumps the slab's counter with an acquire-release atomic; the warp does not
// wait for the atomic's result: it checks it after its next tile (or at the
// end of its run). The warp that completes a slab sums the slab's partials in
// fixed order (y is deterministic) and writes y.
struct PendingSlab {
    uint32_t slab;  // 0xffffffff: nothing pending
    uint32_t old;   // counter value before this warp's increment (lane 0)
    int rows;
};

__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* addr, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
    return old;
}

// Tensor-parallel push of one finished row slab: each row sum goes to
// slot[e & 1][rank][row] of every rank's exchange buffer (through CUDA IPC
// mappings for the peers) as ONE 8-byte store of (fp32 value, e + 1): the
// consumer polls each slot until its epoch half reads e + 1, and an aligned
// 8-byte store is never seen half-written, so no fence, counter or separate
// flag is needed (the low-latency scheme of small all-reduces). Buffer
// layout: include/ecq_comm.h.
__device__ __forceinline__ void st_relaxed_sys_u64(uint8_t* addr, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ void tp_push_slab(const MatrixParams& p, uint32_t slab, int row, bool writer, float s) {
    if (!writer) return;
    const uint32_t e = *reinterpret_cast<volatile const uint32_t*>(p.tp_epoch);
    const size_t off = 256u + ((static_cast<size_t>(e & 1u) * p.tp_world + p.tp_rank) * p.tp_nmax +
                               static_cast<size_t>(slab) * kTileRows + row) * sizeof(uint64_t);
    const uint64_t v = (static_cast<uint64_t>(e + 1u) << 32) | __float_as_uint(s);
    for (uint32_t q = 0; q < p.tp_world; ++q) st_relaxed_sys_u64(p.tp_peer[q] + off, v);
}

// A finished row's value through the fused epilogue (all lanes call it; the
// lanes with `writer` set store). Rows 2i and 2i+1 of a slab sit in lanes
// 2i and 2i+1 of the same 8-lane group, so a pair meets with one shuffle.
//  ROPE_KV:  y = q | k | v, each part_rows rows (heads x head_dim); q and k
//            rotate pairs (2i, 2i+1) by angle index i (cos, sin [head_dim/2]);
//            the rotated k and the v rows also go to the KV-cache slot
//            (head h at h * cache_stride). The arithmetic is ecq_rope_kv_f16's
//            on the fp16-rounded GEMV outputs.
//  SILU_MUL: rows interleave gate and up (row 2j gate j, 2j + 1 up j); y[j] =
//            silu(gate j) * up j, the arithmetic of ecq_silu_mul_f16.
__device__ __forceinline__ void gemv_epilogue(const MatrixParams& p, uint32_t slab, int row, bool writer, float s) {
    const uint32_t r = slab * kTileRows + row;
    const float v = __half2float(__float2half_rn(s));
    const float pv = __shfl_xor_sync(0xffffffffu, v, 1);
    if (p.epi_kind == ECQ_EPI_ROPE_KV) {
        const uint32_t part = r / p.epi_part_rows, rr = r - part * p.epi_part_rows;
        const uint32_t head = rr / p.epi_head_dim, d = rr - head * p.epi_head_dim;
        __half out = __float2half_rn(v);
        if (part < 2) {
            const float c = __half2float(p.epi_cos[d >> 1]), sn = __half2float(p.epi_sin[d >> 1]);
            out = (d & 1) ? __float2half_rn(pv * sn + v * c) : __float2half_rn(v * c - pv * sn);
        }
        if (writer) {
            p.y[r] = out;
            if (part == 1) p.epi_kc[head * p.epi_cache_stride + d] = out;
            if (part == 2) p.epi_vc[head * p.epi_cache_stride + d] = out;
        }
    } else {  // ECQ_EPI_SILU_MUL
        if (writer && !(row & 1)) {
            const float g = __half2float(__float2half_rn(v / (1.f + __expf(-v))));
            p.y[r >> 1] = __float2half_rn(g * pv);
        }
    }
}

__device__ __forceinline__ void complete_pending(const MatrixParams& p, PendingSlab& pend, int lane) {
    if (pend.slab == 0xffffffffu) return;
    const uint32_t old = __shfl_sync(0xffffffffu, pend.old, 0);
    if (old == p.n_ktiles - 1) {
        __threadfence();
        const uint32_t slab = pend.slab;
        const int row = lane & 7, kp = lane >> 3;
        const float* base = p.partials + static_cast<size_t>(slab) * p.n_ktiles * kTileRows;
        float s = 0.f;
        for (uint32_t k = kp; k < p.n_ktiles; k += 4) s += __ldcg(base + static_cast<size_t>(k) * kTileRows + row);
        s += __shfl_xor_sync(0xffffffffu, s, 8);
        s += __shfl_xor_sync(0xffffffffu, s, 16);
        if (p.tp_world != 0) {
            tp_push_slab(p, slab, row, kp == 0 && row < pend.rows, s);
        } else if (p.epi_kind != 0) {
            gemv_epilogue(p, slab, row, kp == 0 && row < pend.rows, s);
        } else {
            if (kp == 0 && row < pend.rows) p.y[slab * kTileRows + row] = __float2half_rn(s);
        }
        if (lane == 0) p.slab_count[slab] = 0u;
    }
    pend.slab = 0xffffffffu;
}

__device__ __forceinline__ void finish_tile(const MatrixParams& p, uint32_t t, uint32_t slab, float (&acc)[8],
                                            int rows_here, int lane, PendingSlab& pend) {
    complete_pending(p, pend, lane);
    // rows past a short slab's end hold 0
    const float v = transpose_reduce8(acc, lane);
    // lane 4*b2 + 8*b3 + 16*b4 holds row 4*b4 + 2*b3 + b2
    float rv[kTileRows];
#pragma unroll
    for (int r = 0; r < kTileRows; ++r)
        rv[r] = __shfl_sync(0xffffffffu, v, ((r >> 2) & 1) * 16 + ((r >> 1) & 1) * 8 + (r & 1) * 4);
    uint32_t old = 0;
    if (lane == 0) {
        float4* dst = reinterpret_cast<float4*>(p.partials + static_cast<size_t>(t) * kTileRows);
        dst[0] = make_float4(rv[0], rv[1], rv[2], rv[3]);
        dst[1] = make_float4(rv[4], rv[5], rv[6], rv[7]);
        old = atom_add_acq_rel(p.slab_count + slab, 1u);
    }
    pend.slab = slab;
    pend.old = old;
    pend.rows = rows_here;
}

// Decode one tile (buf = offset of its bytes in shared memory) and either
// accumulate its GEMV contribution or store its symbols.
template <int MPL, int GPL, int MODE, bool CONSTANT>
__device__ __forceinline__ void process_tile(const MatrixParams& p, uint32_t t, uint32_t slab, uint32_t kt,
                                             uint32_t buf, uint32_t tb, int lane, PendingSlab& pend) {
    constexpr int NSG = MPL / GPL;  // scale groups per tile row
    const uint32_t r0 = slab * kTileRows;
    const int rows_here = static_cast<int>(min(static_cast<uint32_t>(kTileRows), p.rows - r0));
    const uint32_t c0 = kt * (MPL * 32);
    const uint32_t len = p.stream_len[t * 32 + lane];

    uint32_t x, a, b0, b1;  // rANS state, next stream byte's shared-window address, read-ahead bytes
    stream_cursor_init(buf, lane, x, a, b0, b1);
    const uint32_t cent = ((p.flags >> ECQ_FLAG_CONSTANT_SYM_SHIFT) & 15u) << 14;  // constant table: sym field

    constexpr bool GEMV = MODE == kModeGemv;
    constexpr bool SCALED = MODE == kModeGemv || MODE == kModeWeights;  // needs the group scales
    float xs[MPL];  // x * 2^-14 (exact), this lane's columns of the tile
    float acc[kTileRows];
    // Every group scale of the tile, loaded once up front (one load per lane
    // instead of a dependent load per row): value v = r * NSG + sg (row r,
    // group sg) sits in lane v % 32 of sca[v / 32]; rows past the matrix read 0.
    constexpr int NSR = (kTileRows * NSG + 31) / 32;
    float sca[NSR];
    if constexpr (SCALED) {
        const uint32_t g0 = c0 / p.group_size;  // the tile's first group column
#pragma unroll
        for (int k = 0; k < NSR; ++k) {
            const int v = 32 * k + lane;
            const int r = v / NSG;
            float s = 0.f;
            if (r < rows_here) s = __half2float(p.scales[static_cast<size_t>(r0 + r) * p.ng + g0 + (v % NSG)]);
            if constexpr (MODE == kModeWeights) s *= 6.103515625e-05f;  // scale * 2^-14
            sca[k] = s;
        }
    }
    if constexpr (GEMV) {
#pragma unroll
        for (int m = 0; m < MPL; ++m) {
            // x is staged in shared memory right after the table (when it fits)
            const float xv = p.x_bytes ? __half2float(__ushort_as_half(lds_u16(tb + kTableBytes + 2u * (c0 + 32 * m + lane))))
                                       : __half2float(p.x[c0 + 32 * m + lane]);
            xs[m] = xv * 6.103515625e-05f;
        }
#pragma unroll
        for (int r = 0; r < kTileRows; ++r) acc[r] = 0.f;
    }
    // x pairs packed once per tile for the f32x2 multiply-add of the row loop
    constexpr bool PAIRS = GEMV && !CONSTANT && (GPL % 2 == 0);
    uint64_t xp[PAIRS ? MPL / 2 : 1];
    if constexpr (PAIRS) {
#pragma unroll
        for (int i = 0; i < MPL / 2; ++i) xp[i] = pack2(__float_as_uint(xs[2 * i]), __float_as_uint(xs[2 * i + 1]));
    }

    // the row loop is unrolled: a static row index, so a GEMV row's sum lands in
    // acc[r] with no register shuffling, and rows overlap in the schedule
#pragma unroll
    for (int r = 0; r < kTileRows; ++r) {
        if (r >= rows_here) break;
        float rowacc = 0.f;
        float sreg = 0.f;  // the register of sca holding row r's scales
        if constexpr (SCALED) {
            if constexpr (NSR == 1) {
                sreg = sca[0];
            } else {
                const int k = (r * NSG) >> 5;
                sreg = sca[0];
#pragma unroll
                for (int kk = 1; kk < NSR; ++kk) sreg = k == kk ? sca[kk] : sreg;
            }
        }
#pragma unroll
        for (int sg = 0; sg < NSG; ++sg) {
            float part = 0.f;
            if constexpr (PAIRS) {
                // two symbols per packed f32x2 add + fma
                uint64_t part2 = 0;
#pragma unroll
                for (int mm = 0; mm < GPL; mm += 2) {
                    const int m = sg * GPL + mm;
                    const uint32_t e0 = decode_step(x, a, b0, b1, tb);
                    const uint32_t e1 = decode_step(x, a, b0, b1, tb);
                    const uint64_t w2 = add2(pack2(entry_weight_bits(e0), entry_weight_bits(e1)), kNegBias2);
                    part2 = fma2(w2, xp[m / 2], part2);
                }
                float lo, hi;
                unpack2(part2, lo, hi);
                part = lo + hi;
            } else {
                float gscale = 0.f;
                if constexpr (MODE == kModeWeights) gscale = __shfl_sync(0xffffffffu, sreg, (r * NSG + sg) & 31);
                (void)gscale;
#pragma unroll
                for (int mm = 0; mm < GPL; ++mm) {
                    const int m = sg * GPL + mm;
                    uint32_t e;
                    if constexpr (CONSTANT) {
                        e = cent;
                    } else {
                        e = decode_step(x, a, b0, b1, tb);
                    }
                    const size_t idx = static_cast<size_t>(r0 + r) * p.cols + c0 + 32 * m + lane;
                    if constexpr (GEMV) {
                        part = fmaf(entry_weight(e), xs[m], part);
                    } else if constexpr (MODE == kModeWeights) {
                        // (sym - 8) * 2^14 exactly, times scale * 2^-14: one rounding to fp16
                        p.w_out[idx] = __float2half_rn(entry_weight(e) * gscale);
                    } else if constexpr (MODE == kModePacked4) {
                        // lanes 2i and 2i+1 hold columns 2i and 2i+1 (idx is even on even lanes)
                        const uint32_t sv = (e >> 14) & 15u;
                        const uint32_t hi = __shfl_down_sync(0xffffffffu, sv, 1);
                        if (!(lane & 1)) p.sym_out[idx >> 1] = static_cast<uint8_t>(sv | (hi << 4));
                    } else {
                        p.sym_out[idx] = static_cast<uint8_t>((e >> 14) & 15u);
                    }
                }
            }
            if constexpr (GEMV) rowacc = fmaf(__shfl_sync(0xffffffffu, sreg, (r * NSG + sg) & 31), part, rowacc);
        }
        if constexpr (GEMV) acc[r] = rowacc;
    }
    if constexpr (!CONSTANT) {
        if (x != kL || (a - buf - lane) != len * 32u) atomicOr(p.status, ECQ_STATUS_CORRUPT);
    } else {
        if (len != 4u) atomicOr(p.status, ECQ_STATUS_CORRUPT);
    }

    if constexpr (GEMV) finish_tile(p, t, slab, acc, rows_here, lane, pend);
}

// Reduce v[0..N) (N = 2, 4 or 8) over the 32 lanes in a fixed order. Lane l
// ends with the total of value index (l>>4 & 1)*N/2 + (l>>3 & 1)*N/4 +
// (l>>2 & 1)*N/8 (the terms that exist for N); the lanes whose bits below
// log2(N)... are zero hold each index once (see reduce_owner).
template <int N>
__device__ __forceinline__ float transpose_reduce(float (&v)[N], int lane) {
    if constexpr (N == 8) {
        return transpose_reduce8(v, lane);
    } else {
        int w = N;
#pragma unroll
        for (int bit = 16; w > 1; bit >>= 1) {
            const bool hi = lane & bit;
#pragma unroll
            for (int i = 0; i < w / 2; ++i) {
                const float send = hi ? v[i] : v[i + w / 2];
                const float keep = hi ? v[i + w / 2] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
            }
            w >>= 1;
        }
        constexpr int first_full = N == 4 ? 4 : 8;  // the bit after the halving levels
#pragma unroll
        for (int bit = first_full; bit; bit >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], bit);
        return v[0];
    }
}
// value index transpose_reduce<N> leaves in `lane`, and whether this lane is
// the one that stores it
template <int N>
__device__ __forceinline__ int reduce_index(int lane) {
    if constexpr (N == 8) return ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
    if constexpr (N == 4) return ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
    return (lane >> 4) & 1;
}
template <int N>
__device__ __forceinline__ bool reduce_owner(int lane) {
    return (lane & (N == 8 ? 3 : (N == 4 ? 7 : 15))) == 0;
}

// x of NB tokens for one column, fp16 x 8 (pairs of tokens), from the staged
// [cols][NB] block
template <int NB>
__device__ __forceinline__ void lds_x(uint32_t addr, __half2 (&xh)[NB / 2]) {
    if constexpr (NB == 8) {
        uint32_t a, b, c, d;
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr));
        xh[0] = *reinterpret_cast<__half2*>(&a);
        xh[1] = *reinterpret_cast<__half2*>(&b);
        xh[2] = *reinterpret_cast<__half2*>(&c);
        xh[3] = *reinterpret_cast<__half2*>(&d);
    } else if constexpr (NB == 4) {
        uint32_t a, b;
        asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr));
        xh[0] = *reinterpret_cast<__half2*>(&a);
        xh[1] = *reinterpret_cast<__half2*>(&b);
    } else {
        uint32_t a;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(a) : "r"(addr));
        xh[0] = *reinterpret_cast<__half2*>(&a);
    }
}

// Batched GEMV: the slab's last tile sums the partials of its 8 rows x NB
// tokens over the K-tiles in fixed order and writes y[b, row].
template <int NB>
__device__ __forceinline__ void complete_pending_batch(const MatrixParams& p, PendingSlab& pend, int lane) {
    if (pend.slab == 0xffffffffu) return;
    const uint32_t old = __shfl_sync(0xffffffffu, pend.old, 0);
    if (old == p.n_ktiles - 1) {
        __threadfence();
        const uint32_t slab = pend.slab;
        const float* base = p.partials + static_cast<size_t>(slab) * p.n_ktiles * kTileRows * NB;
#pragma unroll
        for (int v = lane; v < kTileRows * NB; v += 32) {
            const int row = v / NB, b = v % NB;
            float s = 0.f;
            for (uint32_t k = 0; k < p.n_ktiles; ++k) s += __ldcg(base + static_cast<size_t>(k) * kTileRows * NB + v);
            if (row < pend.rows && b < static_cast<int>(p.batch_here))
                p.y[static_cast<size_t>(b) * p.rows + slab * kTileRows + row] = __float2half_rn(s);
        }
        if (lane == 0) p.slab_count[slab] = 0u;
    }
    pend.slab = 0xffffffffu;
}

// Decode one tile once and accumulate its contribution for NB tokens. Per
// symbol: the weight (s - 8) / 8 exactly in both halves of an fp16 pair, times
// the NB tokens' x * 8 (fp16 pairs from shared memory), summed in fp16 over
// the GPL symbols a lane holds of one scale group, then in fp32 with the
// group scale; per row, a fixed-order warp reduction of the NB sums.
template <int MPL, int GPL, int NB, bool CONSTANT>
__device__ __forceinline__ void process_tile_batch(const MatrixParams& p, uint32_t t, uint32_t slab, uint32_t kt,
                                                   uint32_t buf, uint32_t tb, uint32_t xsb, int lane,
                                                   PendingSlab& pend) {
    constexpr int NSG = MPL / GPL;
    constexpr int NH = NB / 2;
    const uint32_t r0 = slab * kTileRows;
    const int rows_here = static_cast<int>(min(static_cast<uint32_t>(kTileRows), p.rows - r0));
    const uint32_t c0 = kt * (MPL * 32);
    const uint32_t len = p.stream_len[t * 32 + lane];

    uint32_t x, a, b0, b1;  // rANS state, next stream byte's shared-window address, read-ahead bytes
    stream_cursor_init(buf, lane, x, a, b0, b1);
    const uint32_t cent = ((p.flags >> ECQ_FLAG_CONSTANT_SYM_SHIFT) & 15u) << 14;

    constexpr int NSR = (kTileRows * NSG + 31) / 32;
    float sca[NSR];
    {
        const uint32_t g0 = c0 / p.group_size;
#pragma unroll
        for (int k = 0; k < NSR; ++k) {
            const int v = 32 * k + lane;
            const int r = v / NSG;
            float sv = 0.f;
            if (r < rows_here) sv = __half2float(p.scales[static_cast<size_t>(r0 + r) * p.ng + g0 + (v % NSG)]);
            sca[k] = sv;
        }
    }
    const uint32_t xcol = xsb + (c0 + lane) * (2u * NB);  // this lane's column of the tile, token block

#pragma unroll 1
    for (int r = 0; r < rows_here; ++r) {
        float sreg = sca[0];
        if constexpr (NSR > 1) {
            const int k = (r * NSG) >> 5;
#pragma unroll
            for (int kk = 1; kk < NSR; ++kk) sreg = k == kk ? sca[kk] : sreg;
        }
        float racc[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) racc[b] = 0.f;
#pragma unroll 1
        for (int sg = 0; sg < NSG; ++sg) {
            __half2 gacc[NH];
#pragma unroll
            for (int h = 0; h < NH; ++h) gacc[h] = __float2half2_rn(0.f);
#pragma unroll
            for (int mm = 0; mm < GPL; ++mm) {
                const int m = sg * GPL + mm;
                uint32_t e;
                if constexpr (CONSTANT) {
                    e = cent;
                } else {
                    e = decode_step(x, a, b0, b1, tb);
                }
                // the sym field ORed into the mantissa of 64.0f is 64 + s/8
                const float wf = __uint_as_float((e & 0x3C000u) | 0x42800000u) - 65.0f;  // (s - 8) / 8, exact
                const __half2 w2 = __float2half2_rn(wf);
                __half2 xh[NH];
                lds_x<NB>(xcol + static_cast<uint32_t>(m) * (64u * NB), xh);
#pragma unroll
                for (int h = 0; h < NH; ++h) gacc[h] = __hfma2(w2, xh[h], gacc[h]);
            }
            const float gs = __shfl_sync(0xffffffffu, sreg, (r * NSG + sg) & 31);
#pragma unroll
            for (int h = 0; h < NH; ++h) {
                const float2 f = __half22float2(gacc[h]);
                racc[2 * h] = fmaf(gs, f.x, racc[2 * h]);
                racc[2 * h + 1] = fmaf(gs, f.y, racc[2 * h + 1]);
            }
        }
        const float v = transpose_reduce<NB>(racc, lane);
        if (reduce_owner<NB>(lane))
            p.partials[(static_cast<size_t>(t) * kTileRows + r) * NB + reduce_index<NB>(lane)] = v;
    }
    // rows past a short slab contribute zeros
    for (int r = rows_here; r < kTileRows; ++r)
        if (lane < NB) p.partials[(static_cast<size_t>(t) * kTileRows + r) * NB + lane] = 0.f;
    if constexpr (!CONSTANT) {
        if (x != kL || (a - buf - lane) != len * 32u) atomicOr(p.status, ECQ_STATUS_CORRUPT);
    } else {
        if (len != 4u) atomicOr(p.status, ECQ_STATUS_CORRUPT);
    }
    complete_pending_batch<NB>(p, pend, lane);
    // the owner lanes' partial stores are ordered before lane 0 counts the
    // tile (the warp that completes the slab reads them after its own
    // acquire-release increment)
    __threadfence();
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) old = atom_add_acq_rel(p.slab_count + slab, 1u);
    pend.slab = slab;
    pend.old = old;
    pend.rows = rows_here;
}

// Shared memory: [decode table 64 KB][x][2 stage buffers per warp][read-ahead pad][mbarriers]
template <int MPL, int GPL, int MODE, int NB = 1>
__global__ void __launch_bounds__(1024, 1) matrix_kernel(MatrixParams p) {
    constexpr bool GEMV = MODE == kModeGemv;
    constexpr bool BATCH = MODE == kModeGemvBatch;
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int W = blockDim.x >> 5;
    const uint32_t sbase = smem_addr(smem);  // the decode table's shared-window address
    const uint32_t bufs_off = kTableBytes + ((p.x_bytes + p.xs_bytes + 127u) & ~127u);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + bufs_off + 2 * W * p.buf_bytes + overrun_pad<MPL>());
    const uint32_t table_bar = smem_addr(bars + 2 * W);
    const bool constant = p.flags & ECQ_FLAG_CONSTANT;

    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2 * W + 1; ++i) mbar_init(smem_addr(bars + i), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        mbar_expect_tx(table_bar, kTableBytes + p.x_bytes);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            bulk_copy_g2s(sbase + i * (kTableBytes / 4), reinterpret_cast<const uint8_t*>(p.dec_table) + i * (kTableBytes / 4),
                          kTableBytes / 4, table_bar);
    }

    // contiguous run of tiles for this warp
    const uint64_t GW = static_cast<uint64_t>(gridDim.x) * W;
    const uint64_t gw = static_cast<uint64_t>(blockIdx.x) * W + warp;
    const uint32_t t_begin = static_cast<uint32_t>(gw * p.n_tiles / GW);
    const uint32_t t_end = static_cast<uint32_t>((gw + 1) * p.n_tiles / GW);
    const uint32_t my_bar0 = smem_addr(bars + 2 * warp);
    const uint32_t my_buf0 = bufs_off + 2 * warp * p.buf_bytes;  // offset in smem

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
        if (bytes) bulk_copy_g2s(sbase + my_buf0 + stage * p.buf_bytes, p.data + off, bytes, bar);
    };

    if (lane == 0 && t_begin < t_end) issue(t_begin, 0);
    // x, the outputs and the workspace may belong to the kernel before this
    // one in the stream: wait for it only now, with the table and the first
    // tile on their way
    pdl_wait();
    if (threadIdx.x == 0 && p.x_bytes) bulk_copy_g2s(sbase + kTableBytes, p.x, p.x_bytes, table_bar);
    if constexpr (BATCH) {
        // x of the NB tokens as fp16 x 8, [cols][NB], tokens past batch_here zero
        __half* xs = reinterpret_cast<__half*>(smem + kTableBytes);
        for (uint32_t c = threadIdx.x; c < p.cols; c += blockDim.x) {
            __half v[NB];
#pragma unroll
            for (int b = 0; b < NB; ++b)
                v[b] = b < static_cast<int>(p.batch_here)
                           ? __hmul(p.x[static_cast<size_t>(b) * p.cols + c], __float2half(8.f))
                           : __float2half(0.f);
#pragma unroll
            for (int b = 0; b < NB; ++b) xs[static_cast<size_t>(c) * NB + b] = v[b];
        }
        __syncthreads();
    }
    bool ok = mbar_wait(table_bar, 0);
    if (!ok && lane == 0) atomicOr(p.status, ECQ_STATUS_TIMEOUT);

    uint32_t phase0 = 0, phase1 = 0;
    PendingSlab pend{0xffffffffu, 0u, 0};
    // the run's tiles are consecutive: one division for the first tile's
    // (slab, k-tile), then a carry per tile
    uint32_t slab = t_begin / p.n_ktiles, kt = t_begin - slab * p.n_ktiles;
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
        uint32_t buf = sbase + my_buf0 + stage * p.buf_bytes;
        asm volatile("" : "+r"(buf)::"memory");  // keep this tile's byte loads after its wait
        if constexpr (BATCH) {
            if (constant)
                process_tile_batch<MPL, GPL, NB, true>(p, t, slab, kt, buf, sbase, sbase + kTableBytes, lane, pend);
            else
                process_tile_batch<MPL, GPL, NB, false>(p, t, slab, kt, buf, sbase, sbase + kTableBytes, lane, pend);
        } else {
            if (constant)
                process_tile<MPL, GPL, MODE, true>(p, t, slab, kt, buf, sbase, lane, pend);
            else
                process_tile<MPL, GPL, MODE, false>(p, t, slab, kt, buf, sbase, lane, pend);
        }
        if (++kt == p.n_ktiles) {
            kt = 0;
            ++slab;
        }
    }
    if constexpr (GEMV) complete_pending(p, pend, lane);
    if constexpr (BATCH) complete_pending_batch<NB>(p, pend, lane);
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

template <int MODE, int NB = 1>
KernelFn pick_kernel(int mpl, int gpl) {
#define ECQ_CASE(M_, G_) \
    if (mpl == M_ && gpl == G_) return matrix_kernel<M_, G_, MODE, NB>;
    ECQ_CASE(4, 1) ECQ_CASE(4, 2) ECQ_CASE(4, 4)
    ECQ_CASE(8, 1) ECQ_CASE(8, 2) ECQ_CASE(8, 4) ECQ_CASE(8, 8)
    ECQ_CASE(16, 1) ECQ_CASE(16, 2) ECQ_CASE(16, 4) ECQ_CASE(16, 8) ECQ_CASE(16, 16)
#undef ECQ_CASE
    return nullptr;
}

KernelFn pick_mode(int mode, int nb, int mpl, int gpl) {
    switch (mode) {
        case kModeSymbols: return pick_kernel<kModeSymbols>(mpl, gpl);
        case kModeGemv: return pick_kernel<kModeGemv>(mpl, gpl);
        case kModeWeights: return pick_kernel<kModeWeights>(mpl, gpl);
        case kModePacked4: return pick_kernel<kModePacked4>(mpl, gpl);
        case kModeGemvBatch:
            if (nb == 2) return pick_kernel<kModeGemvBatch, 2>(mpl, gpl);
            if (nb == 4) return pick_kernel<kModeGemvBatch, 4>(mpl, gpl);
            if (nb == 8) return pick_kernel<kModeGemvBatch, 8>(mpl, gpl);
            return nullptr;
    }
    return nullptr;
}

struct LaunchShape {
    int mpl, gpl, warps, ctas;
    uint32_t buf_bytes;
    size_t smem;
    uint32_t x_bytes;   // x bulk-copied into shared memory (GEMV)
    uint32_t xs_bytes;  // x of nb tokens staged as fp16 [cols][nb] (batched GEMV)
};

constexpr int kMinBatchWarps = 16;  // a batched launch keeps at least this many warps per CTA

// mode: what the kernel does (kMode*); nb: tokens per launch (batched GEMV)
int32_t shape_for(const ecq_matrix_view* m, int mode, int nb, LaunchShape* ls) {
    if (!m) return ECQ_ERR_ARG;
    const bool groups = mode == kModeGemv || mode == kModeWeights || mode == kModeGemvBatch;
    if (m->tile_rows != kTileRows) return ECQ_ERR_UNSUPPORTED;
    if (m->tile_cols % 32 || m->tile_cols == 0 || m->cols % m->tile_cols) return ECQ_ERR_SHAPE;
    const int mpl = static_cast<int>(m->tile_cols / 32);
    int gpl = mpl;
    if (groups) {
        const uint32_t g = m->group_size;
        if (g == 0 || g % 32) return ECQ_ERR_UNSUPPORTED;
        if (g < m->tile_cols) {
            if (m->tile_cols % g) return ECQ_ERR_UNSUPPORTED;
            gpl = static_cast<int>(g / 32);
        } else if (g % m->tile_cols) {
            return ECQ_ERR_UNSUPPORTED;
        }
    }
    if (!pick_mode(mode, nb, mpl, gpl)) return ECQ_ERR_UNSUPPORTED;
    const uint32_t slabs = (m->rows + kTileRows - 1) / kTileRows;
    if (m->n_tiles != slabs * (m->cols / m->tile_cols)) return ECQ_ERR_SHAPE;
    uint32_t buf = (m->max_tile_bytes + 127u) & ~127u;
    if (buf < 128) buf = 128;
    const int bar_bytes = 8 * (2 * 32 + 1);
    const int pad = static_cast<int>((32u * (5u + 3u * kTileRows * static_cast<uint32_t>(mpl)) + 127u) & ~127u);
    const int64_t room = kMaxSmem - kTableBytes - pad - bar_bytes;
    uint32_t xb = 0, xsb = 0;
    if (mode == kModeGemv) {
        // stage x in shared memory when it leaves room for at least 16 warps
        xb = m->cols * 2u;
        if (xb > room - 16 * 2 * static_cast<int64_t>(buf)) xb = 0;
    } else if (mode == kModeGemvBatch) {
        xsb = m->cols * 2u * static_cast<uint32_t>(nb);
        if (xsb > room - kMinBatchWarps * 2 * static_cast<int64_t>(buf)) return ECQ_ERR_UNSUPPORTED;
    }
    const int xpad = static_cast<int>((xb + xsb + 127u) & ~127u);
    int warps = static_cast<int>((room - xpad) / (2 * static_cast<int64_t>(buf)));
    if (warps > 32) warps = 32;
    if (warps < 1) return ECQ_ERR_UNSUPPORTED;
    ls->mpl = mpl;
    ls->gpl = gpl;
    ls->warps = warps;
    ls->ctas = sm_count_cached();
    ls->buf_bytes = buf;
    ls->smem = static_cast<size_t>(2 * warps) * buf + kTableBytes + xpad + pad + 8 * (2 * warps + 1);
    ls->x_bytes = xb;
    ls->xs_bytes = xsb;
    return ECQ_OK;
}

// tokens one batched-GEMV launch takes for this batch: the largest of 8, 4, 2
// (not above the batch rounded up to a power of two) whose staged x leaves
// room for kMinBatchWarps warps; 1 when batch is 1 or none fits (then each
// token runs the single-token GEMV)
int gemv_tokens(const ecq_matrix_view* m, uint32_t batch) {
    if (batch <= 1) return 1;
    int nb = batch >= 8 ? 8 : (batch > 2 ? (batch > 4 ? 8 : 4) : 2);
    for (; nb >= 2; nb >>= 1) {
        LaunchShape ls;
        if (shape_for(m, kModeGemvBatch, nb, &ls) == ECQ_OK) return nb;
    }
    return 1;
}

// GEMV workspace: [slab counters, n_slabs u32 (rounded up to 16 bytes)]
// [partials, n_tiles x 8 rows x nb fp32]. The counters come first so that
// their place does not depend on the tile count or the tokens per launch.
size_t ws_counter_bytes(const ecq_matrix_view* m) {
    const size_t slabs = (m->rows + kTileRows - 1) / kTileRows;
    return (slabs * 4 + 15) & ~static_cast<size_t>(15);
}
int64_t ws_bytes(const ecq_matrix_view* m, int nb) {
    return static_cast<int64_t>(ws_counter_bytes(m)) + static_cast<int64_t>(m->n_tiles) * kTileRows * 4 * nb;
}

struct LaunchArgs {
    const __half* x = nullptr;
    const __half* scales = nullptr;
    __half* y = nullptr;
    uint8_t* sym_out = nullptr;
    __half* w_out = nullptr;
    void* workspace = nullptr;
    const ecq_tp_comm* comm = nullptr;
    const ecq_gemv_epilogue* epi = nullptr;
    uint32_t batch_here = 1;
};

int32_t launch_matrix(const ecq_matrix_view* m, int mode, int nb, const LaunchArgs& la, uint32_t* status,
                      cudaStream_t stream) {
    LaunchShape ls;
    int32_t rc = shape_for(m, mode, nb, &ls);
    if (rc != ECQ_OK) return rc;
    MatrixParams p{};
    p.data = m->data;
    p.tile_offset = m->tile_offset;
    p.stream_len = m->stream_len;
    p.dec_table = m->dec_table;
    p.x = la.x;
    p.scales = la.scales;
    p.y = la.y;
    p.sym_out = la.sym_out;
    p.w_out = la.w_out;
    p.status = status;
    p.rows = m->rows;
    p.cols = m->cols;
    p.group_size = m->group_size ? m->group_size : 32;
    p.ng = (m->cols + p.group_size - 1) / p.group_size;
    p.n_ktiles = m->cols / m->tile_cols;
    p.n_tiles = m->n_tiles;
    p.buf_bytes = ls.buf_bytes;
    p.flags = m->flags;
    // x staged by bulk copy needs a 16-byte aligned address
    p.x_bytes = (mode == kModeGemv && (reinterpret_cast<uintptr_t>(la.x) & 15u) == 0) ? ls.x_bytes : 0u;
    p.xs_bytes = ls.xs_bytes;
    p.nb = static_cast<uint32_t>(nb);
    p.batch_here = la.batch_here;
    if (mode == kModeGemv || mode == kModeGemvBatch) {
        p.slab_count = static_cast<uint32_t*>(la.workspace);
        p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(la.workspace) + ws_counter_bytes(m));
    }
    if (la.epi) {
        p.epi_kind = static_cast<uint32_t>(la.epi->kind);
        p.epi_part_rows = la.epi->part_rows;
        p.epi_head_dim = la.epi->head_dim;
        p.epi_cache_stride = la.epi->cache_head_stride;
        p.epi_cos = static_cast<const __half*>(la.epi->cos_f16);
        p.epi_sin = static_cast<const __half*>(la.epi->sin_f16);
        p.epi_kc = static_cast<__half*>(la.epi->k_cache_f16);
        p.epi_vc = static_cast<__half*>(la.epi->v_cache_f16);
    }
    if (la.comm) {
        p.tp_world = la.comm->world;
        p.tp_rank = la.comm->rank;
        p.tp_nmax = la.comm->n_max;
        p.tp_epoch = static_cast<uint32_t*>(la.comm->local);
        for (uint32_t q = 0; q < la.comm->world; ++q) p.tp_peer[q] = static_cast<uint8_t*>(la.comm->peers[q]);
    }
    KernelFn fn = pick_mode(mode, nb, ls.mpl, ls.gpl);
    if (!ensure_smem_limit(reinterpret_cast<const void*>(fn), kMaxSmem)) return ECQ_ERR_CUDA;
    if (launch_pdl(fn, dim3(ls.ctas), dim3(ls.warps * 32), ls.smem, stream, p) != cudaSuccess) {
        cudaGetLastError();
        return ECQ_ERR_CUDA;
    }
    return ECQ_OK;
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
    LaunchArgs la;
    la.sym_out = d_out;
    return launch_matrix(m, kModeSymbols, 1, la, d_status, static_cast<cudaStream_t>(stream));
}

int32_t ecq_matrix_decode_packed4(const ecq_matrix_view* m, uint8_t* d_out, uint32_t* d_status, void* stream) {
    if (!view_ok(m) || !d_out || !d_status) return ECQ_ERR_ARG;
    LaunchArgs la;
    la.sym_out = d_out;
    return launch_matrix(m, kModePacked4, 1, la, d_status, static_cast<cudaStream_t>(stream));
}

int32_t ecq_matrix_dequantize(const ecq_matrix_view* m, const void* scales_f16, void* w_out_f16, uint32_t* d_status,
                              void* stream) {
    if (!view_ok(m) || !scales_f16 || !w_out_f16 || !d_status) return ECQ_ERR_ARG;
    if (m->group_size == 0 || m->group_size % 32 || (m->group_size < m->tile_cols && m->tile_cols % m->group_size) ||
        (m->group_size >= m->tile_cols && m->group_size % m->tile_cols))
        return ECQ_ERR_UNSUPPORTED;
    LaunchArgs la;
    la.scales = static_cast<const __half*>(scales_f16);
    la.w_out = static_cast<__half*>(w_out_f16);
    return launch_matrix(m, kModeWeights, 1, la, d_status, static_cast<cudaStream_t>(stream));
}

int64_t ecq_gemv_workspace_bytes(const ecq_matrix_view* m, uint32_t batch) {
    if (!m || !m->rows || !m->n_tiles) return ECQ_ERR_ARG;
    return ws_bytes(m, gemv_tokens(m, batch));
}

int32_t ecq_gemv(const ecq_matrix_view* m, const void* x_f16, const void* scales_f16, void* y_f16, uint32_t batch,
                 void* workspace, int64_t workspace_bytes, uint32_t* d_status, void* stream) {
    if (!view_ok(m) || !x_f16 || !scales_f16 || !y_f16 || !d_status || batch == 0) return ECQ_ERR_ARG;
    if (!workspace || workspace_bytes < ws_bytes(m, 1)) return ECQ_ERR_WORKSPACE;
    const __half* x = static_cast<const __half*>(x_f16);
    __half* y = static_cast<__half*>(y_f16);
    LaunchArgs la;
    la.scales = static_cast<const __half*>(scales_f16);
    la.workspace = workspace;
    // token batches: up to nb tokens per launch share one decode of every
    // tile; a workspace sized for fewer tokens runs the single-token GEMV
    int nb = gemv_tokens(m, batch);
    while (nb > 1 && workspace_bytes < ws_bytes(m, nb)) nb >>= 1;
    for (uint32_t b = 0; b < batch;) {
        const uint32_t here = nb > 1 ? std::min<uint32_t>(static_cast<uint32_t>(nb), batch - b) : 1u;
        la.x = x + static_cast<size_t>(b) * m->cols;
        la.y = y + static_cast<size_t>(b) * m->rows;
        la.batch_here = here;
        // a last chunk of one token takes the exact single-token kernel
        const int mode = here > 1 ? kModeGemvBatch : kModeGemv;
        int32_t rc = launch_matrix(m, mode, here > 1 ? nb : 1, la, d_status, static_cast<cudaStream_t>(stream));
        if (rc != ECQ_OK) return rc;
        b += here;
    }
    return ECQ_OK;
}

int32_t ecq_gemv_fused(const ecq_matrix_view* m, const void* x_f16, const void* scales_f16, void* y_f16,
                       const ecq_gemv_epilogue* epi, void* workspace, int64_t workspace_bytes, uint32_t* d_status,
                       void* stream) {
    if (!view_ok(m) || !x_f16 || !scales_f16 || !y_f16 || !epi || !d_status) return ECQ_ERR_ARG;
    if (epi->kind == ECQ_EPI_ROPE_KV) {
        if (epi->head_dim < 2 || (epi->head_dim & 1) || epi->part_rows == 0 || epi->part_rows % 8 ||
            epi->part_rows % epi->head_dim || m->rows != 3 * epi->part_rows || !epi->cos_f16 || !epi->sin_f16 ||
            !epi->k_cache_f16 || !epi->v_cache_f16 || epi->cache_head_stride < static_cast<int64_t>(epi->head_dim))
            return ECQ_ERR_ARG;
    } else if (epi->kind == ECQ_EPI_SILU_MUL) {
        if (m->rows & 1) return ECQ_ERR_ARG;
    } else {
        return ECQ_ERR_ARG;
    }
    if (!workspace || workspace_bytes < ws_bytes(m, 1)) return ECQ_ERR_WORKSPACE;
    LaunchArgs la;
    la.x = static_cast<const __half*>(x_f16);
    la.scales = static_cast<const __half*>(scales_f16);
    la.y = static_cast<__half*>(y_f16);
    la.workspace = workspace;
    la.epi = epi;
    return launch_matrix(m, kModeGemv, 1, la, d_status, static_cast<cudaStream_t>(stream));
}

int32_t ecq_gemv_tp(const ecq_matrix_view* m, const void* x_f16, const void* scales_f16, const ecq_tp_comm* comm,
                    void* workspace, int64_t workspace_bytes, uint32_t* d_status, void* stream) {
    if (!view_ok(m) || !x_f16 || !scales_f16 || !comm || !d_status) return ECQ_ERR_ARG;
    if (comm->world < 1 || comm->world > ECQ_TP_MAX_RANKS || comm->rank >= comm->world || !comm->local ||
        m->rows > comm->n_max)
        return ECQ_ERR_ARG;
    for (uint32_t q = 0; q < comm->world; ++q)
        if (!comm->peers[q]) return ECQ_ERR_ARG;
    if (!workspace || workspace_bytes < ws_bytes(m, 1)) return ECQ_ERR_WORKSPACE;
    LaunchArgs la;
    la.x = static_cast<const __half*>(x_f16);
    la.scales = static_cast<const __half*>(scales_f16);
    la.workspace = workspace;
    la.comm = comm;
    return launch_matrix(m, kModeGemv, 1, la, d_status, static_cast<cudaStream_t>(stream));
}

int32_t ecq_device_info(int32_t* sm_count, int32_t* gemv_ctas, int32_t* gemv_warps_per_cta,
                        const ecq_matrix_view* m) {
    if (sm_count) *sm_count = sm_count_cached();
    if (m) {
        LaunchShape ls;
        int32_t rc = shape_for(m, kModeGemv, 1, &ls);
        if (rc != ECQ_OK) return rc;
        if (gemv_ctas) *gemv_ctas = ls.ctas;
        if (gemv_warps_per_cta) *gemv_warps_per_cta = ls.warps;
    }
    return ECQ_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Fused GEMV on library-owned scratch: for callers that cannot allocate.
//
// ecq_gemv needs a few bytes of device workspace per tile. Most callers pass
// a buffer they allocated once. Some cannot: a plugin whose host framework
// owns the whole device-memory budget and gives its plugins none, a C host
// with no device allocator of its own, or a latency-critical serving loop
// that must never call cudaMalloc (it can synchronise the device and stall
// every other stream). ecq_gemv_noalloc serves them from a fixed array that
// lives in this library's device image instead.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds ECQ_NOALLOC_SCRATCH_BYTES of it until the process exits.
// From host code its name is only a host-side stand-in, never a device
// address, so the device address is looked up with cudaGetSymbolAddress once
// per device (with that device current) and cached together with the id of
// the CUDA context it was found in: after cudaDeviceReset the module is
// loaded again into a new context, possibly elsewhere, and the address is
// looked up again. All calls share the one array, so two calls whose kernels
// overlap on the GPU (different streams, or different host threads) race on
// it and must be ordered by the caller.
// ---------------------------------------------------------------------------
struct CUctx_st;  // the driver's opaque context type (CUcontext)

static __device__ __align__(256) uint8_t g_noalloc_scratch[ECQ_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;

// Unique id (cuCtxGetId) of the CUDA context current on this thread, 0 when
// there is none yet or the driver does not offer the query. The driver entry
// points are fetched through the runtime, so libecq needs no libcuda link.
unsigned long long current_context_id() {
    using CtxCurrentFn = int (*)(CUctx_st**);
    using CtxIdFn = int (*)(CUctx_st*, unsigned long long*);
    static CtxCurrentFn ctx_current = nullptr;
    static CtxIdFn ctx_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            ctx_current = reinterpret_cast<CtxCurrentFn>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            ctx_id = reinterpret_cast<CtxIdFn>(f);
    });
    if (!ctx_current || !ctx_id) return 0;
    CUctx_st* c = nullptr;
    if (ctx_current(&c) != 0 || !c) return 0;
    unsigned long long id = 0;
    return ctx_id(c, &id) == 0 ? id : 0;
}

// Device address of g_noalloc_scratch on the current device: looked up on
// the first call for that device (with that device current) and again
// whenever the current context is not the one the cached address came from.
int32_t noalloc_scratch(void** out) {
    struct Entry {
        void* addr;
        unsigned long long ctx;
    };
    static std::mutex mu;
    static Entry cache[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ECQ_ERR_CUDA;
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(mu);
    Entry& e = cache[dev];
    if (!e.addr || ctx == 0 || e.ctx != ctx) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return ECQ_ERR_CUDA;
        e.addr = p;
        e.ctx = ctx ? ctx : current_context_id();  // the lookup made the context current
    }
    *out = e.addr;
    return ECQ_OK;
}

}  // namespace

extern "C" int32_t ecq_gemv_noalloc(const ecq_matrix_view* m, const void* x_f16, const void* scales_f16, void* y_f16,
                                    uint32_t batch, uint32_t* d_status, void* stream) {
    if (!view_ok(m) || !x_f16 || !scales_f16 || !y_f16 || !d_status || batch == 0) return ECQ_ERR_ARG;
    const int64_t need = ecq_gemv_workspace_bytes(m, batch);
    if (need < 0) return static_cast<int32_t>(need);
    if (need > static_cast<int64_t>(ECQ_NOALLOC_SCRATCH_BYTES)) return ECQ_ERR_WORKSPACE;
    void* scratch = nullptr;
    const int32_t rc = noalloc_scratch(&scratch);
    if (rc != ECQ_OK) return rc;
    // The per-slab completion counters sit at the start of the workspace. A
    // finished call leaves them zero, but the array keeps whatever the last
    // call left, including one that failed: clear them on every call (the
    // partial sums after them need no clearing: each is written before it is
    // read).
    if (cudaMemsetAsync(scratch, 0, ws_counter_bytes(m), static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return ECQ_ERR_CUDA;
    return ecq_gemv(m, x_f16, scales_f16, y_f16, batch, scratch, need, d_status, stream);
}
