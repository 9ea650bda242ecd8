/*
 * ecq.h -- C ABI of libecq, the B200 (sm_100a) implementation of ecq's hot
 * path: interleaved rANS decode of 4-bit weight symbols fused with per-group
 * dequantisation and the GEMV that consumes them.
 *
 * Conventions
 *   - Every function returns int32_t status (ECQ_OK == 0, negative on error)
 *     unless it returns a size (int64_t, negative on error).
 *   - Device pointers are owned by the caller; the library never frees caller
 *     memory and launches allocate nothing. Every launch takes a cudaStream_t
 *     (passed as void*, NULL = legacy default stream) and never synchronises
 *     the host.
 *   - Device-side failures are reported through a caller-provided uint32_t
 *     status word in device memory (bits ECQ_STATUS_*), OR-ed in by kernels.
 *   - Thread-safe: there is no global mutable state except the lazily read
 *     device properties.
 *
 * Codec parameters are the reference's (drxddy/ecq src/rans.py:21-23): 16
 * symbols, 14-bit probabilities, 32-bit state, L = 2^23, byte renormalisation.
 * Stream format: src/interleaved_rans.py:76-153 (byte p of stream j at
 * data[j + p*S], streams zero-padded to the longest).
 */
#ifndef ECQ_H
#define ECQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ECQ_VERSION 100
#define ECQ_NSYM 16
#define ECQ_PROB_BITS 14
#define ECQ_RANS_L (1u << 23)
#define ECQ_LANES 32                  /* streams per tile in the packed format */
#define ECQ_MAX_SYMS_PER_STREAM 1024  /* tile_rows*tile_cols/32 upper bound */
#define ECQ_TABLE_ENTRIES 16384

/* status codes */
#define ECQ_OK 0
#define ECQ_ERR_ARG (-1)
#define ECQ_ERR_SHAPE (-2)
#define ECQ_ERR_TABLE (-3)
#define ECQ_ERR_ZERO_FREQ (-4)   /* a present symbol has frequency 0 */
#define ECQ_ERR_CAPACITY (-5)
#define ECQ_ERR_CUDA (-6)
#define ECQ_ERR_INTERNAL (-7)
#define ECQ_ERR_UNSUPPORTED (-8)
#define ECQ_ERR_WORKSPACE (-9)

/* device status word bits */
#define ECQ_STATUS_CORRUPT 1u   /* a stream did not end in (state 2^23, all bytes read) */
#define ECQ_STATUS_TIMEOUT 2u   /* a bounded wait on an mbarrier gave up */
#define ECQ_STATUS_BADARG 4u

/* normaliser used by ecq_table_from_counts */
#define ECQ_NORMALISER_REFERENCE 0
#define ECQ_NORMALISER_CLAMPED 1

/* ecq_build_decode_table flags */
#define ECQ_FLAG_CONSTANT 1u            /* one symbol has frequency 16384 */
#define ECQ_FLAG_CONSTANT_SYM_SHIFT 4   /* its index, in bits 4..7 */

/*
 * Packed matrix: an [rows, cols] matrix of 4-bit symbols cut into tiles of
 * tile_rows x tile_cols (cols % tile_cols == 0, tile_cols % 32 == 0; the last
 * row slab may be short). Tiles are ordered row-slab major, then along K.
 * Tile t's row-major symbols are ONE reference interleaved tile with 32
 * streams, stored verbatim at data + tile_offset[t] (32*max_len bytes,
 * always a multiple of 32); stream_len[32*t + j] is stream j's byte length.
 * dec_table is the 16384-entry packed decode table from
 * ecq_build_decode_table for the matrix's frequency table.
 *
 * Precondition on tile_offset (the view carries no data length, so the
 * kernels cannot check it): tile_offset[0] == 0, the offsets never decrease,
 * every tile's size is a multiple of 32 bytes and at most max_tile_bytes, and
 * tile_offset[n_tiles] does not exceed the data allocation. Check offsets
 * read from an untrusted file on the host before building a view: a tile
 * larger than max_tile_bytes is refused on the device (ECQ_STATUS_BADARG),
 * but offsets past the end of the data make the bulk copies read outside it.
 */
typedef struct ecq_matrix_view {
    uint32_t rows, cols;
    uint32_t tile_rows, tile_cols;
    uint32_t group_size;       /* scales are [rows, ceil(cols/group_size)] */
    uint32_t n_tiles;          /* ceil(rows/tile_rows) * cols/tile_cols */
    uint32_t max_tile_bytes;   /* max over tiles of 32*max_len */
    uint32_t flags;            /* from ecq_build_decode_table */
    const uint8_t *data;       /* device */
    const uint32_t *tile_offset; /* device, n_tiles + 1 entries */
    const uint16_t *stream_len;  /* device, 32 * n_tiles entries */
    const uint32_t *dec_table;   /* device, 16384 entries */
} ecq_matrix_view;

int32_t ecq_version(void);

/* ---------------- host-side codec ---------------- */

/* Frequency table from a 16-bin histogram. Replaces RANSTable.from_counts
 * (src/rans.py:39-60) and gives the same table, except where that normaliser
 * gives frequency 0 to a symbol that occurs (its encoder never terminates on
 * such input): then every frequency is raised to at least 1 before the
 * remainder goes to the largest, and *normaliser = ECQ_NORMALISER_CLAMPED. */
int32_t ecq_table_from_counts(const uint64_t *counts, uint32_t *freq, int32_t *normaliser);

/* 16384 packed decode entries, entry[slot] = (slot - cumfreq[s])
 * | s << 14 | freq[s] << 18 with s = sym_table[slot], for a
 * frequency table summing to 16384. Replaces the sym_table/freq/cumfreq
 * triple the reference's kernels read (src/rans.py:51-58,
 * src/metal_interleaved.py:52-117). */
int32_t ecq_build_decode_table(const uint32_t *freq, uint32_t *entries, uint32_t *flags);

/* Interleaved encoder, byte-identical to interleaved_rans_encode
 * (src/interleaved_rans.py:76-153). Writes n_streams*max_len bytes into
 * data; returns that byte count or a negative error. */
int64_t ecq_encode_interleaved_host(const uint8_t *symbols, int64_t n, int32_t n_streams,
                                    const uint32_t *freq, uint8_t *data, int64_t data_cap,
                                    uint32_t *stream_lengths, uint32_t *max_len);

/* Worst-case byte size of ecq_encode_matrix_host's data output. */
int64_t ecq_matrix_encoded_bound(uint32_t rows, uint32_t cols, uint32_t tile_rows, uint32_t tile_cols);

/* Encode a row-major [rows, cols] symbol matrix into the packed format over
 * n_threads host threads (<= 0: all). Each tile is one call of the
 * reference's interleaved_rans_encode with 32 streams
 * (src/interleaved_rans.py:76-153); replaces the per-layer encode loop of
 * experiments/e2e_validation.py:49-105. tile_offset gets n_tiles+1 entries. */
int32_t ecq_encode_matrix_host(const uint8_t *symbols, uint32_t rows, uint32_t cols, uint32_t tile_rows,
                               uint32_t tile_cols, const uint32_t *freq, int32_t n_threads, uint8_t *data,
                               int64_t data_cap, uint32_t *tile_offset, uint16_t *stream_len,
                               int64_t *total_bytes);

/* ---------------- device: decode ---------------- */

/* Decode one reference tile (any n_streams >= 1, any n_symbols) on the GPU:
 * d_data holds the tile's interleaved bytes (n_streams*max_len), d_lengths
 * its stream lengths, d_dec_table the packed table. Output d_out[n_symbols].
 * Replaces interleaved_rans_decode (src/interleaved_rans.py:156-217) and
 * MetalInterleavedRANS.decode (src/metal_interleaved.py:833-885, kernel
 * parallel_rans_decode :52-117). Semantics are the reference's, guards
 * included: streams shorter than 4 bytes decode to zeros and
 * renormalisation stops at the stream length, so damaged tiles decode to
 * the same bytes the reference returns. Streams that do not end in
 * (state 2^23, all bytes read) set ECQ_STATUS_CORRUPT in *d_status. */
int32_t ecq_decode_interleaved(const uint8_t *d_data, const uint32_t *d_lengths, uint32_t n_streams,
                               uint64_t n_symbols, uint32_t max_len, const uint32_t *d_dec_table,
                               uint32_t decode_flags, uint8_t *d_out, uint32_t *d_status, void *stream);

/* Decode a packed matrix to row-major uint8 symbols d_out[rows*cols] (the
 * CACHED strategy: DecodeOnceStrategy.load_layer,
 * src/decode_strategies.py:43-73, and the GPU_ASYNC decode kernel
 * parallel_rans_decode_async, src/decode_strategies.py:336-390). */
int32_t ecq_matrix_decode(const ecq_matrix_view *m, uint8_t *d_out, uint32_t *d_status, void *stream);

/* Decode a packed matrix to plain packed 4-bit, d_out[rows, cols/2] bytes
 * (column 2i in the low nibble of byte i of its row, column 2i+1 in the
 * high nibble): the CACHED strategy's 4-bit store (DecodeOnceStrategy,
 * src/decode_strategies.py:43-73, "store as 4-bit"), consumed by
 * ecq_plain4_gemv. Symbols are those ecq_matrix_decode returns. */
int32_t ecq_matrix_decode_packed4(const ecq_matrix_view *m, uint8_t *d_out, uint32_t *d_status, void *stream);

/* Decode a packed matrix straight to dequantised fp16 weights
 * w_out[r, c] = (sym[r,c] - 8) * scales[r, c/g] (row-major [rows, cols]):
 * the batched-token path, which decodes once and hands W to a tensor-core
 * GEMM. Replaces the reference's CACHED dequantisation
 * (src/decode_strategies.py:43-73 then src/quantizer.py:33-35). */
int32_t ecq_matrix_dequantize(const ecq_matrix_view *m, const void *scales_f16, void *w_out_f16, uint32_t *d_status,
                              void *stream);

/* ---------------- device: fused decode + dequant + GEMV ---------------- */

/* Bytes of device workspace ecq_gemv needs for this matrix and batch:
 * ceil(ceil(rows/8) * 4 / 16) * 16 bytes of slab counters, then
 * n_tiles * 32 * nb bytes of partial sums, nb being the tokens one launch
 * takes (1 for batch 1; 8, 4 or 2 for token batches, as many as x of that
 * many tokens fits in shared memory). The workspace must be zero-filled once
 * before first use; ecq_gemv leaves the counters zero again on completion,
 * so it can be reused across calls on one stream (calls that overlap on the
 * GPU must use distinct workspaces). A workspace sized for batch 1 also
 * serves larger batches, token by token. */
int64_t ecq_gemv_workspace_bytes(const ecq_matrix_view *m, uint32_t batch);

/* y[b, r] = sum_c (sym[r,c] - 8) * scales[r, c/g] * x[b, c], fp32
 * accumulation, fp16 output, for b < batch. x is [batch, cols] fp16,
 * scales [rows, ceil(cols/g)] fp16, y [batch, rows] fp16 (all device,
 * row-major, contiguous). The dequantisation is the reference's
 * sym*scale + zero with zero = -8*scale (src/quantizer.py:33-35). Replaces
 * the fused kernels fused_parallel_gemv / fused_parallel_gemv_cached /
 * tiled_parallel_gemm (src/metal_interleaved.py:130-484) and the MLX-side
 * entropy_coded_matmul (docs/mlx_integration_plan.md:222-237). No decoded
 * weight is written to memory. For batch > 1 each launch decodes every tile
 * once for up to 8 tokens (x staged in shared memory as fp16 x 8, so
 * |x| < 8188; products summed in fp16 over the 1-16 symbols a lane holds of
 * one scale group, then in fp32); batch 1 is all fp32. */
int32_t ecq_gemv(const ecq_matrix_view *m, const void *x_f16, const void *scales_f16, void *y_f16,
                 uint32_t batch, void *workspace, int64_t workspace_bytes, uint32_t *d_status, void *stream);

/* Fused epilogues of a batch-1 GEMV (ecq_gemv_fused): the element-wise step
 * that follows a projection in a transformer decode step, applied as each
 * row of y is finished, so that it needs no kernel of its own. */
#define ECQ_EPI_ROPE_KV 1   /* y = q | k | v: rotary embedding of q and k, k and v into the KV cache */
#define ECQ_EPI_SILU_MUL 2  /* rows interleave gate and up: y[j] = silu(gate j) * up j */

typedef struct ecq_gemv_epilogue {
    int32_t kind;               /* ECQ_EPI_* */
    uint32_t part_rows;         /* ROPE_KV: rows of each of q, k, v (heads * head_dim, a multiple of 8) */
    uint32_t head_dim;          /* ROPE_KV: even */
    uint32_t reserved;
    int64_t cache_head_stride;  /* ROPE_KV: elements between heads in the cache slot */
    const void *cos_f16;        /* ROPE_KV: [head_dim / 2] for the new token's position */
    const void *sin_f16;
    void *k_cache_f16;          /* ROPE_KV: the new token's slot, head h at h * cache_head_stride */
    void *v_cache_f16;
} ecq_gemv_epilogue;

/* ecq_gemv at batch 1 with a fused epilogue. ROPE_KV (m->rows = 3 *
 * part_rows): y holds q | k | v with q and k rotated pair by pair -- (2i,
 * 2i+1) by angle index i within each head -- and the rotated k and v are
 * also stored into the cache slot (the arithmetic of ecq_rope_kv_f16 on the
 * fp16-rounded GEMV outputs). SILU_MUL (m->rows even, rows interleaving gate
 * and up): y [rows / 2] = silu(gate) * up (the arithmetic of
 * ecq_silu_mul_f16). Replaces a GEMV followed by ecq_rope_kv_f16 or
 * ecq_silu_mul_f16 (the glue of the reference's MLX fork; model structure
 * experiments/real_model_test.py:18-113). Workspace as ecq_gemv for batch 1. */
int32_t ecq_gemv_fused(const ecq_matrix_view *m, const void *x_f16, const void *scales_f16, void *y_f16,
                       const ecq_gemv_epilogue *epi, void *workspace, int64_t workspace_bytes, uint32_t *d_status,
                       void *stream);

/* Size of the scratch array ecq_gemv_noalloc uses (4 MiB per GPU). */
#define ECQ_NOALLOC_SCRATCH_BYTES (4u << 20)

/* ecq_gemv without a caller workspace, for callers that cannot allocate
 * device memory: a plugin whose host framework owns the whole device-memory
 * budget, a C host with no device allocator, or a serving loop that must not
 * call cudaMalloc because it can synchronise the device. This entry point
 * has no counterpart in the reference; the reference's Python/Metal path
 * allocates its buffers on every call.
 *
 * The workspace comes from a fixed array inside the library
 * (ECQ_NOALLOC_SCRATCH_BYTES, held by every GPU that loads the library until
 * exit). A call fits when ecq_gemv_workspace_bytes(m, batch) <=
 * ECQ_NOALLOC_SCRATCH_BYTES: for one token n_tiles * 32 plus the slab
 * counters (~116.5K tiles with one K-tile per row slab to ~130K with 16,
 * e.g. 28672 x 8192 in 8x512 tiles), and nb times the partial sums for token
 * batches; larger calls are rejected with ECQ_ERR_WORKSPACE before anything
 * is launched. Nothing is allocated, by
 * the library or anyone else. The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress, with that device current);
 * make that first call before any stream capture. The address is looked up
 * again when the current CUDA context changes (e.g. after cudaDeviceReset),
 * and every call clears the slab counters at the start of the array with a
 * cudaMemsetAsync on the caller's stream. Every call shares the array: calls whose
 * kernels may overlap on the GPU (other streams, other host threads) race
 * and must be serialised by the caller. Arguments and results are those of
 * ecq_gemv. */
int32_t ecq_gemv_noalloc(const ecq_matrix_view *m, const void *x_f16, const void *scales_f16, void *y_f16,
                         uint32_t batch, uint32_t *d_status, void *stream);

/* ---------------- device: plain 4-bit GEMV ---------------- */

/* y[b, r] = sum_c (q[r, c] - 8) * scales[r, c/g] * x[b, c] for plain packed
 * 4-bit weights q [rows, cols/2] bytes (layout of ecq_matrix_decode_packed4),
 * fp16 scales [rows, cols/g], x [batch, cols] fp16, y [batch, rows] fp16:
 * fp16 products summed 8 at a time, then fp32 with the group scale;
 * deterministic. Up to 4 tokens share one pass over the weights. Needs
 * cols % 32 == 0, group_size a power of two >= 32, q and x 16-byte aligned.
 * Two roles: the CACHED strategy's GEMV after ecq_matrix_decode_packed4
 * (src/decode_strategies.py:43-73 decodes once, then multiplies), and an
 * HBM-bound control beside the fused rANS GEMV on the same shapes (the
 * reference's nibble-LUT kernel fused_memory_bench,
 * src/metal_interleaved.py:555-683, plays that role on Apple GPUs). */
int32_t ecq_plain4_gemv(const void *q_packed, const void *scales_f16, const void *x_f16, void *y_f16, uint32_t rows,
                        uint32_t cols, uint32_t group_size, uint32_t batch, void *stream);

/* ---------------- device: fused decode + dequant + tensor-core GEMM ---------------- */

/* Bytes of device workspace ecq_matmul needs for this matrix and batch, or a
 * negative error code when the matrix's layout has no tensor-core kernel
 * (tile widths 128 and 256 do; 512 does not). Zero-fill it once before first
 * use; ecq_matmul leaves it zeroed again on completion. */
int64_t ecq_matmul_workspace_bytes(const ecq_matrix_view *m, uint32_t batch);

/* y = x . W^T for a token batch: y[b, r] = sum_c (sym[r,c] - 8) * scales[r, c/g]
 * * x[b, c] with W rounded once to fp16 and fp32 accumulation on the tcgen05
 * tensor cores, b < batch (any batch; 128 tokens per launch). Layouts as for
 * ecq_gemv; x must be 16-byte aligned. Each tile is decoded straight into
 * the tensor core's shared-memory operand: no decoded weight is written to
 * memory. Replaces the reference's batched kernel tiled_parallel_gemm
 * (src/metal_interleaved.py:375-484) and the MLX-side entropy_coded_matmul
 * for x with several rows (docs/mlx_integration_plan.md:222-237). Returns
 * ECQ_ERR_UNSUPPORTED for layouts ecq_matmul_workspace_bytes rejects. */
int32_t ecq_matmul(const ecq_matrix_view *m, const void *x_f16, const void *scales_f16, void *y_f16,
                   uint32_t batch, void *workspace, int64_t workspace_bytes, uint32_t *d_status, void *stream);

/* Number of SMs and the persistent grid the fused kernel uses (for tests
 * and the benchmark's launch accounting). */
int32_t ecq_device_info(int32_t *sm_count, int32_t *gemv_ctas, int32_t *gemv_warps_per_cta,
                        const ecq_matrix_view *m);

#ifdef __cplusplus
}
#endif

#endif /* ECQ_H */
