// ecq_host.cpp -- host side of libecq: frequency tables, the packed decode
// table, the interleaved rANS encoder and the tile packer.
//
// The encoder produces exactly the bytes of the reference encoder
// (drxddy/ecq src/interleaved_rans.py:76-153): stream j of a tile holds the
// tile's flat symbols j, j+S, j+2S, ..., each stream is encoded in reverse
// with 32-bit state, 14-bit probabilities, L = 2^23 and byte-wise
// renormalisation, flushed as 4 big-endian bytes, and the streams are
// byte-interleaved (byte p of stream j at j + p*S), zero-padded to the
// longest stream. It is the offline half of the path (the reference runs it
// in Python at ~2 M symbols/s); here it runs in C++ over all host threads.
#include "ecq.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace {

constexpr uint32_t kProbBits = ECQ_PROB_BITS;
constexpr uint32_t kProbScale = 1u << kProbBits;
constexpr uint64_t kRansL = ECQ_RANS_L;

// Encode the symbols sym[j], sym[j+S], ... of one stream. Returns the byte
// count written to out (forward order) or -1 if a symbol has frequency 0.
int64_t encode_one_stream(const uint8_t* sym, int64_t n, int S, int j, const uint32_t* freq,
                          const uint32_t* cum, std::vector<uint8_t>& scratch, uint8_t* out,
                          int64_t cap) {
    int64_t cnt = (j < n) ? (n - j + S - 1) / S : 0;
    if (cnt == 0) return 0;
    scratch.resize(static_cast<size_t>(2 * cnt + 8));
    uint8_t* rev = scratch.data();
    int64_t nb = 0;
    uint64_t x = kRansL;
    for (int64_t k = cnt - 1; k >= 0; --k) {
        const uint32_t s = sym[j + k * S];
        const uint64_t f = freq[s];
        if (f == 0) return -1;
        const uint64_t x_max = ((kRansL >> kProbBits) << 8) * f;
        while (x >= x_max) {
            rev[nb++] = static_cast<uint8_t>(x);
            x >>= 8;
        }
        x = ((x / f) << kProbBits) + (x % f) + cum[s];
    }
    rev[nb++] = static_cast<uint8_t>(x);
    rev[nb++] = static_cast<uint8_t>(x >> 8);
    rev[nb++] = static_cast<uint8_t>(x >> 16);
    rev[nb++] = static_cast<uint8_t>(x >> 24);
    if (nb > cap) return -2;
    for (int64_t i = 0; i < nb; ++i) out[i] = rev[nb - 1 - i];
    return nb;
}

void cumulative(const uint32_t* freq, uint32_t* cum) {
    cum[0] = 0;
    for (int i = 0; i < ECQ_NSYM; ++i) cum[i + 1] = cum[i] + freq[i];
}

// Encode one tile (n symbols, S streams) into dst in the interleaved layout.
// stream_bytes must hold S * (2*ceil(n/S)+4) bytes of scratch.
int64_t encode_tile(const uint8_t* sym, int64_t n, int S, const uint32_t* freq, const uint32_t* cum,
                    uint8_t* dst, int64_t dst_cap, uint32_t* lengths, uint32_t* max_len_out,
                    std::vector<uint8_t>& scratch, std::vector<uint8_t>& streams) {
    const int64_t per = (n + S - 1) / S;
    const int64_t cap = 2 * per + 8;
    streams.resize(static_cast<size_t>(cap * S));
    int64_t max_len = 0;
    for (int j = 0; j < S; ++j) {
        int64_t len = encode_one_stream(sym, n, S, j, freq, cum, scratch, streams.data() + j * cap, cap);
        if (len < 0) return len == -1 ? ECQ_ERR_ZERO_FREQ : ECQ_ERR_INTERNAL;
        lengths[j] = static_cast<uint32_t>(len);
        max_len = std::max(max_len, len);
    }
    if (max_len * S > dst_cap) return ECQ_ERR_CAPACITY;
    std::memset(dst, 0, static_cast<size_t>(max_len * S));
    for (int j = 0; j < S; ++j) {
        const uint8_t* src = streams.data() + j * cap;
        for (uint32_t p = 0; p < lengths[j]; ++p) dst[j + static_cast<int64_t>(p) * S] = src[p];
    }
    *max_len_out = static_cast<uint32_t>(max_len);
    return max_len * S;
}

}  // namespace

extern "C" {

int32_t ecq_version(void) { return ECQ_VERSION; }

int32_t ecq_table_from_counts(const uint64_t* counts, uint32_t* freq, int32_t* normaliser) {
    if (!counts || !freq) return ECQ_ERR_ARG;
    // Reference normaliser (src/rans.py:39-60): float64 scale, truncate,
    // remainder on the first largest entry.
    double c[ECQ_NSYM], sum = 0.0;
    for (int i = 0; i < ECQ_NSYM; ++i) {
        c[i] = static_cast<double>(counts[i] > 0 ? counts[i] : 1);
        sum += c[i];
    }
    int64_t fsum = 0;
    bool hazard = false;
    for (int i = 0; i < ECQ_NSYM; ++i) {
        freq[i] = static_cast<uint32_t>(c[i] / sum * static_cast<double>(kProbScale));
        fsum += freq[i];
        if (counts[i] > 0 && freq[i] == 0) hazard = true;
    }
    if (hazard) {
        // A present symbol got frequency 0, on which the reference encoder
        // never terminates: raise every frequency to at least 1 first.
        fsum = 0;
        for (int i = 0; i < ECQ_NSYM; ++i) {
            if (freq[i] == 0) freq[i] = 1;
            fsum += freq[i];
        }
    }
    int am = 0;
    for (int i = 1; i < ECQ_NSYM; ++i)
        if (freq[i] > freq[am]) am = i;
    freq[am] = static_cast<uint32_t>(static_cast<int64_t>(freq[am]) + (static_cast<int64_t>(kProbScale) - fsum));
    if (normaliser) *normaliser = hazard ? ECQ_NORMALISER_CLAMPED : ECQ_NORMALISER_REFERENCE;
    return ECQ_OK;
}

int32_t ecq_build_decode_table(const uint32_t* freq, uint32_t* entries, uint32_t* flags) {
    if (!freq || !entries) return ECQ_ERR_ARG;
    uint64_t total = 0;
    for (int i = 0; i < ECQ_NSYM; ++i) total += freq[i];
    if (total != kProbScale) return ECQ_ERR_TABLE;
    uint32_t fl = 0;
    uint32_t cum = 0;
    for (int s = 0; s < ECQ_NSYM; ++s) {
        const uint32_t f = freq[s];
        if (f == kProbScale) {
            // single-symbol table: decoding never changes the state
            fl |= ECQ_FLAG_CONSTANT | (static_cast<uint32_t>(s) << ECQ_FLAG_CONSTANT_SYM_SHIFT);
        }
        for (uint32_t k = 0; k < f; ++k) {
            const uint32_t slot = cum + k;
            const uint32_t ff = (f == kProbScale) ? 0u : f;  // unused when constant
            entries[slot] = k | (static_cast<uint32_t>(s) << 14) | (ff << 18);
        }
        cum += f;
    }
    if (flags) *flags = fl;
    return ECQ_OK;
}

int64_t ecq_encode_interleaved_host(const uint8_t* symbols, int64_t n, int32_t n_streams, const uint32_t* freq,
                                    uint8_t* data, int64_t data_cap, uint32_t* stream_lengths,
                                    uint32_t* max_len) {
    if (n < 0 || n_streams < 1 || !freq || !stream_lengths || !max_len || (n > 0 && !symbols)) return ECQ_ERR_ARG;
    uint32_t cum[ECQ_NSYM + 1];
    cumulative(freq, cum);
    if (cum[ECQ_NSYM] != kProbScale) return ECQ_ERR_TABLE;
    std::vector<uint8_t> scratch, streams;
    return encode_tile(symbols, n, n_streams, freq, cum, data, data_cap, stream_lengths, max_len, scratch,
                       streams);
}

int64_t ecq_matrix_encoded_bound(uint32_t rows, uint32_t cols, uint32_t tile_rows, uint32_t tile_cols) {
    if (!rows || !cols || !tile_rows || !tile_cols) return ECQ_ERR_ARG;
    const int64_t slabs = (rows + tile_rows - 1) / tile_rows;
    const int64_t kt = (cols + tile_cols - 1) / tile_cols;
    const int64_t per = (static_cast<int64_t>(tile_rows) * tile_cols + ECQ_LANES - 1) / ECQ_LANES;
    return slabs * kt * ECQ_LANES * (2 * per + 4);
}

int32_t ecq_encode_matrix_host(const uint8_t* symbols, uint32_t rows, uint32_t cols, uint32_t tile_rows,
                               uint32_t tile_cols, const uint32_t* freq, int32_t n_threads, uint8_t* data,
                               int64_t data_cap, uint32_t* tile_offset, uint16_t* stream_len,
                               int64_t* total_bytes) {
    if (!symbols || !freq || !data || !tile_offset || !stream_len || !total_bytes) return ECQ_ERR_ARG;
    if (!rows || !cols || !tile_rows || !tile_cols || tile_cols % ECQ_LANES || cols % tile_cols) return ECQ_ERR_SHAPE;
    if (static_cast<uint64_t>(tile_rows) * tile_cols / ECQ_LANES > ECQ_MAX_SYMS_PER_STREAM) return ECQ_ERR_SHAPE;
    uint32_t cum[ECQ_NSYM + 1];
    cumulative(freq, cum);
    if (cum[ECQ_NSYM] != kProbScale) return ECQ_ERR_TABLE;
    const uint32_t slabs = (rows + tile_rows - 1) / tile_rows;
    const uint32_t kt = cols / tile_cols;
    const int64_t n_tiles = static_cast<int64_t>(slabs) * kt;
    const int64_t per = static_cast<int64_t>(tile_rows) * tile_cols / ECQ_LANES;
    const int64_t tile_cap = ECQ_LANES * (2 * per + 4);
    // Pass 1: encode every tile into its worst-case slot, in parallel.
    std::vector<uint8_t> staging(static_cast<size_t>(n_tiles * tile_cap));
    std::vector<int64_t> tile_bytes(static_cast<size_t>(n_tiles), 0);
    std::atomic<int64_t> next{0};
    std::atomic<int32_t> err{ECQ_OK};
    unsigned hw = std::thread::hardware_concurrency();
    int nt = n_threads > 0 ? n_threads : static_cast<int>(hw ? hw : 1);
    nt = static_cast<int>(std::min<int64_t>(nt, n_tiles));
    auto worker = [&]() {
        std::vector<uint8_t> scratch, streams, blk(static_cast<size_t>(tile_rows) * tile_cols);
        uint32_t lens[ECQ_LANES];
        for (;;) {
            const int64_t t = next.fetch_add(1);
            if (t >= n_tiles || err.load() != ECQ_OK) break;
            const uint32_t slab = static_cast<uint32_t>(t / kt), k = static_cast<uint32_t>(t % kt);
            const uint32_t r0 = slab * tile_rows, nr = std::min(tile_rows, rows - r0);
            const uint32_t c0 = k * tile_cols;
            for (uint32_t r = 0; r < nr; ++r)
                std::memcpy(blk.data() + static_cast<size_t>(r) * tile_cols,
                            symbols + static_cast<size_t>(r0 + r) * cols + c0, tile_cols);
            uint32_t ml = 0;
            const int64_t b = encode_tile(blk.data(), static_cast<int64_t>(nr) * tile_cols, ECQ_LANES, freq, cum,
                                          staging.data() + t * tile_cap, tile_cap, lens, &ml, scratch, streams);
            if (b < 0) {
                err.store(static_cast<int32_t>(b));
                break;
            }
            tile_bytes[static_cast<size_t>(t)] = b;
            for (int j = 0; j < ECQ_LANES; ++j) stream_len[t * ECQ_LANES + j] = static_cast<uint16_t>(lens[j]);
        }
    };
    std::vector<std::thread> pool;
    for (int i = 1; i < nt; ++i) pool.emplace_back(worker);
    worker();
    for (auto& th : pool) th.join();
    if (err.load() != ECQ_OK) return err.load();
    // Pass 2: concatenate (every tile is a multiple of 32 bytes, so every
    // tile starts 32-byte aligned, as the bulk copies into shared memory need).
    int64_t off = 0;
    for (int64_t t = 0; t < n_tiles; ++t) {
        if (off + tile_bytes[static_cast<size_t>(t)] > data_cap) return ECQ_ERR_CAPACITY;
        if (off > 0xFFFFFFFFll) return ECQ_ERR_CAPACITY;
        tile_offset[t] = static_cast<uint32_t>(off);
        std::memcpy(data + off, staging.data() + t * tile_cap, static_cast<size_t>(tile_bytes[static_cast<size_t>(t)]));
        off += tile_bytes[static_cast<size_t>(t)];
    }
    if (off > 0xFFFFFFFFll) return ECQ_ERR_CAPACITY;
    tile_offset[n_tiles] = static_cast<uint32_t>(off);
    *total_bytes = off;
    return ECQ_OK;
}

}  // extern "C"
