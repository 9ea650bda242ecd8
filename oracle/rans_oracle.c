/*
 * rans_oracle.c -- CPU restatement of ecq's rANS codec, for TEST USE ONLY.
 *
 * This file is the oracle: the checker that the CUDA path is compared
 * against. Nothing in the shipped package links, loads or calls it; only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
 *
 * Parity is pinned: tests/test_oracle_golden.py checks every function here
 * against golden vectors produced by the reference's own Python codec
 * (tests/golden/make_golden.py, which imports the reference's src/rans.py
 * and src/interleaved_rans.py).
 *
 * Reference algorithm (drxddy/ecq), restated in C:
 *   constants            src/rans.py:21-23   PROB_BITS=14, M=16384, L=2^23
 *   table normaliser     src/rans.py:39-60   RANSTable.from_counts
 *   interleaved encode   src/interleaved_rans.py:76-153
 *   interleaved decode   src/interleaved_rans.py:156-217
 *   single-stream codec  src/rans.py:99-181 (identical to the interleaved
 *                        codec with n_streams == 1)
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_PROB_BITS 14u
#define OR_PROB_SCALE (1u << OR_PROB_BITS)
#define OR_RANS_L (1u << 23)

/* Reference normaliser, src/rans.py:39-60:
 *   counts = max(counts, 1) as float64
 *   freq   = uint32(counts / counts.sum() * 16384)      (truncation)
 *   freq[argmax(freq)] += 16384 - freq.sum()            (first max wins)
 * Returns the number of symbols whose count > 0 but whose freq == 0 (the
 * zero-frequency hazard: the reference encoder never terminates on them). */
int oracle_table_reference(const uint64_t *counts, int n, uint32_t *freq) {
    double c[256], sum = 0.0;
    for (int i = 0; i < n; i++) {
        c[i] = (double)(counts[i] > 0 ? counts[i] : 1);
        sum += c[i];
    }
    uint64_t fsum = 0;
    for (int i = 0; i < n; i++) {
        freq[i] = (uint32_t)(c[i] / sum * (double)OR_PROB_SCALE);
        fsum += freq[i];
    }
    int am = 0;
    for (int i = 1; i < n; i++)
        if (freq[i] > freq[am]) am = i;
    freq[am] = (uint32_t)((int64_t)freq[am] + ((int64_t)OR_PROB_SCALE - (int64_t)fsum));
    int bad = 0;
    for (int i = 0; i < n; i++)
        if (counts[i] > 0 && freq[i] == 0) bad++;
    return bad;
}

/* Clamped normaliser: the reference formula with every freq raised to at
 * least 1 before the residual goes to the (first) largest entry. Used only
 * where oracle_table_reference reports a zero-frequency hazard. The codec
 * parameters are unchanged, so the reference decoder decodes these tiles. */
void oracle_table_clamped(const uint64_t *counts, int n, uint32_t *freq) {
    double c[256], sum = 0.0;
    for (int i = 0; i < n; i++) {
        c[i] = (double)(counts[i] > 0 ? counts[i] : 1);
        sum += c[i];
    }
    int64_t fsum = 0;
    for (int i = 0; i < n; i++) {
        uint32_t f = (uint32_t)(c[i] / sum * (double)OR_PROB_SCALE);
        freq[i] = f ? f : 1u;
        fsum += freq[i];
    }
    int am = 0;
    for (int i = 1; i < n; i++)
        if (freq[i] > freq[am]) am = i;
    freq[am] = (uint32_t)((int64_t)freq[am] + ((int64_t)OR_PROB_SCALE - fsum));
}

/* cumfreq[0..n] and sym_table[16384] from freq, src/rans.py:51-58. */
void oracle_table_derive(const uint32_t *freq, int n, uint32_t *cumfreq, uint8_t *sym_table) {
    cumfreq[0] = 0;
    for (int i = 0; i < n; i++) cumfreq[i + 1] = cumfreq[i] + freq[i];
    for (int s = 0; s < n; s++)
        for (uint32_t k = cumfreq[s]; k < cumfreq[s + 1] && k < OR_PROB_SCALE; k++)
            sym_table[k] = (uint8_t)s;
}

/* Encode one stream (every S-th symbol starting at j) in reverse order, as
 * src/interleaved_rans.py:94-129. Writes the forward-order bytes into out
 * (capacity cap) and returns the length, or -1 if a symbol has freq 0 (the
 * reference loops forever there) or -2 if cap is too small. */
static long encode_stream(const uint8_t *sym, long n, int S, int j, const uint32_t *freq,
                          const uint32_t *cumfreq, uint8_t *out, long cap) {
    long cnt = 0;
    for (long i = j; i < n; i += S) cnt++;
    if (cnt == 0) return 0;
    /* bytes are produced in reverse; build reversed then flip */
    uint8_t *rev = (uint8_t *)malloc((size_t)(2 * cnt + 8));
    long nb = 0;
    uint64_t state = OR_RANS_L;
    for (long k = cnt - 1; k >= 0; k--) {
        uint32_t s = sym[j + k * (long)S];
        uint64_t f = freq[s], st = cumfreq[s];
        if (f == 0) { free(rev); return -1; }
        uint64_t x_max = ((uint64_t)(OR_RANS_L >> OR_PROB_BITS) << 8) * f;
        while (state >= x_max) {
            rev[nb++] = (uint8_t)(state & 0xFF);
            state >>= 8;
        }
        state = ((state / f) << OR_PROB_BITS) + (state % f) + st;
    }
    rev[nb++] = (uint8_t)(state & 0xFF);
    rev[nb++] = (uint8_t)((state >> 8) & 0xFF);
    rev[nb++] = (uint8_t)((state >> 16) & 0xFF);
    rev[nb++] = (uint8_t)((state >> 24) & 0xFF);
    if (nb > cap) { free(rev); return -2; }
    for (long i = 0; i < nb; i++) out[i] = rev[nb - 1 - i];
    free(rev);
    return nb;
}

/* Interleaved encode, src/interleaved_rans.py:76-153. Output layout: byte p
 * of stream j at data[j + p*S]; streams zero-padded to max_len.
 * data must hold S * (2*ceil(n/S) + 4) bytes (worst case). Returns max_len,
 * or a negative error (see encode_stream). */
long oracle_encode_interleaved(const uint8_t *sym, long n, int S, const uint32_t *freq,
                               uint8_t *data, uint32_t *stream_lengths) {
    uint32_t cumfreq[257];
    cumfreq[0] = 0;
    for (int i = 0; i < 16; i++) cumfreq[i + 1] = cumfreq[i] + freq[i];
    long per = (n + S - 1) / S;
    long cap = 2 * per + 8;
    uint8_t *tmp = (uint8_t *)malloc((size_t)(cap * S + 1));
    long max_len = 0;
    for (int j = 0; j < S; j++) {
        long len = encode_stream(sym, n, S, j, freq, cumfreq, tmp + (long)j * cap, cap);
        if (len < 0) { free(tmp); return len; }
        stream_lengths[j] = (uint32_t)len;
        if (len > max_len) max_len = len;
    }
    memset(data, 0, (size_t)(max_len * S));
    for (int j = 0; j < S; j++)
        for (long p = 0; p < (long)stream_lengths[j]; p++)
            data[j + p * S] = tmp[(long)j * cap + p];
    free(tmp);
    return max_len;
}

/* Interleaved decode, src/interleaved_rans.py:156-217, including its two
 * guards: streams shorter than 4 bytes are skipped (their outputs stay 0),
 * and renormalisation stops at the stream's length. Also reports, per
 * stream, the final state and read position (end_state/end_ptr may be
 * NULL); for a stream produced by the reference encoder these are
 * exactly (2^23, stream_length). Returns the number of streams whose end
 * state differs from that (0 for intact data). */
int oracle_decode_interleaved(const uint8_t *data, const uint32_t *stream_lengths, int S, long n,
                              const uint32_t *freq, uint8_t *out, uint32_t *end_state,
                              uint32_t *end_ptr) {
    uint32_t cumfreq[17];
    uint8_t *sym_table = (uint8_t *)malloc(OR_PROB_SCALE);
    memset(sym_table, 0, OR_PROB_SCALE);
    oracle_table_derive(freq, 16, cumfreq, sym_table);
    memset(out, 0, (size_t)n);
    int bad = 0;
    for (int j = 0; j < S; j++) {
        uint32_t len = stream_lengths[j];
        if (end_state) end_state[j] = 0;
        if (end_ptr) end_ptr[j] = 0;
        if (len < 4) {
            /* the reference skips the stream; its symbols stay 0 */
            if (j < n) bad++;
            continue;
        }
        uint64_t x = ((uint64_t)data[j] << 24) | ((uint64_t)data[j + S] << 16) |
                     ((uint64_t)data[j + 2 * S] << 8) | (uint64_t)data[j + 3 * S];
        uint32_t ptr = 4;
        for (long i = j; i < n; i += S) {
            uint32_t slot = (uint32_t)(x & (OR_PROB_SCALE - 1));
            uint32_t s = sym_table[slot];
            out[i] = (uint8_t)s;
            x = (uint64_t)freq[s] * (x >> OR_PROB_BITS) + slot - cumfreq[s];
            while (x < OR_RANS_L && ptr < len) {
                x = (x << 8) | data[j + (long)ptr * S];
                ptr++;
            }
        }
        if (end_state) end_state[j] = (uint32_t)x;
        if (end_ptr) end_ptr[j] = ptr;
        if (x != OR_RANS_L || ptr != len) bad++;
    }
    free(sym_table);
    return bad;
}

/* y[r] = sum_c (float(sym[r,c]) - 8) * scale[r, c/g] * x[c], accumulated
 * in double, for a row-major [M,K] symbol matrix and fp32 scales/x.
 * The dequantisation is the reference form sym*scale + zero with
 * zero = -8*scale (src/quantizer.py:33-35). */
void oracle_dequant_gemv(const uint8_t *sym, long M, long K, const float *scale, long g,
                         const float *x, float *y) {
    long ng = (K + g - 1) / g;
    for (long r = 0; r < M; r++) {
        double acc = 0.0;
        for (long c = 0; c < K; c++) {
            double w = ((double)sym[r * K + c] - 8.0) * (double)scale[r * ng + c / g];
            acc += w * (double)x[c];
        }
        y[r] = (float)acc;
    }
}

/* The reference's CPU path over the tiles [t0, t1) of a packed matrix:
 * interleaved_rans_decode per tile (src/interleaved_rans.py:156-217), then
 * dequantise (sym - 8) * scale (src/quantizer.py:33-35) and accumulate the
 * matvec into y_acc (double, indexed by row). Tiles are 32-stream tiles of
 * tile_rows x tile_cols, row-slab major. Callers that run several ranges
 * in parallel give each a disjoint set of row slabs. Returns the number of
 * streams that failed the end-state check. */
int oracle_gemv_packed(const uint8_t *data, const uint32_t *tile_offset, const uint16_t *stream_len,
                       long rows, long cols, long tile_rows, long tile_cols, const uint32_t *freq,
                       const float *scales, long g, const float *x, long t0, long t1, double *y_acc) {
    long nk = cols / tile_cols;
    long ng = (cols + g - 1) / g;
    uint8_t *sym = (uint8_t *)malloc((size_t)(tile_rows * tile_cols));
    uint32_t lens[32];
    int bad = 0;
    for (long t = t0; t < t1; t++) {
        long slab = t / nk, k = t % nk;
        long r0 = slab * tile_rows, c0 = k * tile_cols;
        long nr = rows - r0 < tile_rows ? rows - r0 : tile_rows;
        for (int j = 0; j < 32; j++) lens[j] = stream_len[t * 32 + j];
        bad += oracle_decode_interleaved(data + tile_offset[t], lens, 32, nr * tile_cols, freq, sym, NULL, NULL);
        for (long r = 0; r < nr; r++) {
            double acc = 0.0;
            const uint8_t *sr = sym + r * tile_cols;
            const float *sc = scales + (r0 + r) * ng;
            for (long c = 0; c < tile_cols; c++)
                acc += ((double)sr[c] - 8.0) * (double)sc[(c0 + c) / g] * (double)x[c0 + c];
            y_acc[r0 + r] += acc;
        }
    }
    free(sym);
    return bad;
}
