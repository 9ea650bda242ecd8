/*
 * A plain C host of libecq's C ABI (no Python, no CUDA headers): builds a
 * frequency table from symbol counts, encodes one 32-stream interleaved tile
 * with the host codec and builds the decode table, then prints the results
 * for tests/test_c_abi_host.py to check against the oracle.
 *
 *   cc -I include tests/c/abi_host_example.c -Lecq_b200/_lib -lecq -o example
 *
 * Symbols come from a 64-bit LCG mapped onto a peaked distribution around 8,
 * so that the test can regenerate them.
 */
#include <inttypes.h>
#include <stdio.h>
#include <stdlib.h>

#include "ecq.h"

static uint8_t next_symbol(uint64_t *x) {
    *x = *x * 6364136223846793005ull + 1442695040888963407ull;
    const unsigned u = (unsigned)((*x >> 40) % 1000u);
    if (u < 600) return 8;
    if (u < 760) return 7;
    if (u < 920) return 9;
    if (u < 950) return 6;
    if (u < 980) return 10;
    return (u & 1u) ? 5 : 11;
}

int main(int argc, char **argv) {
    const int64_t n = argc > 1 ? atoll(argv[1]) : 4099;
    const int32_t streams = 32;
    uint8_t *sym = malloc((size_t)n);
    uint64_t x = 12345u, counts[16] = {0};
    for (int64_t i = 0; i < n; ++i) {
        sym[i] = next_symbol(&x);
        counts[sym[i]]++;
    }
    uint32_t freq[16];
    int32_t normaliser = -1;
    if (ecq_table_from_counts(counts, freq, &normaliser) != ECQ_OK) return 2;
    const int64_t cap = 64 + 2 * n + 8 * streams;
    uint8_t *data = malloc((size_t)cap);
    uint32_t lens[32], max_len = 0;
    const int64_t nbytes = ecq_encode_interleaved_host(sym, n, streams, freq, data, cap, lens, &max_len);
    if (nbytes < 0) return 3;
    uint32_t *entries = malloc(16384 * sizeof(uint32_t));
    uint32_t flags = 0;
    if (ecq_build_decode_table(freq, entries, &flags) != ECQ_OK) return 4;
    uint64_t table_sum = 0;
    for (int i = 0; i < 16384; ++i) table_sum += entries[i];
    printf("version %d\nnormaliser %d\nfreq", ecq_version(), normaliser);
    for (int s = 0; s < 16; ++s) printf(" %u", freq[s]);
    printf("\nlens");
    for (int j = 0; j < streams; ++j) printf(" %u", lens[j]);
    printf("\nmax_len %u\nbytes %" PRId64 "\ntable_sum %" PRIu64 "\nflags %u\ndata ", max_len, nbytes, table_sum, flags);
    for (int64_t i = 0; i < nbytes; ++i) printf("%02x", data[i]);
    printf("\n");
    free(sym);
    free(data);
    free(entries);
    return 0;
}
