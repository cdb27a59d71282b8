/*
 * C restatement of the reference rANS decode path -- TEST INFRASTRUCTURE ONLY.
 *
 * Used by tests/ (checker), __graft_entry__.smoke() and the CPU-baseline leg
 * of bench.py.  Never linked into the product library.
 *
 *   oracle_build_table   kernel/rans.py:34-51   (12-bit static table)
 *   oracle_encode        kernel/rans.py:55-98   (lane order + encoder)
 *   oracle_decode        kernel/rans.py:101-123 (decoder, final-state check)
 *   oracle_decode_gemv   kernel/rans.py:101-123 + kernel/bench.py:52-56
 *                        (decode, then dot with the step-folded activation)
 *
 * Stream s = (rb*ncb + cb)*32 + lane holds, for k < C/32 and r < R, the code
 * at row rb*R + r and column cb*C + lane + 32k (kernel/rans.py:55-59).
 */
#include <math.h>
#include <stdlib.h>
#include <stdint.h>
#include <string.h>

#define SCALE_BITS 12
#define PROB_M (1u << SCALE_BITS)
#define RANS_L (1u << 16)
#define SYM_OFFSET 128

/* Returns 0, or 1 for a single-symbol (degenerate) distribution. */
int oracle_build_table(const uint8_t* sym, int64_t n, int64_t* freq, int64_t* cum,
                       uint32_t* table) {
    int64_t count[256];
    memset(count, 0, sizeof(count));
    for (int64_t i = 0; i < n; ++i) count[sym[i]]++;
    double total = 0.0;
    for (int s = 0; s < 256; ++s) total += (double)count[s];
    int64_t sum = 0;
    for (int s = 0; s < 256; ++s) {
        freq[s] = 0;
        if (count[s] > 0) {
            /* numpy: round-half-to-even of count*M/total, at least 1 */
            double v = nearbyint((double)count[s] * (double)PROB_M / total);
            freq[s] = v < 1.0 ? 1 : (int64_t)v;
        }
        sum += freq[s];
    }
    while (sum != (int64_t)PROB_M) {
        int64_t gap = (int64_t)PROB_M - sum;
        int top = 0;
        for (int s = 1; s < 256; ++s)
            if (freq[s] > freq[top]) top = s; /* first maximum */
        int64_t d = gap;
        if (gap < 0 && gap < 1 - freq[top]) d = 1 - freq[top];
        freq[top] += d;
        sum += d;
    }
    for (int s = 0; s < 256; ++s)
        if (freq[s] >= (int64_t)PROB_M) return 1;
    int64_t c = 0;
    for (int s = 0; s < 256; ++s) {
        cum[s] = c;
        for (int64_t k = 0; k < freq[s]; ++k)
            table[c + k] = (uint32_t)s | ((uint32_t)freq[s] << 8) | ((uint32_t)k << 20);
        c += freq[s];
    }
    return 0;
}

/* Decode one stream into out[0..n).  Returns 0 on success, 1 if the final
 * state is not RANS_L. */
static int decode_one(const uint16_t* words, uint32_t start, const uint32_t* table, int n,
                      int8_t* out) {
    const uint16_t* p = words + start;
    uint32_t st = ((uint32_t)p[0] << 16) | p[1];
    p += 2;
    for (int i = 0; i < n; ++i) {
        uint32_t e = table[st & (PROB_M - 1)];
        st = ((e >> 8) & 0xFFFu) * (st >> SCALE_BITS) + (e >> 20);
        if (st < RANS_L) st = (st << 16) | *p++;
        out[i] = (int8_t)((int)(e & 0xFFu) - SYM_OFFSET);
    }
    return st != RANS_L;
}

/* Decode streams [first, first+count) into out (count x n, stream order).
 * Returns the number of streams whose final state is wrong. */
int64_t oracle_decode(const uint16_t* words, const uint32_t* offs, const uint32_t* table,
                      int rows, int cols, int R, int C, int64_t first, int64_t count,
                      int8_t* out) {
    (void)rows;
    (void)cols;
    const int n = (C / 32) * R;
    int64_t bad = 0;
    for (int64_t s = 0; s < count; ++s)
        bad += decode_one(words, offs[first + s], table, n, out + s * n);
    return bad;
}

/* Decode streams [first, first+count) and accumulate y[row] += code * xs[col]
 * (float64).  xs is the step-folded activation x*step.  `threads` > 1 uses
 * OpenMP over streams when compiled with -fopenmp (row sums are combined
 * with atomic adds).  Returns the number of bad streams. */
int64_t oracle_decode_gemv(const uint16_t* words, const uint32_t* offs, const uint32_t* table,
                           int rows, int cols, int R, int C, int64_t first, int64_t count,
                           const double* xs, double* y, int threads) {
    const int n = (C / 32) * R;
    const int ncb = cols / C;
    int64_t bad = 0;
    if (R > 64) return -1;
#ifdef _OPENMP
#pragma omp parallel num_threads(threads > 0 ? threads : 1) reduction(+ : bad)
#endif
    {
        int8_t codes[4096];
        int8_t* buf = n <= 4096 ? codes : NULL;
        double part[64];
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int64_t s = first; s < first + count; ++s) {
            const int64_t tile = s / 32;
            const int lane = (int)(s % 32);
            const int rb = (int)(tile / ncb), cb = (int)(tile % ncb);
            for (int r = 0; r < R; ++r) part[r] = 0.0;
            if (buf) {
                bad += decode_one(words, offs[s], table, n, buf);
                for (int k = 0; k < C / 32; ++k) {
                    const double xv = xs[cb * C + lane + 32 * k];
                    for (int r = 0; r < R; ++r) part[r] += (double)buf[k * R + r] * xv;
                }
            } else {
                /* streams longer than the local buffer: decode on the fly */
                const uint16_t* p = words + offs[s];
                uint32_t st = ((uint32_t)p[0] << 16) | p[1];
                p += 2;
                for (int k = 0; k < C / 32; ++k) {
                    const double xv = xs[cb * C + lane + 32 * k];
                    for (int r = 0; r < R; ++r) {
                        uint32_t e = table[st & (PROB_M - 1)];
                        st = ((e >> 8) & 0xFFFu) * (st >> SCALE_BITS) + (e >> 20);
                        if (st < RANS_L) st = (st << 16) | *p++;
                        part[r] += (double)((int)(e & 0xFFu) - SYM_OFFSET) * xv;
                    }
                }
                bad += st != RANS_L;
            }
            for (int r = 0; r < R; ++r) {
#ifdef _OPENMP
#pragma omp atomic
#endif
                y[rb * R + r] += part[r];
            }
        }
    }
    (void)rows;
    return bad;
}

/* Symbol i (0..n-1) of stream s in stream order: for k < C/32, for r < R, the
 * code at row rb*R + r, column cb*C + lane + 32k (kernel/rans.py:55-59). */
static inline uint8_t stream_sym(const int8_t* codes, int cols, int R, int C, int64_t s, int i) {
    const int ncb = cols / C;
    const int64_t tile = s / 32;
    const int lane = (int)(s % 32);
    const int64_t rb = tile / ncb, cb = tile % ncb;
    const int k = i / R, r = i % R;
    return (uint8_t)((int)codes[(rb * R + r) * (int64_t)cols + cb * C + lane + 32 * k] + SYM_OFFSET);
}

/* Encodes stream s (kernel/rans.py:70-91): symbols pushed last to first from
 * state RANS_L; before a push the state emits its low 16 bits while
 * state >= freq << 20.  With out == NULL only counts the emitted words;
 * otherwise writes [state >> 16, state & 0xffff, emitted words reversed]. */
static int encode_one(const int8_t* codes, int cols, int R, int C, int64_t s, const int64_t* freq,
                      const int64_t* cum, int nemit_known, uint16_t* out) {
    const int n = (C / 32) * R;
    uint64_t x = RANS_L;
    int nemit = 0;
    for (int i = n - 1; i >= 0; --i) {
        const uint8_t sym = stream_sym(codes, cols, R, C, s, i);
        const uint64_t f = (uint64_t)freq[sym], c = (uint64_t)cum[sym];
        if (x >= (f << 20)) {
            if (out) out[2 + nemit_known - 1 - nemit] = (uint16_t)(x & 0xFFFFu);
            ++nemit;
            x >>= 16;
        }
        x = ((x / f) << SCALE_BITS) + x % f + c;
    }
    if (out) {
        out[0] = (uint16_t)(x >> 16);
        out[1] = (uint16_t)(x & 0xFFFFu);
    }
    return nemit;
}

/* Encode int8 codes (rows x cols, row-major) with the table's freq/cum into
 * words (+8 zero pad words) and offs; two passes over the streams (count,
 * then write), OpenMP over streams.  Returns 0, -3 when words_cap is too
 * small. */
int oracle_encode(const int8_t* codes, int rows, int cols, int R, int C, const int64_t* freq,
                  const int64_t* cum, uint16_t* words, int64_t words_cap, uint32_t* offs,
                  int64_t* nwords_out, int threads) {
    const int64_t nstreams = (int64_t)rows * cols * 32 / ((int64_t)R * C);
    int* nemit = (int*)malloc(sizeof(int) * (size_t)(nstreams > 0 ? nstreams : 1));
    if (!nemit) return -3;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t s = 0; s < nstreams; ++s) nemit[s] = encode_one(codes, cols, R, C, s, freq, cum, 0, NULL);
    int64_t total = 0;
    for (int64_t s = 0; s < nstreams; ++s) {
        offs[s] = (uint32_t)total;
        total += nemit[s] + 2;
    }
    if (total + 8 > words_cap) {
        free(nemit);
        return -3;
    }
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t s = 0; s < nstreams; ++s)
        encode_one(codes, cols, R, C, s, freq, cum, nemit[s], words + offs[s]);
    memset(words + total, 0, 8 * sizeof(uint16_t));
    *nwords_out = total + 8;
    free(nemit);
    return 0;
}
