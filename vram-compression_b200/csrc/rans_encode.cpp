// Host-side producer of the tile-interleaved rANS bitstream, bit-exact with the
// reference encoder (kernel/rans.py:34-98: build_table, lane_order, encode).
//
// The reference encodes every stream in lock-step with numpy (rans.py:76-83)
// and reverses the emitted words per stream in a Python loop (rans.py:90-91).
// Here each thread owns a contiguous range of tiles: pass 1 encodes to count
// the words each stream emits, a prefix sum turns the counts into offsets,
// pass 2 re-encodes and writes the emitted words back-to-front directly into
// their final position, so no per-stream temporary or reversal is needed.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/rans_b200.h"

namespace {

constexpr int kScaleBits = 12;
constexpr uint32_t kProbM = 1u << kScaleBits;
constexpr uint32_t kRansL = 1u << 16;
constexpr int kPadWords = 8;

int clamp_threads(int n) {
    if (n > 0) return n;
    const unsigned hw = std::thread::hardware_concurrency();
    return hw ? static_cast<int>(hw) : 1;
}

template <class F>
void parallel_for(int64_t n, int nthreads, F&& f) {
    nthreads = clamp_threads(nthreads);
    if (nthreads > n) nthreads = static_cast<int>(n > 0 ? n : 1);
    if (nthreads <= 1) {
        f(0, int64_t(0), n);
        return;
    }
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; ++t) {
        const int64_t a = n * t / nthreads, b = n * (t + 1) / nthreads;
        pool.emplace_back([&f, t, a, b] { f(t, a, b); });
    }
    for (auto& th : pool) th.join();
}

struct Coder {
    uint32_t freq[256];
    uint32_t cum[256];
};

// freq/cum from a table in the reference layout sym | freq<<8 | (slot-cum)<<20.
bool coder_from_table(const uint32_t* table, Coder& c) {
    std::memset(&c, 0, sizeof(c));
    for (uint32_t slot = 0; slot < kProbM; ++slot) {
        const uint32_t e = table[slot];
        const uint32_t s = e & 0xFFu, f = (e >> 8) & 0xFFFu, b = e >> 20;
        if (b == 0) {
            c.freq[s] = f;
            c.cum[s] = slot;
        }
    }
    uint32_t total = 0;
    for (int s = 0; s < 256; ++s) total += c.freq[s];
    return total == kProbM;
}

// Encodes the 32 streams of tile (rb, cb).  sym(lane, i) reads the code at
// row rb*R + i%R, column cb*C + lane + 32*(i/R).  Emits words via emit(lane,
// j, word) in encode order (j = 0 is the LAST payload word of the stream) and
// returns per-lane counts and final states.
template <class Emit>
void encode_tile(const int8_t* codes, int cols, int R, int C, int rb, int cb, const Coder& cd,
                 uint32_t* nemit, uint32_t* final_state, Emit&& emit) {
    const int n = (C / 32) * R;
    for (int lane = 0; lane < 32; ++lane) {
        uint64_t x = kRansL;
        uint32_t cnt = 0;
        const int col0 = cb * C + lane;
        for (int i = n - 1; i >= 0; --i) {
            const int r = i % R, k = i / R;
            const int code = codes[(int64_t)(rb * R + r) * cols + col0 + 32 * k];
            const uint32_t s = static_cast<uint32_t>(code + 128);
            const uint64_t f = cd.freq[s];
            if (x >= (f << 20)) {
                emit(lane, cnt, static_cast<uint16_t>(x & 0xFFFFu));
                ++cnt;
                x >>= 16;
            }
            x = ((x / f) << kScaleBits) + (x % f) + cd.cum[s];
        }
        nemit[lane] = cnt;
        final_state[lane] = static_cast<uint32_t>(x);
    }
}

}  // namespace

extern "C" int rans_build_table_host(const int8_t* codes, int64_t n, uint32_t* table, int32_t* freq_out,
                                     int32_t* cum_out, int nthreads) {
    const int nt = clamp_threads(nthreads);
    std::vector<std::vector<int64_t>> hist(nt, std::vector<int64_t>(256, 0));
    parallel_for(n, nt, [&](int t, int64_t a, int64_t b) {
        int64_t* h = hist[t].data();
        for (int64_t i = a; i < b; ++i) h[static_cast<uint8_t>(codes[i] + 128)]++;
    });
    int64_t count[256] = {0};
    for (auto& h : hist)
        for (int s = 0; s < 256; ++s) count[s] += h[s];
    // kernel/rans.py:36-44: round-half-to-even of count*M/total (min 1), then
    // the first largest bin absorbs the rounding difference
    double total = 0.0;
    for (int s = 0; s < 256; ++s) total += static_cast<double>(count[s]);
    int64_t freq[256];
    int64_t sum = 0;
    for (int s = 0; s < 256; ++s) {
        freq[s] = 0;
        if (count[s] > 0) {
            const double v = std::nearbyint(static_cast<double>(count[s]) * kProbM / total);
            freq[s] = v < 1.0 ? 1 : static_cast<int64_t>(v);
        }
        sum += freq[s];
    }
    while (sum != static_cast<int64_t>(kProbM)) {
        const int64_t gap = static_cast<int64_t>(kProbM) - sum;
        int top = 0;
        for (int s = 1; s < 256; ++s)
            if (freq[s] > freq[top]) top = s;
        int64_t d = gap;
        if (gap < 0 && gap < 1 - freq[top]) d = 1 - freq[top];
        freq[top] += d;
        sum += d;
    }
    for (int s = 0; s < 256; ++s)
        if (freq[s] >= static_cast<int64_t>(kProbM)) return 1;
    int64_t c = 0;
    for (int s = 0; s < 256; ++s) {
        if (freq_out) freq_out[s] = static_cast<int32_t>(freq[s]);
        if (cum_out) cum_out[s] = static_cast<int32_t>(c);
        for (int64_t k = 0; k < freq[s]; ++k)
            table[c + k] = static_cast<uint32_t>(s) | (static_cast<uint32_t>(freq[s]) << 8) |
                           (static_cast<uint32_t>(k) << 20);
        c += freq[s];
    }
    return 0;
}

extern "C" int64_t rans_encode_bound(int rows, int cols, int R, int C) {
    if (R <= 0 || C <= 0 || rows % R || cols % C || C % 32) return -2;
    const int64_t streams = (int64_t)(rows / R) * (cols / C) * 32;
    return streams * ((C / 32) * R + 2) + kPadWords;
}

extern "C" int rans_encode_host(const int8_t* codes, int rows, int cols, int R, int C, const uint32_t* table,
                                uint16_t* words, int64_t words_cap, uint32_t* offs, int64_t* nwords_out,
                                int nthreads) {
    if (R <= 0 || C <= 0 || rows <= 0 || cols <= 0 || rows % R || cols % C || C % 32) return -2;
    Coder cd;
    if (!coder_from_table(table, cd)) return -4;
    const int ncb = cols / C;
    const int64_t ntiles = (int64_t)(rows / R) * ncb;
    const int64_t nstreams = ntiles * 32;
    std::vector<uint32_t> len(nstreams);
    // pass 1: stream lengths (2 state words + emitted words)
    parallel_for(ntiles, nthreads, [&](int, int64_t a, int64_t b) {
        uint32_t cnt[32], st[32];
        for (int64_t t = a; t < b; ++t) {
            encode_tile(codes, cols, R, C, (int)(t / ncb), (int)(t % ncb), cd, cnt, st,
                        [](int, uint32_t, uint16_t) {});
            for (int l = 0; l < 32; ++l) len[t * 32 + l] = cnt[l] + 2;
        }
    });
    int64_t total = 0;
    for (int64_t s = 0; s < nstreams; ++s) {
        offs[s] = static_cast<uint32_t>(total);
        total += len[s];
        if (total > 0xFFFFFFFFll) return -5;   // offsets are 32-bit word indices
    }
    if (total + kPadWords > words_cap) return -3;
    // pass 2: write [state_hi, state_lo, emitted words reversed]
    parallel_for(ntiles, nthreads, [&](int, int64_t a, int64_t b) {
        uint32_t cnt[32], st[32];
        for (int64_t t = a; t < b; ++t) {
            const int64_t s0 = t * 32;
            encode_tile(codes, cols, R, C, (int)(t / ncb), (int)(t % ncb), cd, cnt, st,
                        [&](int lane, uint32_t j, uint16_t w) {
                            const int64_t s = s0 + lane;
                            // emitted word j lands at offs + 2 + (len-2) - 1 - j
                            words[offs[s] + len[s] - 1 - j] = w;
                        });
            for (int l = 0; l < 32; ++l) {
                words[offs[s0 + l]] = static_cast<uint16_t>(st[l] >> 16);
                words[offs[s0 + l] + 1] = static_cast<uint16_t>(st[l] & 0xFFFFu);
            }
        }
    });
    for (int i = 0; i < kPadWords; ++i) words[total + i] = 0;
    if (nwords_out) *nwords_out = total + kPadWords;
    return 0;
}
