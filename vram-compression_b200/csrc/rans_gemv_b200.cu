// Fused rANS-decode + batch-1 GEMV for B200 (sm_100a).
//
// Bitstream: the reference's tile-interleaved rANS (kernel/rans_gemv.cu:1-15,
// kernel/rans.py:55-98); see include/rans_b200.h for the format.
//
// Execution model (differs from the reference's one-stream-per-lane, one
// global load per renormalisation, kernel/rans_gemv.cu:39-77):
//   * a warp owns a WORK ITEM: a row block rb and a range of its column
//     blocks (a segment), decoded K tiles per pass.  The tiles of a pass are
//     consecutive in stream order, so their word streams form ONE contiguous
//     span of `words`.
//   * the span is staged into a per-warp shared-memory buffer with 16-byte
//     cp.async copies (fully coalesced), and every renormalisation word is then
//     read from shared memory instead of global memory (a one-tile pass too
//     large for the buffer goes through per-lane windows of it);
//   * each lane decodes K independent streams (lane l of K tiles) interleaved
//     symbol by symbol, hiding the table-lookup -> multiply -> compare chain;
//   * the 16 KB slot table is re-laid in shared memory (16 KB-aligned) as
//       bias | sym << 12 | freq << 20
//     so the entry address is one shift + one LOP3, freq one shift, bias one
//     mask, and 4096*code one LOP3 + FADD (the float 2^23 + 4096*sym);
//   * fp32 accumulation; the R partial sums per lane are combined with
//     a transpose-reduce (reduce-scatter) butterfly, R-1 + log2(32/R) shuffles
//     instead of 5*R, and stored without atomics whenever a warp covers every
//     column block of its rows.
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <mutex>
#include <unordered_map>
#include <vector>

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/rans_b200.h"

namespace rb200 {

constexpr int kScaleBits = 12;
constexpr uint32_t kProbM = 1u << kScaleBits;
constexpr uint32_t kRansL = 1u << 16;
constexpr int kPadWords = 8;
#ifndef RB_WARPS
#define RB_WARPS 8
#endif
#ifndef RB_STAGE_BYTES
#define RB_STAGE_BYTES 8192
#endif
#ifndef RB_MINB
#define RB_MINB 2        // 2 CTAs/SM: lets ptxas use up to 128 registers (no rematerialisation)
#endif
#ifndef RB_PDL
#define RB_PDL 1         // programmatic dependent launch of the step kernel
#endif
#ifndef RB_POLL_MAX_NS
#define RB_POLL_MAX_NS 256   // chain waits: longest sleep between two polls of a completion counter
#endif
#ifndef RB_PREFETCH
#define RB_PREFETCH 0    // each CTA warms L2 for the chunk one wave ahead (measured: no gain)
#endif
#ifndef RB_LAYOUT
#define RB_LAYOUT 1      // shared-memory table entry: 0 = sym|bias<<8|freq<<20, 1 = bias|sym<<12|freq<<20
#endif
#ifndef RB_I4_UNROLL
#define RB_I4_UNROLL 4   // int4 baseline: column groups in flight per lane
#endif
#ifndef RB_ALIGNTAB
#define RB_ALIGNTAB 1    // place the table at a 16 KB-aligned shared address (address = one LOP3)
#endif
#ifndef RB_TABCOPIES
#define RB_TABCOPIES 2   // copies of the slot table in shared memory, interleaved by lane (1 or 2)
#endif
// The table sits at an aligned address (entry address = shift + one LOP3)
// only with one copy; two lane-interleaved copies (entry of slot s for lane l
// at word 2s + (l & 1): the lanes of one parity reach only every other bank)
// use and + shift-add at any address.
#define RB_TAB_ALIGNED (RB_ALIGNTAB && RB_TABCOPIES == 1)
constexpr int kWarps = RB_WARPS;          // warps per CTA
constexpr int kI4Unroll = RB_I4_UNROLL;
constexpr int kThreads = kWarps * 32;
constexpr int kStageBytes = RB_STAGE_BYTES;  // per-warp staging buffer (0: no staging)
constexpr int kTabCopies = RB_TABCOPIES;
static_assert(kTabCopies == 1 || kTabCopies == 2, "one or two table copies");
constexpr int kTableBytes = kProbM * 4 * kTabCopies;     // in shared memory
constexpr int kAlignPad = RB_TAB_ALIGNED ? kTableBytes : 0;
constexpr int kSmemBytes = kTableBytes + kWarps * kStageBytes + kAlignPad;
// Layout 1 yields 4096*code from one LOP3; the sums are scaled back by 2^-12 (exact).
constexpr float kCodeScale = RB_LAYOUT == 1 ? 4096.0f : 1.0f;
constexpr float kInvCodeScale = 1.0f / kCodeScale;

constexpr int kMaxPeers = 8;              // ranks of one NVLink/NVSwitch node

// Device view of one matrix plus its work decomposition.
struct MatDev {
    const uint16_t* words;
    const uint32_t* offs;
    const uint32_t* table;
    const void* x;
    const float* step;     // NULL: x is fp32 pre-scaled; else x is bf16
    float* y;
    int64_t nwords;        // incl. pad, or -1
    int64_t wlimit;        // nwords < 0: words readable from `words` on (to the end of its
                           // device allocation), 0 = unknown
    int rows, cols, C, ncb, nrb, nk;
    int kcol;              // column-mode streams per lane (2..4)
    int nseg, cbs;         // column-mode segments per row block, cbs per segment
    int nitems;
    int accumulate;        // 1: atomicAdd into y (split rows), 0: store
    int npeer;             // > 0: store every output row to all of ypeer[] instead of y
    int tail_words;        // most words one stream can hold: 2 state words + one per symbol
    int combine;           // 1: the nseg segments of a row block are consecutive warps of one
                           // CTA and add up in shared memory (step kernel, one item per warp)
    float* ypeer[kMaxPeers];   // the same rows of every rank's output buffer (peer addresses)
    float* partials;       // nseg > 1 without accumulate: [nrb][nseg][R] segment sums (workspace)
    uint32_t* counters;    // [nrb] arrivals per row block, zero between launches (workspace)
};

struct Chunk {             // one CTA's share of work: items [item0, item0 + nitems) of one matrix
    int desc, item0, nitems;
    int phase;             // chain launcher: dependency phase of the matrix (0 for a step plan)
};

struct StepHeader {
    int ndesc, nchunks, R;
    int ahead;             // L2-prefetch distance in chunks (co-resident CTAs), 0 = off
    int64_t spans_off;     // byte offset of uint2 spans[nchunks] (word range per chunk)
    int64_t pad_;
};

// The CTA's dynamic shared memory: the 16 KB slot table and one stage per
// warp.  With RB_ALIGNTAB the table sits at the first 16 KB-aligned shared
// address of the block, stages fill the space before and after it.
extern __shared__ __align__(16) uint8_t g_smem[];

struct SmemMap {
    uint32_t* tab;       // generic pointer to the table
    uint32_t tab_s;      // its shared-window address
    uint16_t* stage;     // this warp's stage
};

__device__ __forceinline__ SmemMap smem_map(int warp) {
    SmemMap m;
    const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(g_smem));
    const uint32_t toff = RB_TAB_ALIGNED ? ((uint32_t)kTableBytes - (base & (kTableBytes - 1))) & (kTableBytes - 1) : 0u;
    m.tab = reinterpret_cast<uint32_t*>(g_smem + toff);
    m.tab_s = base + toff;
    const int nbefore = kStageBytes > 0 ? (int)(toff / kStageBytes) : 0;
    const uint32_t soff = warp < nbefore ? (uint32_t)warp * kStageBytes
                                         : toff + kTableBytes + (uint32_t)(warp - nbefore) * kStageBytes;
    m.stage = reinterpret_cast<uint16_t*>(g_smem + soff);
    return m;
}

// ------------------------------------------------------------ primitives
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* gptr) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(gptr));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }

// Programmatic dependent launch.  A step kernel lets the next kernel of its
// stream start as soon as all of its CTAs are running, and itself waits for
// the previous kernel only before it touches anything that kernel may produce
// or consume (activations, outputs, split counters/partials).  Table loads,
// offsets and word staging read immutable weights and overlap the previous
// kernel's tail.  In a kernel launched without the attribute both are no-ops.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Reference table entry sym | freq<<8 | bias<<20 re-laid for the decoder.
__device__ __forceinline__ uint32_t relayout_entry(uint32_t e) {
    const uint32_t sym = e & 0xFFu, freq = (e >> 8) & 0xFFFu, bias = e >> 20;
#if RB_LAYOUT == 1
    return bias | (sym << 12) | (freq << 20);
#else
    return sym | (bias << 8) | (freq << 20);
#endif
}

// Every kernel that calls this runs kThreads threads: a compile-time stride
// lets each thread issue all of its loads before the first store (one L2
// round trip per table instead of one per few entries).
__device__ __forceinline__ void load_table(uint32_t* tab, const uint32_t* __restrict__ table) {
    static_assert(kProbM % kThreads == 0, "table entries per thread");
    constexpr int kPer = kProbM / kThreads;
    uint32_t e[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) e[k] = __ldg(table + threadIdx.x + k * kThreads);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const uint32_t v = relayout_entry(e[k]);
        const int i = threadIdx.x + k * kThreads;
#pragma unroll
        for (int c = 0; c < kTabCopies; ++c) tab[i * kTabCopies + c] = v;
    }
}

// The table entry of a state for this thread's lane (C++ paths), and the
// shared address the PTX paths add the slot offset to.
__device__ __forceinline__ uint32_t tab_entry(const uint32_t* tab, uint32_t st) {
    return tab[(st & (kProbM - 1)) * kTabCopies + (threadIdx.x & (kTabCopies - 1))];
}
__device__ __forceinline__ uint32_t tab_lane_base(uint32_t tab_s) {
    return tab_s + 4u * (threadIdx.x & (kTabCopies - 1));
}

__device__ __forceinline__ uint32_t entry_freq(uint32_t e) { return e >> 20; }
__device__ __forceinline__ uint32_t entry_bias(uint32_t e) {
    return RB_LAYOUT == 1 ? (e & 0xFFFu) : ((e >> 8) & 0xFFFu);
}

// kCodeScale * code as an exact float.  Layout 0: the float 2^23 + sym built
// by one byte-permute, minus 2^23 + 128.  Layout 1: the float 2^23 + 4096*sym
// (sym already sits at bits 12..19), minus 2^23 + 4096*128.
__device__ __forceinline__ float entry_code(uint32_t e) {
#if RB_LAYOUT == 1
    return __int_as_float((e & 0x000FF000u) | 0x4B000000u) - 8912896.0f;
#else
    return __int_as_float(__byte_perm(e, 0x4B000000u, 0x7540)) - 8388736.0f;
#endif
}

// Activation load mode XM: bit 0 set = bf16 x times the fp32 step (folded
// here), clear = fp32 x already multiplied by the step; bit 1 set = load x
// with plain (weak, L1-cached) global loads instead of the read-only path,
// for kernels in which x may have been written by other CTAs earlier in the
// same launch (the chain kernel: a phase's input is an earlier phase's
// output).  There the CTA's reads follow an ld.acquire of the producer's
// completion counter and a bar.sync, which the memory model extends to weak
// loads; the non-coherent read-only path is outside it.
// Bit 2 set = load the activations of k-step k+1 while k-step k decodes
// (hides their latency where they miss L1: large activation vectors next to
// 192 KB of shared memory per SM; the chain kernel uses it).
// Bit 3 set = the chain kernel: before the first activation load each warp
// waits for the previous phase (dep_wait) instead of the previous kernel.
constexpr int kXBf16 = 1, kXCoherent = 2, kXPref = 4, kXChain = 8;

// Per-CTA dependency state of the chain kernel, read inside the decode path:
// the workspace header, the phase the current chunk waits for (-1: none) and,
// per warp, the highest phase that warp has already seen complete.
struct ChainHeader;
__device__ bool chain_wait(const ChainHeader* h, int p);
__shared__ const ChainHeader* g_chain_hdr;
__shared__ int g_chain_wait;
__shared__ int g_chain_known[kWarps];

// Where the decode path may first touch activations: a step kernel waits for
// the previous kernel of its stream (programmatic dependent launch), a chain
// kernel's warp for the previous phase -- after its words are staged and its
// states read, so both overlap the wait.  A chain wait that runs out has
// recorded the error for the host; the warp then goes on (its outputs are
// reported invalid) so the kernel always ends.
template <int XM>
__device__ __forceinline__ void dep_wait() {
    if constexpr ((XM & kXChain) != 0) {
        const int p = g_chain_wait;
        const int w = threadIdx.x >> 5;
        if (p >= 0 && p > g_chain_known[w]) {
            int ok = 1;
            if ((threadIdx.x & 31) == 0) ok = chain_wait(g_chain_hdr, p) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (ok && (threadIdx.x & 31) == 0) g_chain_known[w] = p;
            __syncwarp();   // lane 0's acquire orders every lane's later loads
        }
    } else {
        pdl_wait();
    }
}

template <int XM>
__device__ __forceinline__ float load_x(const MatDev& d, int c) {
    if (XM & kXBf16) {
        const unsigned short* xb = reinterpret_cast<const unsigned short*>(d.x);
        const uint32_t v = xb[c];   // plain load: never the read-only path
        return __uint_as_float(v << 16) * __ldg(d.step + c);   // bf16 -> fp32 is exact
    } else {
        const float* xf = reinterpret_cast<const float*>(d.x);
        return (XM & kXCoherent) ? xf[c] : __ldg(xf + c);
    }
}

// Transpose-reduce V values (power of two <= 32) across the warp.  Lane l ends
// with the full 32-lane sum of value index l >> (5 - log2 V).
template <int V>
__device__ __forceinline__ float reduce_scatter(float (&v)[V], int lane) {
    int m = 16;
#pragma unroll
    for (int h = V / 2; h >= 1; h >>= 1) {
        const bool up = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < h; ++i) {
            const float send = up ? v[i] : v[i + h];
            const float keep = up ? v[i + h] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
        m >>= 1;
    }
    float s = v[0];
    for (; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    return s;
}

template <int V>
struct Log2 { static constexpr int value = 1 + Log2<V / 2>::value; };
template <>
struct Log2<1> { static constexpr int value = 0; };

// ------------------------------------------------------------ staging
// Span of words [w0, w1) (word indices into d.words).  Copies the 16-byte
// aligned chunks covering it into `stage` and returns the stage index of word
// w0.  Every copied chunk contains at least one byte of the span, so no chunk
// touches a page the span does not touch.
__device__ __forceinline__ uint32_t stage_span(const MatDev& d, uint16_t* stage, uint32_t w0,
                                               uint64_t w1, int lane) {
    const uintptr_t b0 = reinterpret_cast<uintptr_t>(d.words) + 2ull * w0;
    const uintptr_t b1 = reinterpret_cast<uintptr_t>(d.words) + 2ull * w1;
    const uintptr_t a0 = b0 & ~uintptr_t(15);
    const uintptr_t a1 = (b1 + 15) & ~uintptr_t(15);
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(stage));
    const int n16 = static_cast<int>((a1 - a0) >> 4);
    for (int i = lane; i < n16; i += 32) cp_async16(s + 16u * i, reinterpret_cast<const void*>(a0 + 16ull * i));
    cp_async_commit();
    cp_async_wait_all();
    __syncwarp();
    return static_cast<uint32_t>((b0 - a0) >> 1);
}

// Bytes a staged span [w0, w1) occupies (+16 for the one-word look-ahead).
__device__ __forceinline__ uint64_t staged_bytes(const MatDev& d, uint32_t w0, uint64_t w1) {
    const uintptr_t b0 = reinterpret_cast<uintptr_t>(d.words) + 2ull * w0;
    const uintptr_t b1 = reinterpret_cast<uintptr_t>(d.words) + 2ull * w1;
    return ((b1 + 15) & ~uintptr_t(15)) - (b0 & ~uintptr_t(15)) + 16;
}

// End (exclusive word index) of the span that ends at stream `s_end`
// (one past the last stream of the span), or UINT64_MAX when unknown.
__device__ __forceinline__ uint64_t span_end(const MatDev& d, int64_t s_end) {
    const int64_t nstreams = (int64_t)d.nrb * d.ncb * 32;
    if (s_end < nstreams) return d.offs[s_end];
    if (d.nwords >= 0) return (uint64_t)(d.nwords - kPadWords);
    if (d.wlimit > 0) {
        // Length unknown (the reference entry points pass none): the final
        // stream ends within tail_words of its start (a symbol takes at most
        // one renormalisation word) and within the words' device allocation,
        // so staging up to the nearer bound copies every word it holds.
        const uint64_t e = (uint64_t)d.offs[nstreams - 1] + (uint64_t)d.tail_words;
        return e < (uint64_t)d.wlimit ? e : (uint64_t)d.wlimit;
    }
    return UINT64_MAX;
}

// ------------------------------------------------------------ decode core
// Decodes one pass: K streams per lane, C/32 k-steps of R symbols each.
// wb/pos: word base (shared stage or global words) and per-stream word index
// of the stream's first (state) word.  NACC == 1: all streams share rows
// (column mode, acc[0][r]); NACC == K: stream j owns acc[j] (row mode, shared x).
// Word source of a pass.  Staged: `pos` are BYTE offsets into the CTA's
// shared memory (the stage lives there), so a renormalisation read is one
// LDS at [offset + array base] with no address arithmetic.  Global: `pos`
// are word indices into d.words (spans too large to stage, or whose end is
// unknown).
template <bool STAGED>
struct WordSrc;
template <>
struct WordSrc<true> {
    static constexpr uint32_t kStep = 2;
    __device__ __forceinline__ static uint32_t at(const MatDev&, uint32_t p) {
        return *reinterpret_cast<const uint16_t*>(g_smem + p);
    }
};
template <>
struct WordSrc<false> {
    static constexpr uint32_t kStep = 1;
    __device__ __forceinline__ static uint32_t at(const MatDev& d, uint32_t p) { return __ldg(d.words + p); }
};

template <int K, int NACC, int XM>
__device__ __forceinline__ void load_xs(const MatDev& d, const int (&xcol)[K], int kk, int k, float (&xv)[K]) {
    if (NACC == K) {
        const float v = load_x<XM>(d, xcol[0] + 32 * k);
#pragma unroll
        for (int j = 0; j < K; ++j) xv[j] = v;
    } else {
#pragma unroll
        for (int j = 0; j < K; ++j) xv[j] = (j < kk) ? load_x<XM>(d, xcol[j] + 32 * k) : 0.f;
    }
}

#ifndef RB_INNER
#define RB_INNER 1       // 0: C++ symbol step, 1: PTX symbol step (staged passes)
#endif
#ifndef RB_XPREF
#define RB_XPREF 0
#endif

// One symbol of a staged stream, written in PTX so the instruction sequence
// is fixed: table lookup (LDS), freq/bias fields, state update (IMAD),
// predicated renormalisation (PRMT shift-in + pointer bump + LDS of the next
// word), code value (one logic op + FADD) and the FMA.
// st: state, w: next word, pw: shared byte address of w, tb: shared address
// of the table (16 KB-aligned with RB_ALIGNTAB, so the entry address is
// (st << 2 & 0x3ffc) | tb).
#if RB_LAYOUT == 1
#define RB_PTX_FIELDS                                  \
    "shr.u32 f, e, 20;\n\t"                            \
    "and.b32 b, e, 4095;\n\t"                          \
    "shr.u32 hi, %0, 12;\n\t"                          \
    "mad.lo.u32 %0, f, hi, b;\n\t"                     \
    "setp.lt.u32 p, %0, 65536;\n\t"                    \
    "@p prmt.b32 %0, %1, %0, 0x5410;\n\t"              \
    "@p add.u32 %2, %2, 2;\n\t"                        \
    "@p ld.shared.u16 %1, [%2];\n\t"                   \
    "lop3.b32 c, e, 0x000FF000, %6, 0xEA;\n\t"          \
    "sub.f32 c, c, 0f4B080000;\n\t"                    \
    "fma.rn.f32 %3, c, %4, %3;\n\t}"
#else
#define RB_PTX_FIELDS                                  \
    "shr.u32 f, e, 20;\n\t"                            \
    "bfe.u32 b, e, 8, 12;\n\t"                         \
    "shr.u32 hi, %0, 12;\n\t"                          \
    "mad.lo.u32 %0, f, hi, b;\n\t"                     \
    "setp.lt.u32 p, %0, 65536;\n\t"                    \
    "@p prmt.b32 %0, %1, %0, 0x5410;\n\t"              \
    "@p add.u32 %2, %2, 2;\n\t"                        \
    "@p ld.shared.u16 %1, [%2];\n\t"                   \
    "prmt.b32 c, e, 0x4B000000, 0x7540;\n\t"           \
    "sub.f32 c, c, 0f4B000080;\n\t"                    \
    "fma.rn.f32 %3, c, %4, %3;\n\t}"
#endif
// magic: 0x4B000000 in a register (the code value is then one LOP3 with a
// single immediate: (e & 0xff000) | magic).
__device__ __forceinline__ void sym_step_ptx(uint32_t& st, uint32_t& w, uint32_t& pw, float& acc, float xv,
                                             uint32_t tb, uint32_t magic) {
#if RB_TABCOPIES == 2
    // two lane-interleaved copies: tb is this lane's copy (table + 4 * (lane & 1))
    asm("{\n\t.reg .pred p;\n\t.reg .b32 e, f, b, hi, a, c;\n\t"
        "and.b32 a, %0, 4095;\n\t"
        "shl.b32 a, a, 3;\n\t"
        "add.u32 a, a, %5;\n\t"
        "ld.shared.u32 e, [a];\n\t" RB_PTX_FIELDS
        : "+r"(st), "+r"(w), "+r"(pw), "+f"(acc)
        : "f"(xv), "r"(tb), "r"(magic));
#elif RB_ALIGNTAB
    asm("{\n\t.reg .pred p;\n\t.reg .b32 e, f, b, hi, a, c;\n\t"
        "shl.b32 a, %0, 2;\n\t"
        "and.b32 a, a, 0x3FFC;\n\t"
        "or.b32 a, a, %5;\n\t"
        "ld.shared.u32 e, [a];\n\t" RB_PTX_FIELDS
        : "+r"(st), "+r"(w), "+r"(pw), "+f"(acc)
        : "f"(xv), "r"(tb), "r"(magic));
#else
    asm("{\n\t.reg .pred p;\n\t.reg .b32 e, f, b, hi, a, c;\n\t"
        "and.b32 a, %0, 4095;\n\t"
        "shl.b32 a, a, 2;\n\t"
        "add.u32 a, a, %5;\n\t"
        "ld.shared.u32 e, [a];\n\t" RB_PTX_FIELDS
        : "+r"(st), "+r"(w), "+r"(pw), "+f"(acc)
        : "f"(xv), "r"(tb), "r"(magic));
#endif
}

template <int R, int K, int NACC, int XM, bool STAGED>
__device__ __forceinline__ void decode_pass(const uint32_t (&pos)[K], const int (&xcol)[K], int kk,
                                            const MatDev& d, float (&acc)[NACC][R], int& bad) {
    using W = WordSrc<STAGED>;
    const SmemMap sm = smem_map(0);
    // a shuffle result: the compiler cannot fold it back into an immediate
    const uint32_t magic = __shfl_sync(0xffffffffu, 0x4B000000u, 0);
    const uint32_t* tab = sm.tab;
    const uint32_t tb = tab_lane_base(sm.tab_s);
    uint32_t st[K], w[K], p[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        p[j] = pos[j];
        st[j] = (W::at(d, p[j]) << 16) | W::at(d, p[j] + W::kStep);
        p[j] += 2 * W::kStep;
        w[j] = W::at(d, p[j]);
        // absolute shared address (offset from g_smem + its window address) for the PTX step
        if (STAGED && RB_INNER != 0) p[j] += static_cast<uint32_t>(__cvta_generic_to_shared(g_smem));
    }
    const int nk = d.nk;
    dep_wait<XM>();   // activations may come from the previous kernel (or phase)
    float xn[K];
    constexpr bool kPref = RB_XPREF || (XM & kXPref);
    if (kPref) load_xs<K, NACC, XM>(d, xcol, kk, 0, xn);
    for (int k = 0; k < nk; ++k) {
        float xv[K];
        if (kPref) {
#pragma unroll
            for (int j = 0; j < K; ++j) xv[j] = xn[j];
            if (k + 1 < nk) load_xs<K, NACC, XM>(d, xcol, kk, k + 1, xn);   // prefetch next k-step
        } else {
            load_xs<K, NACC, XM>(d, xcol, kk, k, xv);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int j = 0; j < K; ++j) {
                float& a = acc[NACC == 1 ? 0 : j][r];
                if (STAGED && RB_INNER != 0) {
                    sym_step_ptx(st[j], w[j], p[j], a, xv[j], tb, magic);
                    continue;
                }
                const uint32_t e = tab_entry(tab, st[j]);
                st[j] = entry_freq(e) * (st[j] >> kScaleBits) + entry_bias(e);
                if (st[j] < kRansL) {
                    st[j] = __byte_perm(w[j], st[j], 0x5410);
                    p[j] += W::kStep;
                    w[j] = W::at(d, p[j]);
                }
                a = fmaf(entry_code(e), xv[j], a);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < K; ++j)
        if (j < kk && st[j] != kRansL) ++bad;
}

// One-tile pass whose words do not fit the stage (large tiles: C of a few
// thousand columns): windowed staging.  Each lane copies the next window of
// its own stream -- kWinBytes from the 16-byte boundary at or below its read
// position -- into its 1/32 of the stage, decodes up to 120 symbols with the
// staged symbol step (at most one word per symbol, so the reads stay inside
// the window), and refills.  Copies stop at `limit` (words readable from
// d.words); words beyond the stream's end are never consumed.
constexpr int kWinBytes = kStageBytes / 32;   // per-lane window of a windowed pass
constexpr int kWinWords = kWinBytes / 2;

// Copies this lane's window: kWinBytes of d.words from the 16-byte boundary at
// or below word p (that chunk holds word p, so it lies on a page the buffer
// touches), nothing at or past byte `wend`.  Returns the shared address of
// word p in the window.
__device__ __forceinline__ uint32_t refill_window(const MatDev& d, uint8_t* wgen, uint32_t win, uint32_t p,
                                                  uintptr_t wend) {
    const uintptr_t b = reinterpret_cast<uintptr_t>(d.words) + 2ull * p;
    const uintptr_t a0 = b & ~uintptr_t(15);
#pragma unroll 4
    for (int c = 0; c < kWinBytes / 16; ++c) {
        const uintptr_t src = a0 + 16ull * c;
        if (src + 16 <= wend) {
            cp_async16(win + 16u * c, reinterpret_cast<const void*>(src));
        } else if (src < wend) {   // the buffer ends inside this chunk: word by word
            for (uintptr_t q = src; q < wend; q += 2)
                *reinterpret_cast<uint16_t*>(wgen + 16u * c + (q - src)) = __ldg(reinterpret_cast<const uint16_t*>(q));
        }
    }
    cp_async_commit();
    cp_async_wait_all();
    return win + static_cast<uint32_t>(b - a0);
}

template <int R, int XM>
__device__ __forceinline__ void decode_pass_windowed(uint32_t pos, const int (&xcol)[1], const MatDev& d,
                                                  float (&acc)[1][R], int& bad, uint16_t* stage, int lane,
                                                  uint64_t limit) {
    constexpr int kChunkK = (kWinWords - 8) / R;   // head <= 7 words, then <= 1 word per symbol
    static_assert(kChunkK >= 1, "stage too small for windowed staging");
    static_assert(RB_LAYOUT == 1 && (RB_ALIGNTAB || RB_TABCOPIES == 2), "windowed passes use the PTX symbol step");
    const SmemMap sm = smem_map(0);
    const uint32_t magic = __shfl_sync(0xffffffffu, 0x4B000000u, 0);
    const uint32_t tb = tab_lane_base(sm.tab_s);
    uint8_t* const wgen = reinterpret_cast<uint8_t*>(stage) + lane * kWinBytes;   // this lane's window
    const uint32_t win = static_cast<uint32_t>(__cvta_generic_to_shared(wgen));
    const uintptr_t wbase = reinterpret_cast<uintptr_t>(d.words);
    const uintptr_t wend = wbase + 2ull * limit;
    uint32_t st = (static_cast<uint32_t>(__ldg(d.words + pos)) << 16) | __ldg(d.words + pos + 1);
    uint32_t p = pos + 2;                       // index of the next unread word (held in w)
    uint32_t w = __ldg(d.words + p);
    const int nk = d.nk;
    dep_wait<XM>();   // activations may come from the previous kernel (or phase)
    for (int k0 = 0; k0 < nk; k0 += kChunkK) {
        const uint32_t pw0 = refill_window(d, wgen, win, p, wend);
        uint32_t pw = pw0;
        const int k1 = min(nk, k0 + kChunkK);
        for (int k = k0; k < k1; ++k) {
            float xv[1];
            load_xs<1, 1, XM>(d, xcol, 1, k, xv);
#pragma unroll
            for (int r = 0; r < R; ++r) sym_step_ptx(st, w, pw, acc[0][r], xv[0], tb, magic);
        }
        p += (pw - pw0) >> 1;
    }
    if (st != kRansL) ++bad;
}

// Sets up a pass over tiles [t0, t0+kk) (consecutive), staging when possible,
// and decodes it.  Streams j >= kk replay stream kk-1 with zero activation.
template <int R, int K, int NACC, int XM>
__device__ __forceinline__ void run_pass(const MatDev& d, const uint32_t*, uint16_t* stage,
                                         int64_t t0, int kk, const int (&xcol)[K],
                                         float (&acc)[NACC][R], int& bad, int lane) {
    const int64_t s0 = t0 * 32;
    const uint32_t w0 = d.offs[s0];
    const uint64_t w1 = span_end(d, s0 + 32ll * kk);
    uint32_t pos[K];
#pragma unroll
    for (int j = 0; j < K; ++j) pos[j] = d.offs[s0 + 32 * (j < kk ? j : kk - 1) + lane];
    if (kStageBytes > 0 && w1 != UINT64_MAX && staged_bytes(d, w0, w1) <= (uint64_t)kStageBytes) {
        const uint32_t head = stage_span(d, stage, w0, w1, lane);
        // byte offset of the stage inside the CTA's shared memory
        const uint32_t sbase = static_cast<uint32_t>(reinterpret_cast<uint8_t*>(stage) - g_smem);
#pragma unroll
        for (int j = 0; j < K; ++j) pos[j] = sbase + 2u * (pos[j] - w0 + head);
        decode_pass<R, K, NACC, XM, true>(pos, xcol, kk, d, acc, bad);
        __syncwarp();   // stage is rewritten by the next pass
    } else {
        const uint64_t limit = d.nwords >= 0 ? (uint64_t)d.nwords : (d.wlimit > 0 ? (uint64_t)d.wlimit : 0);
        if constexpr (K == 1 && NACC == 1 && kStageBytes >= 32 * 32) {
            if (limit > 0) {
                decode_pass_windowed<R, XM>(pos[0], xcol, d, acc, bad, stage, lane, limit);
                __syncwarp();   // stage is rewritten by the next pass
                return;
            }
        }
        decode_pass<R, K, NACC, XM, false>(pos, xcol, kk, d, acc, bad);
    }
}

// Fused output exchange of the row-sharded path: the row goes to every rank's
// output buffer (plain stores over NVLink; ypeer[] includes this rank's own
// buffer).  No fence here: the caller's cross-GPU barrier runs after this
// kernel in stream order, so these stores happen before its system-scope
// release, and a fence per row would stall every warp for an NVLink round trip.
__device__ __forceinline__ void store_peers(const MatDev& d, int row, float s) {
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p)
        if (p < d.npeer) d.ypeer[p][row] = s;
}

// Column mode: rows rb*R..rb*R+R-1, column blocks of segment `seg`.
template <int R>
__device__ __forceinline__ void colmode_epilogue(const MatDev& d, int rb, int seg, float s, int lane,
                                                 uint16_t* stage, int warp, int nactive);

template <int R, int K, int XM>
__device__ void colmode_item(const MatDev& d, int item, const uint32_t* tab, uint16_t* stage,
                             int lane, int& bad, int warp, int nactive) {
    const int rb = item / d.nseg;
    const int seg = item - rb * d.nseg;
    const int cb_begin = seg * d.cbs;
    const int cb_end = min(d.ncb, cb_begin + d.cbs);
    float acc[1][R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[0][r] = 0.f;
    for (int cb0 = cb_begin; cb0 < cb_end; cb0 += K) {
        const int kk = min(K, cb_end - cb0);
        int xcol[K];
#pragma unroll
        for (int j = 0; j < K; ++j) xcol[j] = (cb0 + (j < kk ? j : 0)) * d.C + lane;
        run_pass<R, K, 1, XM>(d, tab, stage, (int64_t)rb * d.ncb + cb0, kk, xcol, acc, bad, lane);
    }
    colmode_epilogue<R>(d, rb, seg, reduce_scatter<R>(acc[0], lane) * kInvCodeScale, lane, stage, warp, nactive);
}

// Output of one column-mode item: lane l holds the full 32-lane sum s of row
// rb*R + (l >> (5 - log2 R)).
template <int R>
__device__ __forceinline__ void colmode_epilogue(const MatDev& d, int rb, int seg, float s, int lane,
                                                 uint16_t* stage, int warp, int nactive) {
    constexpr int kShift = 5 - Log2<R>::value;
    const bool owner = (lane & ((1 << kShift) - 1)) == 0;
    const int r = lane >> kShift;
    if (d.combine) {
        // The row block's segments are warps warp-seg .. warp-seg+nseg-1 of
        // this CTA: each leaves its R sums in its own stage (free after its
        // passes), one named barrier over the CTA's nactive working warps
        // (each reaches it once), and the segment-0 warp adds them in
        // segment order (deterministic).  No global fence or atomic.
        if (owner) reinterpret_cast<float*>(stage)[r] = s;
        asm volatile("bar.sync 1, %0;\n" ::"r"(nactive * 32) : "memory");
        if (seg != 0) return;
        if (owner) {
            float t = 0.f;
            for (int g = 0; g < d.nseg; ++g) t += reinterpret_cast<const float*>(smem_map(warp + g).stage)[r];
            s = t;
        }
    } else if (d.nseg > 1 && d.partials != nullptr) {
        // Row block split over nseg warps: publish this segment's R sums, and
        // let the last warp to finish add all segments in segment order
        // (deterministic) and store y.  The counter is reset for the next launch.
        if (owner) d.partials[((int64_t)rb * d.nseg + seg) * R + r] = s;
        __threadfence();
        __syncwarp();
        uint32_t prev = 0;
        if (lane == 0) prev = atomicAdd(d.counters + rb, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != (uint32_t)d.nseg - 1) return;
        if (lane == 0) d.counters[rb] = 0u;
        __threadfence();
        if (owner) {
            const volatile float* part = d.partials + (int64_t)rb * d.nseg * R + r;
            float t = 0.f;
            for (int g = 0; g < d.nseg; ++g) t += part[(int64_t)g * R];
            s = t;
        }
    }
    if (owner) {
        const int row = rb * R + r;
        if (d.accumulate) atomicAdd(d.y + row, s);
        else if (d.npeer > 0) store_peers(d, row, s);
        else d.y[row] = s;
    }
}

// warp / nactive: this warp's index and the CTA's number of working warps
// (used only when d.combine is set: the step kernel, one item per warp).
template <int R, int XM>
__device__ __forceinline__ void process_item(const MatDev& d, int item, const uint32_t* tab,
                                             uint16_t* stage, int lane, int& bad, int warp, int nactive) {
    switch (d.kcol) {
        case 1: colmode_item<R, 1, XM>(d, item, tab, stage, lane, bad, warp, nactive); break;
        case 2: colmode_item<R, 2, XM>(d, item, tab, stage, lane, bad, warp, nactive); break;
        case 3: colmode_item<R, 3, XM>(d, item, tab, stage, lane, bad, warp, nactive); break;
        default: colmode_item<R, 4, XM>(d, item, tab, stage, lane, bad, warp, nactive); break;
    }
}

// ------------------------------------------------------------ kernels
// One matrix: CTA b handles items [b*kWarps, b*kWarps + kWarps).
template <int R, bool BF16X>
__global__ void __launch_bounds__(kThreads, RB_MINB) gemv_matrix_kernel(MatDev d) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const SmemMap sm = smem_map(warp);
    uint32_t* tab = sm.tab;
    uint16_t* stage = sm.stage;
    load_table(tab, d.table);
    __syncthreads();
    // grid-stride over items: the grid holds only as many CTAs as fit on the
    // GPU at once, so a large matrix has no half-empty last wave.  Items are
    // taken last-first: without a known buffer length (the reference entry
    // points pass none) the item holding the final stream cannot be staged
    // and is the slowest, so it starts in the first wave.
    int bad = 0;
    for (int i = blockIdx.x * kWarps + warp; i < d.nitems; i += gridDim.x * kWarps)
        process_item<R, BF16X ? kXBf16 : 0>(d, d.nitems - 1 - i, tab, stage, lane, bad, warp, 0);
}

// Tiles [t_begin, t_end) of a work item (consecutive in stream order).
__device__ __forceinline__ void item_tiles(const MatDev& d, int item, int64_t& t_begin, int64_t& t_end) {
    const int rb = item / d.nseg, seg = item - rb * d.nseg;
    t_begin = (int64_t)rb * d.ncb + seg * d.cbs;
    t_end = (int64_t)rb * d.ncb + min(d.ncb, seg * d.cbs + d.cbs);
}

// Activation prescale of a throughput step: out[c] = float(x_bf16[c]) * step[c]
// for every matrix with a bf16 input, into the workspace, so the step kernel
// loads one fp32 activation per column instead of a bf16 value, a step and a
// multiply (and keeps a third less of them in L1).  Same product, same fp32
// rounding as the fused path: results are unchanged.
struct PrescaleJob {
    const __nv_bfloat16* x;
    const float* step;
    float* out;
    int cols, pad_;
};

__global__ void __launch_bounds__(256) prescale_kernel(const PrescaleJob* __restrict__ jobs, int njobs) {
    // Let the step kernel start (table loads, staging) once every block of
    // this grid runs; it waits for this grid to complete before reading x'.
    if (RB_PDL) pdl_launch_dependents();
    pdl_wait();   // x may be the output of the previous kernel of the stream
    for (int j = blockIdx.x; j < njobs; j += gridDim.x) {
        const PrescaleJob jb = jobs[j];
        for (int c = threadIdx.x; c < jb.cols; c += blockDim.x)
            jb.out[c] = __bfloat162float(jb.x[c]) * jb.step[c];
    }
}

// Plan-time: the contiguous word range [x, y) of every chunk.
__global__ void fill_spans_kernel(const StepHeader* __restrict__ hdr, int R) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= hdr->nchunks) return;
    const MatDev* descs = reinterpret_cast<const MatDev*>(hdr + 1);
    const Chunk* chunks = reinterpret_cast<const Chunk*>(descs + hdr->ndesc);
    uint2* spans = reinterpret_cast<uint2*>(const_cast<uint8_t*>(reinterpret_cast<const uint8_t*>(hdr) + hdr->spans_off));
    const Chunk ch = chunks[c];
    const MatDev& d = descs[ch.desc];
    int64_t t0, t1, u0, u1;
    item_tiles(d, ch.item0, t0, t1);
    item_tiles(d, ch.item0 + ch.nitems - 1, u0, u1);
    const uint32_t w0 = d.offs[t0 * 32];
    const uint64_t w1 = span_end(d, u1 * 32);
    spans[c] = make_uint2(w0, w1 == UINT64_MAX ? w0 : static_cast<uint32_t>(w1));
}

// TMA bulk prefetch of [p, p + bytes) into L2, 16-byte aligned outward (each
// 16-byte block touched overlaps the range, so no page outside it is touched).
__device__ __forceinline__ void prefetch_l2(const void* p, uint64_t bytes) {
    uintptr_t a = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15);
    const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes + 15) & ~uintptr_t(15);
    for (; a < e; a += 65536) {
        const uint32_t n = static_cast<uint32_t>(e - a < 65536 ? e - a : 65536);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(a), "r"(n) : "memory");
    }
}

// Warm L2 for the chunk that starts about one wave after this CTA: its words,
// offsets and table, while this CTA loads its own.
__device__ __forceinline__ void prefetch_next_chunk(const StepHeader* hdr, const MatDev* descs, const Chunk* chunks) {
    const int nb = blockIdx.x + hdr->ahead;
    if (hdr->ahead <= 0 || nb >= hdr->nchunks) return;
    const uint2 sp = reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(hdr) + hdr->spans_off)[nb];
    const MatDev& dn = descs[chunks[nb].desc];
    if (sp.y > sp.x) prefetch_l2(dn.words + sp.x, 2ull * (sp.y - sp.x));
    prefetch_l2(dn.table, kProbM * 4);
}

// Every projection of a decoder step: CTA b processes chunk b (one matrix).
template <int R>
__global__ void __launch_bounds__(kThreads, RB_MINB) gemv_step_kernel(const StepHeader* __restrict__ hdr) {
    const MatDev* descs = reinterpret_cast<const MatDev*>(hdr + 1);
    const Chunk* chunks = reinterpret_cast<const Chunk*>(descs + hdr->ndesc);
    const Chunk ch = chunks[blockIdx.x];
    const MatDev& d = descs[ch.desc];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (RB_PDL) pdl_launch_dependents();
    if (RB_PREFETCH && threadIdx.x == kThreads - 1) prefetch_next_chunk(hdr, descs, chunks);
    const SmemMap sm = smem_map(warp);
    uint32_t* tab = sm.tab;
    uint16_t* stage = sm.stage;
    load_table(tab, d.table);
    __syncthreads();
    if (warp >= ch.nitems) return;
    int bad = 0;
    const MatDev dl = d;
    if (dl.step != nullptr) process_item<R, kXBf16>(dl, ch.item0 + warp, tab, stage, lane, bad, warp, ch.nitems);
    else process_item<R, 0>(dl, ch.item0 + warp, tab, stage, lane, bad, warp, ch.nitems);
}

// One symbol of a staged stream returning kCodeScale*code (no FMA): the
// decode-to-dense path.  Same sequence as sym_step_ptx.
__device__ __forceinline__ float sym_code(uint32_t& st, uint32_t& w, uint32_t& pw, uint32_t tb, const uint32_t* tab,
                                          bool staged, const MatDev& d, uint32_t magic) {
#if RB_LAYOUT == 1 && (RB_ALIGNTAB || RB_TABCOPIES == 2)
    if (staged) {
        float c;
        asm("{\n\t.reg .pred p;\n\t.reg .b32 e, f, b, hi, a, t;\n\t"
#if RB_TABCOPIES == 2
            "and.b32 a, %0, 4095;\n\t"
            "shl.b32 a, a, 3;\n\t"
            "add.u32 a, a, %4;\n\t"
#else
            "shl.b32 a, %0, 2;\n\t"
            "and.b32 a, a, 0x3FFC;\n\t"
            "or.b32 a, a, %4;\n\t"
#endif
            "ld.shared.u32 e, [a];\n\t"
            "shr.u32 f, e, 20;\n\t"
            "and.b32 b, e, 4095;\n\t"
            "shr.u32 hi, %0, 12;\n\t"
            "mad.lo.u32 %0, f, hi, b;\n\t"
            "setp.lt.u32 p, %0, 65536;\n\t"
            "@p prmt.b32 %0, %1, %0, 0x5410;\n\t"
            "@p add.u32 %2, %2, 2;\n\t"
            "@p ld.shared.u16 %1, [%2];\n\t"
            "lop3.b32 t, e, 0x000FF000, %5, 0xEA;\n\t"
            "sub.f32 %3, t, 0f4B080000;\n\t}"
            : "+r"(st), "+r"(w), "+r"(pw), "=f"(c)
            : "r"(tb), "r"(magic));
        return c;
    }
#endif
    const uint32_t e = tab_entry(tab, st);
    st = entry_freq(e) * (st >> kScaleBits) + entry_bias(e);
    if (st < kRansL) {
        st = __byte_perm(w, st, 0x5410);
        if (staged) {
            pw += 2;
            w = *reinterpret_cast<const uint16_t*>(g_smem + pw);
        } else {
            ++pw;
            w = __ldg(d.words + pw);
        }
    }
    return entry_code(e);
}

template <int R, int K, bool STAGED>
__device__ __forceinline__ void decode_store(const MatDev& d, const uint32_t (&pos)[K], int kk,
                                             __nv_bfloat16* const (&orow)[K], const int (&col0)[K]) {
    const SmemMap sm = smem_map(0);
    const bool ptx = STAGED && RB_LAYOUT == 1 && (RB_ALIGNTAB || RB_TABCOPIES == 2);
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(g_smem));
    uint32_t st[K], w[K], p[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        p[j] = pos[j];
        if (STAGED) {
            st[j] = (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(g_smem + p[j])) << 16) |
                    *reinterpret_cast<const uint16_t*>(g_smem + p[j] + 2);
            p[j] += 4;
            w[j] = *reinterpret_cast<const uint16_t*>(g_smem + p[j]);
            if (ptx) p[j] += sbase;
        } else {
            st[j] = (static_cast<uint32_t>(__ldg(d.words + p[j])) << 16) | __ldg(d.words + p[j] + 1);
            p[j] += 2;
            w[j] = __ldg(d.words + p[j]);
        }
    }
    const uint32_t magic = __shfl_sync(0xffffffffu, 0x4B000000u, 0);   // kept in a register
    // element offsets of the tile's rows (R x cols < 2^32 elements: checked by the launcher)
    uint32_t roff[R];
#pragma unroll
    for (int r = 0; r < R; ++r) roff[r] = (uint32_t)r * (uint32_t)d.cols;
    for (int k = 0; k < d.nk; ++k) {
        float sv[K];
        __nv_bfloat16* o[K];
#pragma unroll
        for (int j = 0; j < K; ++j) {
            sv[j] = __ldg(d.step + col0[j] + 32 * k) * kInvCodeScale;
            o[j] = orow[j] + 32 * k;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int j = 0; j < K; ++j) {
                float c;
                if (ptx) {
                    c = sym_code(st[j], w[j], p[j], tab_lane_base(sm.tab_s), sm.tab, true, d, magic);
                } else {
                    // generic pointer bookkeeping of the C++ step uses offsets from g_smem
                    c = sym_code(st[j], w[j], p[j], tab_lane_base(sm.tab_s), sm.tab, STAGED, d, magic);
                }
                // no branch on j < kk: a slot past kk replays tile kk-1 and
                // stores the same values to the same place
                o[j][roff[r]] = __float2bfloat16(c * sv[j]);
            }
        }
    }
}

// Decode-only: K consecutive tiles per warp, bf16(code * step) into a dense
// row-major matrix (the "decompress, then cuBLAS" comparator).  Same staging
// and symbol step as the fused GEMV; each symbol becomes one 2-byte store,
// coalesced across the warp (64 B per row segment).
// decode_store for one tile whose words do not fit the stage: per-lane
// windows as in decode_pass_windowed.
template <int R>
__device__ __forceinline__ void decode_store_windowed(const MatDev& d, uint32_t pos, __nv_bfloat16* orow,
                                                      int col0, uint16_t* stage, int lane, uint64_t limit) {
    constexpr int kChunkK = (kWinWords - 8) / R;
    static_assert(RB_LAYOUT == 1 && (RB_ALIGNTAB || RB_TABCOPIES == 2), "windowed passes use the PTX symbol step");
    const SmemMap sm = smem_map(0);
    const uint32_t magic = __shfl_sync(0xffffffffu, 0x4B000000u, 0);
    uint8_t* const wgen = reinterpret_cast<uint8_t*>(stage) + lane * kWinBytes;
    const uint32_t win = static_cast<uint32_t>(__cvta_generic_to_shared(wgen));
    const uintptr_t wend = reinterpret_cast<uintptr_t>(d.words) + 2ull * limit;
    uint32_t st = (static_cast<uint32_t>(__ldg(d.words + pos)) << 16) | __ldg(d.words + pos + 1);
    uint32_t p = pos + 2;
    uint32_t w = __ldg(d.words + p);
    uint32_t roff[R];
#pragma unroll
    for (int r = 0; r < R; ++r) roff[r] = (uint32_t)r * (uint32_t)d.cols;
    const int nk = d.nk;
    for (int k0 = 0; k0 < nk; k0 += kChunkK) {
        const uint32_t pw0 = refill_window(d, wgen, win, p, wend);
        uint32_t pw = pw0;
        const int k1 = min(nk, k0 + kChunkK);
        for (int k = k0; k < k1; ++k) {
            const float sv = __ldg(d.step + col0 + 32 * k) * kInvCodeScale;
            __nv_bfloat16* o = orow + 32 * k;
#pragma unroll
            for (int r = 0; r < R; ++r)
                o[roff[r]] = __float2bfloat16(sym_code(st, w, pw, tab_lane_base(sm.tab_s), sm.tab, true, d, magic) * sv);
        }
        p += (pw - pw0) >> 1;
    }
}

template <int R, int K>
__device__ __forceinline__ void decode_tiles(const MatDev& d, const SmemMap& sm, __nv_bfloat16* __restrict__ out,
                                             int64_t ntiles, int64_t t0, int lane) {
    const int kk = ntiles - t0 < K ? (int)(ntiles - t0) : K;
    const int64_t s0 = t0 * 32;
    const uint32_t w0 = d.offs[s0];
    const uint64_t w1 = span_end(d, s0 + 32ll * kk);
    uint32_t pos[K];
    __nv_bfloat16* orow[K];
    int col0[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        const int jj = j < kk ? j : kk - 1;
        pos[j] = d.offs[s0 + 32 * jj + lane];
        const int64_t t = t0 + jj;
        const int rb = (int)(t / d.ncb), cb = (int)(t % d.ncb);
        col0[j] = cb * d.C + lane;
        orow[j] = out + (int64_t)rb * R * d.cols + col0[j];
    }
    if (kStageBytes > 0 && w1 != UINT64_MAX && staged_bytes(d, w0, w1) <= (uint64_t)kStageBytes) {
        const uint32_t head = stage_span(d, sm.stage, w0, w1, lane);
        const uint32_t soff = static_cast<uint32_t>(reinterpret_cast<uint8_t*>(sm.stage) - g_smem);
#pragma unroll
        for (int j = 0; j < K; ++j) pos[j] = soff + 2u * (pos[j] - w0 + head);
        decode_store<R, K, true>(d, pos, kk, orow, col0);
    } else {
        if constexpr (K == 1 && kStageBytes >= 32 * 32) {
            const uint64_t limit = d.nwords >= 0 ? (uint64_t)d.nwords : (d.wlimit > 0 ? (uint64_t)d.wlimit : 0);
            if (limit > 0) {
                decode_store_windowed<R>(d, pos[0], orow[0], col0[0], sm.stage, lane, limit);
                return;
            }
        }
        decode_store<R, K, false>(d, pos, kk, orow, col0);
    }
}

// Grid-stride over groups of K tiles, last group first (it holds the final
// stream, unstaged when the buffer length is unknown); the grid holds only
// resident CTAs.
template <int R, int K>
__global__ void __launch_bounds__(kThreads, RB_MINB) decode_kernel(MatDev d, __nv_bfloat16* __restrict__ out,
                                                                   int64_t ntiles) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const SmemMap sm = smem_map(warp);
    load_table(sm.tab, d.table);
    __syncthreads();
    const int64_t ngroups = (ntiles + K - 1) / K;
    for (int64_t g = (int64_t)blockIdx.x * kWarps + warp; g < ngroups; g += (int64_t)gridDim.x * kWarps) {
        decode_tiles<R, K>(d, sm, out, ntiles, (ngroups - 1 - g) * K, lane);
        __syncwarp();   // every lane is done with this span before the stage is refilled
    }
}

// Fixed-rate int4 baseline.  A warp owns kInt4Rows consecutive rows: lane l
// reads the 8-code words g = l, l+32, ... of every row (32-bit loads, 128 B
// per warp and row, coalesced) and the 8 activations of group g once for all
// its rows.  Nibble b of a word becomes an exact float with one LOP3 and one
// FADD, without a shift: (q & 0xF << 4b) | 0x4B000000 is the float
// 2^23 + n * 16^b (exact while the nibble stays below bit 23, b <= 4), and
// subtracting 2^23 + 8 * 16^b leaves (n - 8) * 16^b; the activation of that
// column is pre-multiplied by 16^-b (a power of two: exact), once per group
// for all rows.  Nibbles 5..7 use q >> 20 the same way (b = 0..2).  The
// kInt4Rows partial sums are transpose-reduced.
template <int kInt4Rows>
__global__ void __launch_bounds__(256) int4_gemv_kernel(const uint32_t* __restrict__ w,
                                                        const float4* __restrict__ x,
                                                        float* __restrict__ y, int rows, int cols) {
    const int lane = threadIdx.x & 31;
    const int ngroup = cols / 8;
    // per nibble position: scale of the activation
    constexpr float kScale[8] = {1.f, 0.0625f, 0.00390625f, 0.000244140625f, 1.52587890625e-05f,
                                 1.f, 0.0625f, 0.00390625f};
    const uint32_t magic = __shfl_sync(0xffffffffu, 0x4B000000u, 0);   // kept in a register
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    // grid-stride over groups of kInt4Rows rows: the grid holds only resident CTAs
    for (int row0 = ((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * kInt4Rows; row0 < rows;
         row0 += nwarps * kInt4Rows) {
        const uint32_t* wr[kInt4Rows];
#pragma unroll
        for (int r = 0; r < kInt4Rows; ++r)
            wr[r] = w + (int64_t)min(row0 + r, rows - 1) * ngroup;   // rows past the end repeat the last
        float acc[kInt4Rows];
#pragma unroll
        for (int r = 0; r < kInt4Rows; ++r) acc[r] = 0.f;
#pragma unroll kI4Unroll
        for (int g = lane; g < ngroup; g += 32) {
            const float4 x0 = __ldg(x + 2 * g);
            const float4 x1 = __ldg(x + 2 * g + 1);
            const float xv[8] = {x0.x * kScale[0], x0.y * kScale[1], x0.z * kScale[2], x0.w * kScale[3],
                                 x1.x * kScale[4], x1.y * kScale[5], x1.z * kScale[6], x1.w * kScale[7]};
            uint32_t q[kInt4Rows];
#pragma unroll
            for (int r = 0; r < kInt4Rows; ++r) q[r] = __ldg(wr[r] + g);
#pragma unroll
            for (int r = 0; r < kInt4Rows; ++r) {
                const uint32_t qh = q[r] >> 20;
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    const int sh = b < 5 ? b : b - 5;
                    const uint32_t src = b < 5 ? q[r] : qh;
                    uint32_t bits;   // (src & 0xF << 4sh) | magic: one LOP3
                    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(bits) : "r"(src), "r"(0xFu << (4 * sh)), "r"(magic));
                    const float off = 8388608.0f + 8.0f * static_cast<float>(1u << (4 * sh));
                    acc[r] = fmaf(__int_as_float(bits) - off, xv[b], acc[r]);
                }
            }
        }
        const float s = reduce_scatter<kInt4Rows>(acc, lane);
        constexpr int kShift = 5 - Log2<kInt4Rows>::value;
        const int r = lane >> kShift;
        if ((lane & ((1 << kShift) - 1)) == 0 && row0 + r < rows) y[row0 + r] = s;
    }
}

// ------------------------------------------------------------ host side
static bool valid_R(int R) { return R == 1 || R == 2 || R == 4 || R == 8 || R == 16; }


static int sm_count() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

// Most symbols one staged pass should hold: 90% of the stage at the matrix's
// mean size per symbol (state words included) when the buffer length is
// known, else a bound for up to ~5.3 bits/symbol.  A pass whose span still
// does not fit is decoded from global memory (same results, slower).
static int64_t pass_symbols(const MatDev& d) {
    if (kStageBytes <= 0) return 12288;
    if (d.nwords > 0 && d.rows > 0 && d.cols > 0) {
        const double bytes_per_symbol = 2.0 * (double)d.nwords / ((double)d.rows * (double)d.cols);
        return std::max<int64_t>(1, (int64_t)(0.9 * kStageBytes / bytes_per_symbol));
    }
    return (int64_t)kStageBytes * 3 / 2;
}

// Fills the work decomposition of d.  `split_for` > 0 is the number of warps
// resident at once and allows column blocks to be split across warps
// (accumulating into y) where that shortens the launch.
static void plan_matrix(MatDev& d, int R, int split_for, int kcap = 4) {
    d.ncb = d.cols / d.C;
    d.nrb = d.rows / R;
    d.nk = d.C / 32;
    d.tail_words = 2 + R * d.nk;
    d.accumulate = 0;
    // Every matrix is decoded in column mode, a matrix of one column block
    // (cols == C) included: K = 1, one tile per pass.  (Decoding several row
    // blocks of such a matrix as interleaved streams of one pass measured 1.5
    // to 3.5 times slower on B200: larger spans that fall out of the stage,
    // a 32-value reduction and activations reloaded per stream.)
    // K that divides ncb (no idle stream slots), preferring more streams per
    // lane, with at most pass_symbols(d) symbols per pass so that the pass's
    // words fit the stage.
    const int kmax = (int)std::max<int64_t>(1, std::min<int64_t>(kcap, pass_symbols(d) / ((int64_t)R * d.C)));
    int k = 1;
    for (int c = kmax; c >= 2; --c)
        if (d.ncb % c == 0) { k = c; break; }
    if (k == 1 && kmax >= 2 && d.ncb > 1) {
        // no divisor: accept idle stream slots in the last pass only when they
        // are at most 1/8 of all slots (K = 2 over 3 tiles wastes 1/4: slower)
        for (int c = std::min(kmax, d.ncb); c >= 2; --c) {
            const int passes = (d.ncb + c - 1) / c;
            if ((passes * c - d.ncb) * 8 <= passes * c) { k = c; break; }
        }
    }
    // A small matrix that may be split is latency-bound: one tile per warp
    // gives the most independent warps (the serial chain of one stream is the
    // floor either way).
    if (split_for > 0 && (int64_t)d.nrb * d.ncb <= split_for) k = 1;
    d.kcol = k;
    const int passes = (d.ncb + k - 1) / k;
    // Segments per row block (equal: a divisor of passes), chosen for the
    // shortest makespan when split_for warps run at once: waves of items times
    // passes per item, plus a small per-item cost (setup, reduction, atomics)
    // of 1/20 pass.  Few row blocks -> many segments so every warp has work;
    // many row blocks -> segments still shrink the last, partly idle wave.
    int nseg = 1;
    if (split_for > 0) {
        int64_t best = INT64_MAX;
        for (int s = 1; s <= passes; ++s) {
            if (passes % s) continue;
            const int64_t waves = ((int64_t)d.nrb * s + split_for - 1) / split_for;
            const int64_t cost = waves * (20ll * (passes / s) + 1);
            if (cost < best) { best = cost; nseg = s; }
        }
    }
    d.nseg = nseg;
    d.cbs = (passes / nseg) * k;
    d.nitems = d.nrb * nseg;
    d.accumulate = nseg > 1 ? 1 : 0;
}

// The dynamic shared-memory opt-in is per function and per device; remember
// which (function, device) pairs are done.
static bool set_smem_attr(const void* fn, unsigned long long* done_mask) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    const unsigned long long bit = 1ull << (dev & 63);
    if (__atomic_load_n(done_mask, __ATOMIC_ACQUIRE) & bit) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
        return false;
    __atomic_fetch_or(done_mask, bit, __ATOMIC_ACQ_REL);
    return true;
}

// CTAs of `fn` (threads per CTA, dynamic shared bytes) resident at once on
// the current device; cached per device in `cache` (0 = not yet asked).
static int resident_blocks_any(const void* fn, int threads, size_t smem, int* cache) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 1;
    int* slot = &cache[dev & 63];
    int v = __atomic_load_n(slot, __ATOMIC_ACQUIRE);
    if (v > 0) return v;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    v = per_sm * sm_count();
    __atomic_store_n(slot, v, __ATOMIC_RELEASE);
    return v;
}

// CTAs of `fn` (kThreads threads, kSmemBytes shared) resident at once on the
// current device; cached per device in `cache` (0 = not yet asked).
static int resident_blocks(const void* fn, int* cache) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 1;
    int* slot = &cache[dev & 63];
    int v = __atomic_load_n(slot, __ATOMIC_ACQUIRE);
    if (v > 0) return v;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, kSmemBytes) != cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    v = per_sm * sm_count();
    __atomic_store_n(slot, v, __ATOMIC_RELEASE);
    return v;
}

template <int R>
static int launch_matrix(const MatDev& d, bool bf16x, cudaStream_t stream) {
    int grid = (d.nitems + kWarps - 1) / kWarps;
    if (grid == 0) return 0;
    const void* fn = bf16x ? (const void*)gemv_matrix_kernel<R, true> : (const void*)gemv_matrix_kernel<R, false>;
    static unsigned long long done[2] = {0, 0};
    static int resident[2][64] = {};
    set_smem_attr(fn, &done[bf16x ? 1 : 0]);
    grid = std::min(grid, resident_blocks(fn, resident[bf16x ? 1 : 0]));
    if (bf16x) gemv_matrix_kernel<R, true><<<grid, kThreads, kSmemBytes, stream>>>(d);
    else gemv_matrix_kernel<R, false><<<grid, kThreads, kSmemBytes, stream>>>(d);
    return (int)cudaGetLastError();
}

static int dispatch_matrix(int R, const MatDev& d, bool bf16x, cudaStream_t stream) {
    switch (R) {
        case 1: return launch_matrix<1>(d, bf16x, stream);
        case 2: return launch_matrix<2>(d, bf16x, stream);
        case 4: return launch_matrix<4>(d, bf16x, stream);
        case 8: return launch_matrix<8>(d, bf16x, stream);
        case 16: return launch_matrix<16>(d, bf16x, stream);
        default: return -1;
    }
}

static bool shape_ok(int R, int rows, int cols, int C) {
    return rows > 0 && cols > 0 && C > 0 && C % 32 == 0 && cols % C == 0 && rows % R == 0;
}

// Words readable from `words` to the end of the mapped device memory region
// holding it (cuMemGetAddressRange, reached through the runtime's driver entry
// point so there is no link to libcuda), 0 when the driver does not know the
// pointer.
static int64_t readable_words(const void* words) {
    static const PFN_cuMemGetAddressRange_v3020 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<PFN_cuMemGetAddressRange_v3020>(nullptr);
        return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
    }();
    if (fn == nullptr || words == nullptr) return 0;
    CUdeviceptr base = 0;
    size_t size = 0;
    const CUdeviceptr w = reinterpret_cast<CUdeviceptr>(words);
    if (fn(&base, &size, w) != CUDA_SUCCESS || w < base || w >= base + size) return 0;
    return static_cast<int64_t>((base + size - w) / 2);
}

static MatDev make_desc(const void* words, const void* offs, const void* table, const void* x,
                        const void* step, void* y, int rows, int cols, int C, int64_t nwords) {
    MatDev d;
    std::memset(&d, 0, sizeof(d));
    d.words = static_cast<const uint16_t*>(words);
    d.offs = static_cast<const uint32_t*>(offs);
    d.table = static_cast<const uint32_t*>(table);
    d.x = x;
    d.step = static_cast<const float*>(step);
    d.y = static_cast<float*>(y);
    d.nwords = nwords;
    d.wlimit = nwords < 0 ? readable_words(words) : 0;
    d.rows = rows;
    d.cols = cols;
    d.C = C;
    return d;
}

// Enough warps to occupy the GPU for single-matrix launches.
static int split_target() { return sm_count() * 16; }

}  // namespace rb200

using namespace rb200;

extern "C" int launch_rans_gemv(int R, const void* words, const void* offs, const void* table,
                                const void* x, void* y, int rows, int cols, int C,
                                cudaStream_t stream) {
    if (!valid_R(R)) return -1;
    if (!shape_ok(R, rows, cols, C)) return -2;
    MatDev d = make_desc(words, offs, table, x, nullptr, y, rows, cols, C, -1);
    // the caller zero-fills y when cols != C (reference contract), so column
    // blocks may be split across warps and accumulated
    plan_matrix(d, R, cols != C ? split_target() : 0);
    return dispatch_matrix(R, d, false, stream);
}

extern "C" int rans_gemv_bf16(int R, const void* words, const void* offs, const void* table,
                              const void* x_bf16, const void* step, void* y, int rows, int cols,
                              int C, int64_t nwords, cudaStream_t stream) {
    if (!valid_R(R)) return -1;
    if (!shape_ok(R, rows, cols, C) || step == nullptr) return -2;
    MatDev d = make_desc(words, offs, table, x_bf16, step, y, rows, cols, C, nwords);
    plan_matrix(d, R, 0);   // whole row blocks per warp: y is stored, no atomics
    {
        // Splitting the column blocks of a row block across warps (and
        // accumulating into a zeroed y) pays when whole rows give too few
        // warps (e.g. a 1536 x 8960 down projection), or when it shortens the
        // launch by 10% or more: makespan = waves of items x column blocks
        // per item, with split_target() warps per wave.
        const int64_t W = split_target();
        MatDev s = d;
        plan_matrix(s, R, (int)W);
        const bool few = (int64_t)d.nitems * (d.ncb / d.kcol) <= W;
        const int64_t span_whole = (d.nitems + W - 1) / W * d.cbs;
        const int64_t span_split = (s.nitems + W - 1) / W * s.cbs;
        if (few || span_split * 10 < span_whole * 9) {
            d = s;
            if (d.accumulate) {
                const cudaError_t e = cudaMemsetAsync(y, 0, sizeof(float) * (size_t)rows, stream);
                if (e != cudaSuccess) return (int)e;
            }
        }
    }
    return dispatch_matrix(R, d, true, stream);
}

template <int R, int K>
static int launch_decode_t(const MatDev& d, void* out, cudaStream_t stream) {
    const int64_t ntiles = (int64_t)d.nrb * d.ncb;
    const int64_t warps = (ntiles + K - 1) / K;
    int64_t grid = (warps + kWarps - 1) / kWarps;
    if (grid == 0) return 0;
    static unsigned long long done = 0;
    static int resident[64] = {};
    set_smem_attr((const void*)decode_kernel<R, K>, &done);
    grid = std::min<int64_t>(grid, resident_blocks((const void*)decode_kernel<R, K>, resident));
    decode_kernel<R, K><<<grid, kThreads, kSmemBytes, stream>>>(d, static_cast<__nv_bfloat16*>(out), ntiles);
    return (int)cudaGetLastError();
}

template <int R>
static int launch_decode_k(const MatDev& d, void* out, int k, cudaStream_t stream) {
    switch (k) {
        case 4: return launch_decode_t<R, 4>(d, out, stream);
        case 3: return launch_decode_t<R, 3>(d, out, stream);
        case 2: return launch_decode_t<R, 2>(d, out, stream);
        default: return launch_decode_t<R, 1>(d, out, stream);
    }
}

extern "C" int launch_rans_decode(int R, const void* words, const void* offs, const void* table,
                                  const void* step, void* out, int rows, int cols, int C,
                                  cudaStream_t stream) {
    if (!valid_R(R)) return -1;
    if (!shape_ok(R, rows, cols, C)) return -2;
    if ((int64_t)R * cols >= (int64_t(1) << 32)) return -2;   // row offsets of a tile are 32-bit
    MatDev d = make_desc(words, offs, table, nullptr, step, nullptr, rows, cols, C, -1);
    d.ncb = cols / C;
    d.nrb = rows / R;
    d.nk = C / 32;
    d.tail_words = 2 + R * d.nk;
    // tiles per warp pass: as many as the stage holds (1..4), while the
    // matrix still gives two waves of warps (small matrices: at most 2)
    const int64_t ntiles = (int64_t)d.nrb * d.ncb;
    int64_t k = std::min<int64_t>(4, std::max<int64_t>(1, pass_symbols(d) / ((int64_t)R * C)));
    while (k > 2 && ntiles / k < 2 * (int64_t)split_target()) --k;
    switch (R) {
        case 1: return launch_decode_k<1>(d, out, (int)k, stream);
        case 2: return launch_decode_k<2>(d, out, (int)k, stream);
        case 4: return launch_decode_k<4>(d, out, (int)k, stream);
        case 8: return launch_decode_k<8>(d, out, (int)k, stream);
        case 16: return launch_decode_k<16>(d, out, (int)k, stream);
        default: return -1;
    }
}

extern "C" int launch_int4_gemv(const void* w, const void* x, void* y, int rows, int cols,
                                cudaStream_t stream) {
    if (rows <= 0 || cols <= 0 || cols % 32) return -2;
    const int threads = 256;
    // rows per warp: 4 (each activation load serves 4 rows) while that still
    // keeps a quarter of the resident warps busy, else 2, else 1 (few rows,
    // many columns).  Measured on the BASELINE shapes: 8 rows per warp or
    // one-row warps on tall matrices are up to 1.8x slower.
    static int resident[64] = {};
    const int64_t slots = (int64_t)resident_blocks_any((const void*)int4_gemv_kernel<4>, threads, 0, resident) *
                          (threads / 32);
    int rw = rows / 4 >= slots / 4 ? 4 : rows / 2 >= slots / 4 ? 2 : 1;
    const int64_t warps = (rows + rw - 1) / rw;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    const int grid = (int)std::min<int64_t>(blocks, std::max<int64_t>(1, slots / (threads / 32)));
    const uint32_t* wq = static_cast<const uint32_t*>(w);
    const float4* xv = static_cast<const float4*>(x);
    float* yv = static_cast<float*>(y);
    switch (rw) {
        case 4: int4_gemv_kernel<4><<<grid, threads, 0, stream>>>(wq, xv, yv, rows, cols); break;
        case 2: int4_gemv_kernel<2><<<grid, threads, 0, stream>>>(wq, xv, yv, rows, cols); break;
        default: int4_gemv_kernel<1><<<grid, threads, 0, stream>>>(wq, xv, yv, rows, cols); break;
    }
    return (int)cudaGetLastError();
}

// ------------------------------------------------------------ step launcher
static size_t step_bytes(int ndesc, int64_t nchunks) {
    return sizeof(StepHeader) + sizeof(MatDev) * (size_t)ndesc + sizeof(Chunk) * (size_t)nchunks;
}

static int64_t count_chunks(const RansGemvDesc* descs, int n, int R, std::vector<MatDev>* out, int kcap = 4) {
    int64_t nchunks = 0;
    for (int i = 0; i < n; ++i) {
        const RansGemvDesc& s = descs[i];
        if (!shape_ok(R, s.rows, s.cols, s.C)) return -1;
        MatDev d = make_desc(s.words, s.offs, s.table, s.x, s.step, s.y, s.rows, s.cols, s.C, s.nwords);
        plan_matrix(d, R, 0, kcap);
        nchunks += (d.nitems + kWarps - 1) / kWarps;
        if (out) out->push_back(d);
    }
    return nchunks;
}

// Work plan of a step launch: decomposition of every matrix plus the
// workspace layout [header][MatDev x n][Chunk x nchunks][counters][partials].
// A launch with few whole-row items (a small phase of a decoder step: q/k/v,
// o, down) leaves most SMs idle and is bound by a few long serial chains, so
// its column-mode matrices are split to one tile per warp; the segments of a
// row block meet in `partials` and the last-arriving warp stores y.
struct StepLayout {
    std::vector<MatDev> mats;
    int64_t nchunks = 0;
    int njobs = 0;             // activation prescale jobs (throughput plans with bf16 x)
    size_t jobs_off = 0, counters_off = 0, partials_off = 0, spans_off = 0, xprime_off = 0, bytes = 0;
    std::vector<size_t> xprime;   // per matrix: byte offset of its x' (0 = none)
};

static size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

// Items per CTA of the step kernel: 8, or whole row blocks when the segments
// of a row block add up in shared memory.
static int chunk_items(const MatDev& d) { return d.combine ? (kWarps / d.nseg) * d.nseg : kWarps; }

// Work decomposition of a group of matrices that run together -- one step
// launch, or one phase of a chain -- starting from plan_matrix(d, R, 0):
// latency-bound groups are split into segments, groups of a few waves cut
// into row segments.  Adds the segment counters and partials the group needs;
// returns true when the group was planned as latency-bound (split).
static bool plan_group(std::vector<MatDev>& mats, int R, int64_t& ncounters, int64_t& npartials, int kcap = 4) {
    int64_t items = 0;
    for (const MatDev& d : mats) items += d.nitems;
    const bool split = items * 2 < split_target();
    if (split) {
        // Split column-mode matrices into segments of T consecutive tiles,
        // decoded as T interleaved streams in one pass.  Start from T = 1 (the
        // most warps) and, while the launch has more items than warps resident
        // at once, coarsen the matrix with the most items to its next T that
        // divides ncb (T <= 4): a second, mostly idle wave would cost a whole
        // serial chain, more T costs only interleaving.
        const int64_t W = split_target();
        std::vector<int> T(mats.size(), 0);
        int64_t total = 0;
        for (size_t i = 0; i < mats.size(); ++i) {
            const MatDev& d = mats[i];
            if (d.ncb > 1) T[i] = 1;
            total += T[i] ? (int64_t)d.nrb * d.ncb : d.nitems;
        }
        auto next_t = [&](size_t i) {
            const MatDev& d = mats[i];
            for (int t = T[i] + 1; t <= kcap && (int64_t)t * R * d.C <= pass_symbols(d); ++t)
                if (d.ncb % t == 0) return t;
            return 0;
        };
        while (total > W) {
            size_t best = SIZE_MAX;
            int64_t best_items = 0;
            for (size_t i = 0; i < mats.size(); ++i) {
                if (!T[i] || !next_t(i)) continue;
                const int64_t it = (int64_t)mats[i].nrb * (mats[i].ncb / T[i]);
                if (it > best_items) { best_items = it; best = i; }
            }
            if (best == SIZE_MAX) break;
            const int t = next_t(best);
            total -= best_items - (int64_t)mats[best].nrb * (mats[best].ncb / t);
            T[best] = t;
        }
        for (size_t i = 0; i < mats.size(); ++i) {
            if (!T[i]) continue;
            MatDev& d = mats[i];
            d.kcol = T[i];
            d.nseg = d.ncb / T[i];
            d.cbs = T[i];
            d.nitems = d.nrb * d.nseg;
            d.accumulate = 0;
            // a launch this short is latency-bound: segments of a row block
            // meet in shared memory when they fit one CTA (idle warps cost
            // nothing here), else in global partials
            d.combine = d.nseg > 1 && d.nseg <= kWarps ? 1 : 0;
            if (d.nseg > 1 && !d.combine) {
                ncounters += d.nrb;
                npartials += (int64_t)d.nrb * d.nseg * R;
            }
        }
    } else if (items < 16 * (int64_t)split_target()) {
        // A launch of a few waves of whole-row items loses up to one wave to
        // quantisation (e.g. 3.03 waves run as 4).  Give each column-mode
        // matrix a share of the resident warps in proportion to its items and
        // let the makespan model of plan_matrix cut its rows into equal
        // segments of passes (same K); segments meet in `partials`, as above.
        const int64_t W = split_target();
        for (MatDev& d : mats) {
            if (d.ncb <= d.kcol) continue;
            const int share = (int)std::max<int64_t>(1, W * d.nitems / items);
            MatDev sp = d;
            plan_matrix(sp, R, share, kcap);
            if (sp.nseg <= 1 || sp.kcol != d.kcol) continue;
            d = sp;
            d.accumulate = 0;
            // segments meet in shared memory when whole row blocks fill a CTA
            // exactly (no idle warps), else in global partials
            d.combine = kWarps % d.nseg == 0 ? 1 : 0;
            if (!d.combine) {
                ncounters += d.nrb;
                npartials += (int64_t)d.nrb * d.nseg * R;
            }
        }
    }
    return split;
}

static int layout_step(const RansGemvDesc* descs, int n, int R, StepLayout& L) {
    L.mats.clear();
    if (count_chunks(descs, n, R, &L.mats) < 0) return -2;
    int64_t ncounters = 0, npartials = 0;
    const bool split = plan_group(L.mats, R, ncounters, npartials);
    L.nchunks = 0;
    for (MatDev& d : L.mats) L.nchunks += (d.nitems + chunk_items(d) - 1) / chunk_items(d);
    // Launches of two or more waves of items read activations through a
    // prescaled fp32 copy (5% faster on a whole decoder step); shorter ones
    // skip the extra kernel, which would cost more than it saves.
    int64_t planned_items = 0;
    for (const MatDev& d : L.mats) planned_items += d.nitems;
    L.njobs = 0;
    L.xprime.assign(L.mats.size(), 0);
    if (!split && planned_items >= 2 * (int64_t)split_target())
        for (const MatDev& d : L.mats)
            if (d.step != nullptr) ++L.njobs;
    L.jobs_off = align16(step_bytes(n, L.nchunks));
    L.counters_off = align16(L.jobs_off + sizeof(PrescaleJob) * (size_t)L.njobs);
    L.partials_off = align16(L.counters_off + sizeof(uint32_t) * (size_t)ncounters);
    L.spans_off = align16(L.partials_off + sizeof(float) * (size_t)npartials);
    L.xprime_off = align16(L.spans_off + sizeof(uint2) * (size_t)L.nchunks);
    size_t off = L.xprime_off;
    if (L.njobs > 0)
        for (size_t i = 0; i < L.mats.size(); ++i)
            if (L.mats[i].step != nullptr) {
                L.xprime[i] = off;
                off = align16(off + sizeof(float) * (size_t)L.mats[i].cols);
            }
    L.bytes = off;
    return 0;
}

extern "C" int64_t rans_gemv_step_workspace_bytes(const RansGemvDesc* descs, int n, int R) {
    if (!valid_R(R) || n <= 0) return -1;
    StepLayout L;
    if (layout_step(descs, n, R, L) != 0) return -2;
    return (int64_t)L.bytes;
}

static int plan_step(const RansGemvDesc* descs, const void* const* peer_y, int npeers, int n, int R,
                     void* workspace, size_t workspace_bytes, int* grid_out, cudaStream_t stream);
static void register_prescale(const void* ws, size_t jobs_off, int njobs);

// CTAs of the step kernel resident at once on the whole GPU (the L2-prefetch
// distance: chunk b + resident starts roughly when chunk b's CTA is running).
template <int R>
static int resident_ctas_t() {
    static unsigned long long done = 0;
    set_smem_attr((const void*)gemv_step_kernel<R>, &done);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_step_kernel<R>, kThreads, kSmemBytes) !=
        cudaSuccess)
        return 0;
    return per_sm * sm_count();
}

static int resident_ctas(int R) {
    switch (R) {
        case 1: return resident_ctas_t<1>();
        case 2: return resident_ctas_t<2>();
        case 4: return resident_ctas_t<4>();
        case 8: return resident_ctas_t<8>();
        case 16: return resident_ctas_t<16>();
        default: return 0;
    }
}

extern "C" int rans_gemv_step_plan(const RansGemvDesc* descs, int n, int R, void* workspace,
                                   size_t workspace_bytes, int* grid_out, cudaStream_t stream) {
    return plan_step(descs, nullptr, 0, n, R, workspace, workspace_bytes, grid_out, stream);
}

extern "C" int rans_gemv_step_plan_peers(const RansGemvDesc* descs, const void* const* peer_y, int npeers,
                                         int n, int R, void* workspace, size_t workspace_bytes,
                                         int* grid_out, cudaStream_t stream) {
    if (npeers < 1 || npeers > kMaxPeers || peer_y == nullptr) return -2;
    return plan_step(descs, peer_y, npeers, n, R, workspace, workspace_bytes, grid_out, stream);
}

static int plan_step(const RansGemvDesc* descs, const void* const* peer_y, int npeers, int n, int R,
                     void* workspace, size_t workspace_bytes, int* grid_out, cudaStream_t stream) {
    if (!valid_R(R)) return -1;
    if (n <= 0) return -2;
    StepLayout L;
    if (layout_step(descs, n, R, L) != 0) return -2;
    std::vector<MatDev>& mats = L.mats;
    const int64_t nchunks = L.nchunks;
    for (int i = 0; i < n && peer_y != nullptr; ++i) {
        if (mats[i].accumulate) return -2;   // atomically accumulated rows cannot be exchanged by stores
        mats[i].npeer = npeers;
        for (int p = 0; p < npeers; ++p)
            mats[i].ypeer[p] = static_cast<float*>(const_cast<void*>(peer_y[(size_t)i * npeers + p]));
    }
    if (L.bytes > workspace_bytes) return -3;
    // counters (zeroed here, reset by the kernel after each use) and partials
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int64_t coff = 0, poff = 0;
    for (MatDev& d : mats) {
        if (d.nseg > 1 && !d.accumulate && !d.combine) {
            d.counters = reinterpret_cast<uint32_t*>(ws + L.counters_off) + coff;
            d.partials = reinterpret_cast<float*>(ws + L.partials_off) + poff;
            coff += d.nrb;
            poff += (int64_t)d.nrb * d.nseg * R;
        }
    }
    std::vector<uint8_t> host(L.partials_off, 0);
    // activation prescale: the step kernel reads x' (fp32) from the workspace
    PrescaleJob* jobs = reinterpret_cast<PrescaleJob*>(host.data() + L.jobs_off);
    int nj = 0;
    for (size_t i = 0; i < mats.size(); ++i) {
        if (L.xprime[i] == 0) continue;
        MatDev& d = mats[i];
        jobs[nj].x = static_cast<const __nv_bfloat16*>(d.x);
        jobs[nj].step = d.step;
        jobs[nj].out = reinterpret_cast<float*>(ws + L.xprime[i]);
        jobs[nj].cols = d.cols;
        jobs[nj].pad_ = 0;
        ++nj;
        d.x = ws + L.xprime[i];
        d.step = nullptr;
    }
    StepHeader* h = reinterpret_cast<StepHeader*>(host.data());
    h->ndesc = n;
    h->nchunks = (int)nchunks;
    h->R = R;
    h->ahead = resident_ctas(R);
    h->spans_off = (int64_t)L.spans_off;
    MatDev* md = reinterpret_cast<MatDev*>(h + 1);
    Chunk* ch = reinterpret_cast<Chunk*>(md + n);
    int64_t c = 0;
    for (int i = 0; i < n; ++i) {
        md[i] = mats[i];
        const int cs = chunk_items(mats[i]);
        for (int it = 0; it < mats[i].nitems; it += cs) {
            ch[c].desc = i;
            ch[c].item0 = it;
            ch[c].nitems = mats[i].nitems - it < cs ? mats[i].nitems - it : cs;
            ch[c].phase = 0;
            ++c;
        }
    }
    // Longest chunks first: CTAs start in blockIdx order, so the grid's last
    // wave holds the shortest chunks and the tail stays short.
    auto item_cost = [&](const MatDev& d) -> int64_t {
        return (int64_t)R * d.cbs * d.C;
    };
    std::stable_sort(ch, ch + nchunks, [&](const Chunk& a, const Chunk& b) {
        return item_cost(md[a.desc]) > item_cost(md[b.desc]);
    });
    if (grid_out) *grid_out = (int)nchunks;
    cudaError_t e = cudaMemcpyAsync(workspace, host.data(), host.size(), cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return (int)e;
    // word span of every chunk (needs the device offsets), for the L2 prefetch
    fill_spans_kernel<<<(unsigned)((nchunks + 255) / 256), 256, 0, stream>>>(
        static_cast<const StepHeader*>(workspace), R);
    e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    // the pageable source must stay valid until the copy has been staged
    e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess) register_prescale(workspace, L.jobs_off, nj);
    return (int)e;
}

// Prescale jobs of each planned workspace (host side: the launch entry point
// takes only the workspace pointer and the grid).  Re-planning a workspace
// replaces its entry.
struct PrescaleInfo {
    size_t jobs_off;
    int njobs;
};
static std::mutex g_prescale_mu;
static std::unordered_map<const void*, PrescaleInfo> g_prescale;

static void register_prescale(const void* ws, size_t jobs_off, int njobs) {
    std::lock_guard<std::mutex> lock(g_prescale_mu);
    if (njobs > 0) g_prescale[ws] = PrescaleInfo{jobs_off, njobs};
    else g_prescale.erase(ws);
}

static PrescaleInfo find_prescale(const void* ws) {
    std::lock_guard<std::mutex> lock(g_prescale_mu);
    const auto it = g_prescale.find(ws);
    return it == g_prescale.end() ? PrescaleInfo{0, 0} : it->second;
}

static cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

static int launch_prescale(const void* ws, const PrescaleInfo& p, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.njobs < 65535 ? p.njobs : 65535);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = RB_PDL ? 1 : 0;
    const PrescaleJob* jobs = reinterpret_cast<const PrescaleJob*>(static_cast<const uint8_t*>(ws) + p.jobs_off);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, prescale_kernel, jobs, p.njobs);
    if (e != cudaSuccess) return (int)e;
    return (int)cudaGetLastError();
}

template <int R>
static int launch_step_t(const void* ws, int nchunks, cudaStream_t stream) {
    static unsigned long long done = 0;
    set_smem_attr((const void*)gemv_step_kernel<R>, &done);
    // programmatic dependent launch: may start while the previous kernel of the
    // stream drains; the kernel waits for it before touching activations/outputs
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nchunks);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = RB_PDL ? 1 : 0;
    const StepHeader* h = static_cast<const StepHeader*>(ws);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_step_kernel<R>, h);
    if (e != cudaSuccess) return (int)e;
    return (int)cudaGetLastError();
}

extern "C" int rans_gemv_step_kernels(const void* workspace) {
    return find_prescale(workspace).njobs > 0 ? 2 : 1;
}

extern "C" int rans_gemv_step_launch(int R, const void* workspace, int grid, cudaStream_t stream) {
    const int nchunks = grid;
    if (nchunks <= 0) return 0;
    if (!valid_R(R)) return -1;
    const PrescaleInfo p = find_prescale(workspace);
    if (p.njobs > 0) {
        const int e = launch_prescale(workspace, p, stream);
        if (e != 0) return e;
    }
    switch (R) {
        case 1: return launch_step_t<1>(workspace, nchunks, stream);
        case 2: return launch_step_t<2>(workspace, nchunks, stream);
        case 4: return launch_step_t<4>(workspace, nchunks, stream);
        case 8: return launch_step_t<8>(workspace, nchunks, stream);
        case 16: return launch_step_t<16>(workspace, nchunks, stream);
        default: return -1;
    }
}

namespace rb200 {

// ------------------------------------------------------------ chain launcher
// Every projection of a decoder step, in dependency order, from ONE persistent
// grid.  A decoder step is a chain of phases -- per layer {q,k,v} -> o ->
// {gate,up} -> down -- and phase p+1 reads what phase p wrote.  The chain
// kernel runs as many CTAs as fit on the GPU at once; each takes chunks (up to
// 8 items of one matrix) from a queue ordered by phase with one atomic, loads
// its matrix's table, warms L2 with the chunk's words, and, for a chunk of
// phase p > 0, waits until every chunk of phase p-1 is complete (and, when the
// projections are row-sharded over several GPUs, until every rank has
// signalled phase p-1).  Every chunk of phase p-1 was handed to a CTA that is
// already running before any chunk of phase p was, so the waits always end
// without any co-residency assumption.  Each wait is bounded: after the
// plan's timeout the kernel records the phase, every CTA leaves, and
// rans_gemv_chain_status reports it (the context stays usable).
//
// Memory ordering.  A CTA finishing a chunk: bar.sync, then one thread fences
// (gpu scope; system scope when its rows were also stored to peer GPUs) and
// increments the phase's completion counter.  The CTA that completes a phase
// on a multi-GPU plan then fences at system scope once more and adds 1 to
// that phase's arrival counter on every rank (relaxed reductions).  A waiting thread reads the counters with
// ld.acquire, then bar.sync, then reads activations with weak L1-cached loads.
//
// The last CTA to leave resets the queue and completion counters and counts
// the launch (epoch); arrival counters only grow, and a multi-GPU wait of
// launch e needs nranks * (e + 1) arrivals.  A wait that ran out leaves the
// status set: launches return at once until rans_gemv_chain_status has read
// and cleared it (multi-GPU plans must then be planned again on every rank).
constexpr int32_t kChainTimeout = 1;
constexpr int kDoneStride = 32;   // one 128-byte line per phase's completion counter

struct ChainHeader {
    int ndesc, nchunks, R, nphases;
    int npeer, rank;
    int shift;                 // kernel phase = caller phase + shift (1 when activations are prescaled up front)
    int pad0;
    int64_t phase_off;         // int32 phase_end[nphases]: chunks [phase_end[p-1], phase_end[p]) are phase p
    int64_t ctl_off;           // ChainCtl, then uint32 done[nphases * kDoneStride] (one line per phase)
    int64_t timeout_ns;        // bound of every dependency wait
    int64_t jobs_off;          // PrescaleJob[] of the activation prescale chunks
    uint32_t* arrive;          // this rank's arrival counters [nphases] (multi-GPU), or null
    uint32_t* arrive_peer[kMaxPeers];   // every rank's arrival counters, as addresses valid on this GPU
};

struct ChainCtl {
    uint32_t queue;            // next chunk to hand out
    uint32_t exited;           // CTAs that have left this launch
    uint32_t epoch;            // launches completed on this workspace
    int32_t status;            // 0, or kChainTimeout once a wait ran out (sticky until read)
    int32_t where;             // phase whose wait ran out
    uint32_t pad[3];
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t phase_chunks(const int* phase_end, int p) {
    return (uint32_t)(phase_end[p] - (p > 0 ? phase_end[p - 1] : 0));
}

// Control block and completion counters of a chain workspace.
__device__ __forceinline__ ChainCtl* chain_ctl(const ChainHeader* h) {
    return reinterpret_cast<ChainCtl*>(const_cast<uint8_t*>(reinterpret_cast<const uint8_t*>(h)) + h->ctl_off);
}
__device__ __forceinline__ const int* chain_phase_end(const ChainHeader* h) {
    return reinterpret_cast<const int*>(reinterpret_cast<const uint8_t*>(h) + h->phase_off);
}
__device__ __forceinline__ const PrescaleJob* chain_jobs(const ChainHeader* h) {
    return reinterpret_cast<const PrescaleJob*>(reinterpret_cast<const uint8_t*>(h) + h->jobs_off);
}
__device__ __forceinline__ const Chunk* chain_chunks(const ChainHeader* h) {
    return reinterpret_cast<const Chunk*>(reinterpret_cast<const MatDev*>(h + 1) + h->ndesc);
}

// Thread 0 of a CTA: wait until phase p is complete -- all its chunks on this
// GPU and, multi-GPU, every rank's arrival for this launch.  Polls with a
// growing sleep; returns false when the wait ran out (recording it) or another
// CTA already reported an error.
__device__ bool chain_wait(const ChainHeader* h, int p) {
    ChainCtl* ctl = chain_ctl(h);
    const uint32_t* done = reinterpret_cast<const uint32_t*>(ctl + 1);
    const uint32_t need = phase_chunks(chain_phase_end(h), p);
    // the epoch changes only after every CTA of this launch has left
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&ctl->epoch);
    const uint32_t need_arrive = (uint32_t)h->npeer * (epoch + 1u);
    uint64_t t0 = 0;
    unsigned sleep_ns = 32;
    for (;;) {
        const bool local = ld_acquire_gpu(done + p * kDoneStride) >= need;
        const bool peers = h->npeer == 0 || (int32_t)(ld_acquire_sys(h->arrive + p) - need_arrive) >= 0;
        if (local && peers) return true;
        if (*reinterpret_cast<volatile int32_t*>(&ctl->status) != 0) return false;
        const uint64_t t = global_ns();
        if (t0 == 0) {
            t0 = t;
        } else if (t - t0 > (uint64_t)h->timeout_ns) {
            if (atomicCAS(&ctl->status, 0, kChainTimeout) == 0) atomicExch(&ctl->where, p);
            return false;
        }
        __nanosleep(sleep_ns);
        if (sleep_ns < RB_POLL_MAX_NS) sleep_ns *= 2;
    }
}

// Chunk.phase of a chain chunk: the phase in the low bits; kChainAhead set
// when at least a full wave of chunks of the same phase follows it, so the
// CTA may take its next chunk while it works on this one (no CTA then holds
// a chunk near a phase's end while busy with another).
constexpr int kChainAhead = 1 << 30;
constexpr int kChainPhaseMask = kChainAhead - 1;

// Thread 0: a chunk taken from the queue (`raw`, the queue's old value) as
// the index to run -- nchunks once the queue is empty or an error was
// reported (`status`, read no earlier than the atomic was issued).
__device__ __forceinline__ int chain_take(const ChainHeader* h, uint32_t raw, int32_t status) {
    return status != 0 ? h->nchunks : (int)min(raw, (uint32_t)h->nchunks);
}

// Thread 0: the next chunk of the queue.  The atomic and the status read are
// issued together (one round trip, not two).
__device__ __forceinline__ int chain_grab(const ChainHeader* h) {
    ChainCtl* ctl = chain_ctl(h);
    const uint32_t raw = atomicAdd(&ctl->queue, 1u);
    return chain_take(h, raw, *reinterpret_cast<volatile int32_t*>(&ctl->status));
}

// Thread 0: publish `count` finished chunks of phase p -- every output they
// wrote (ordered before by the bar.sync that ended each chunk) is made
// visible (fence; system scope when rows went to peers) and counted; the CTA
// completing phase p on a multi-GPU plan tells every rank.  A CTA publishes
// the chunks it finished in the middle of a phase together, when it moves to
// another phase, reaches the phase's last wave or leaves (it never waits
// while holding unpublished chunks, and the fence is paid rarely); chunks of
// a phase's last wave are published as soon as they end.
__device__ __forceinline__ void chain_signal(const ChainHeader* h, int p, uint32_t count) {
    uint32_t* done = reinterpret_cast<uint32_t*>(chain_ctl(h) + 1);
    if (h->npeer > 0) {
        __threadfence_system();   // this CTA's stores, peers' rows included, before its count
        const uint32_t prev = atomicAdd(done + p * kDoneStride, count);
        if (prev + count == phase_chunks(chain_phase_end(h), p)) {
            // every CTA of this rank has published phase p: one system fence
            // orders all of it before the signals, which then need no fence of
            // their own (a release per peer would serialise one per rank)
            __threadfence_system();
            for (int q = 0; q < h->npeer; ++q) red_relaxed_sys(h->arrive_peer[q] + p, 1u);
        }
    } else {
        __threadfence();
        atomicAdd(done + p * kDoneStride, count);
    }
}

template <int R>
__global__ void __launch_bounds__(kThreads, RB_MINB) gemv_chain_kernel(const ChainHeader* __restrict__ hdr) {
    __shared__ int s_chunk;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const SmemMap sm = smem_map(warp);
    const uint32_t* cur = nullptr;    // table now in shared memory
    // thread 0: the next chunk -- the queue's old value and the status.  For a
    // chunk that may be taken ahead both are read when this chunk starts and
    // first used when it ends, so the round trip overlaps the chunk (`ahead`);
    // otherwise they are read when it ends.
    bool ahead = false;
    uint32_t ahead_raw = 0;
    int32_t ahead_status = 0;
    int cur_desc = -1;                // descriptor whose table `cur` is
    int pend_phase = -1;              // thread 0: phase of finished, unpublished chunks
    uint32_t pend = 0;                //           and how many
    if (threadIdx.x == 0) {
        g_chain_hdr = hdr;
        s_chunk = chain_grab(hdr);
    }
    if (lane == 0) g_chain_known[warp] = -1;
    __syncthreads();
    for (;;) {
        const int c = s_chunk;
        if (c >= hdr->nchunks) break;
        const Chunk ch = chain_chunks(hdr)[c];
        const int phase = ch.phase & kChainPhaseMask;
        if (threadIdx.x == 0) {
            if (pend > 0 && pend_phase != phase) {
                chain_signal(hdr, pend_phase, pend);   // before any wait of this chunk
                pend = 0;
            }
            if (ch.phase & kChainAhead) {
                ChainCtl* ctl = chain_ctl(hdr);
                ahead_raw = atomicAdd(&ctl->queue, 1u);
                ahead_status = *reinterpret_cast<volatile int32_t*>(&ctl->status);
                ahead = true;
            }
        }
        if (ch.nitems < 0) {
            // activation prescale job: x' = bf16 x * step for columns
            // [item0, item0 - nitems) of one matrix, read by the next phase.
            // Its inputs were written before the launch: no wait.
            const PrescaleJob jb = chain_jobs(hdr)[ch.desc];
            const unsigned short* xb = reinterpret_cast<const unsigned short*>(jb.x);
            for (int col = ch.item0 + (int)threadIdx.x; col < ch.item0 - ch.nitems; col += blockDim.x)
                jb.out[col] = __uint_as_float((uint32_t)xb[col] << 16) * __ldg(jb.step + col);
        } else {
            const MatDev& d = reinterpret_cast<const MatDev*>(hdr + 1)[ch.desc];
            // weights are immutable: the table load and each warp's staging
            // and state reads overlap the previous phase; each warp waits for
            // it only before its first activation load (dep_wait)
            if (ch.desc != cur_desc) {    // a descriptor's table pointer is read once per change
                if (d.table != cur) {
                    load_table(sm.tab, d.table);
                    cur = d.table;
                }
                cur_desc = ch.desc;
            }
            if (threadIdx.x == 0) g_chain_wait = phase > 0 ? phase - 1 : -1;
            __syncthreads();
            if (warp < ch.nitems) {
                // every activation is fp32 x*step here (the planner turned bf16
                // ones into prescale jobs of the previous phase)
                int bad = 0;
                const MatDev dl = d;
                process_item<R, kXCoherent | kXPref | kXChain>(dl, ch.item0 + warp, sm.tab, sm.stage, lane, bad,
                                                                warp, ch.nitems);
            }
        }
        __syncthreads();   // every output of chunk c is written
        if (threadIdx.x == 0) {
            pend_phase = phase;
            ++pend;
            // the next chunk: taken ahead, or the queue atomic issued now,
            // before the publication below, so the two round trips overlap
            if (!ahead) {
                ChainCtl* ctl = chain_ctl(hdr);
                ahead_raw = atomicAdd(&ctl->queue, 1u);
                ahead_status = *reinterpret_cast<volatile int32_t*>(&ctl->status);
            }
            if (!(ch.phase & kChainAhead) && hdr->npeer == 0) {
                // one of the phase's last chunks: its completion may be what
                // the next phase waits for, publish it now (multi-GPU plans
                // publish once per phase and CTA: each publication fences at
                // system scope, an NVLink round trip that stalls warp 0)
                chain_signal(hdr, phase, pend);
                pend = 0;
            }
            s_chunk = chain_take(hdr, ahead_raw, ahead_status);
            ahead = false;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        if (pend > 0) chain_signal(hdr, pend_phase, pend);
        // the last CTA out resets the queue and the completion counters
        ChainCtl* ctl = chain_ctl(hdr);
        __threadfence();
        const uint32_t n = atomicAdd(&ctl->exited, 1u);
        if (n + 1 == gridDim.x) {
            uint32_t* done = reinterpret_cast<uint32_t*>(ctl + 1);
            for (int p = 0; p < hdr->nphases; ++p) done[p * kDoneStride] = 0u;
            ctl->queue = 0u;
            ctl->exited = 0u;
            ctl->epoch = *reinterpret_cast<volatile uint32_t*>(&ctl->epoch) + 1u;
            __threadfence();
        }
    }
}

struct ChainLayout {
    std::vector<MatDev> mats;
    std::vector<PrescaleJob> jobs;     // activation prescale jobs (out set when planned into a workspace)
    std::vector<int> job_mat;          // the matrix of each job
    std::vector<int> parent;           // per decomposition: the caller's matrix it belongs to
    std::vector<int> head_rb;          // per decomposition split in two: first row block of the fine tail
    std::vector<size_t> xprime;        // per matrix: byte offset of its x' (0 = fp32 x given)
    std::vector<Chunk> chunks;         // in hand-out order
    std::vector<int> phase_end;        // per kernel phase: one past its last chunk
    int nphases = 0;                   // kernel phases (the caller's, plus one in front when needed)
    int shift = 0;                     // 1 when that front phase (activation prescale) exists
    size_t jobs_off = 0, phase_off = 0, ctl_off = 0, counters_off = 0, partials_off = 0, xprime_off = 0,
           bytes = 0;
};

constexpr int kPrescaleCols = 8192;    // columns per activation prescale chunk
// Most tiles one chain item decodes at once (the launch planner's limit, 4).
// Smaller items give a phase more CTA chunks to balance, but measured slower
// on B200: 8 layers of the 70B-shaped chain 4.92 ms at 4 tiles, 5.39 at 2,
// 6.75 at 1; one rank's eighth of the 80-layer step 9.49 / 10.36 / 11.90 ms
// (each item's staging, reduction and epilogue cost more than balance gains).
#ifndef RB_CHAIN_TILES
#define RB_CHAIN_TILES 4
#endif
constexpr int kChainTiles = RB_CHAIN_TILES;

// The chain's work list.  Caller phase p becomes kernel phase p + shift; a
// matrix with bf16 activations (written before the launch) reads a prescaled
// fp32 copy x' that prescale chunks of the kernel phase before its own write
// (for caller phase 0 that is an extra kernel phase 0, shift = 1).  Within a
// phase: its prescale chunks first, then its decode chunks, longest first.
static int layout_chain(const RansGemvDesc* descs, const int* phase, int n, int R, ChainLayout& L) {
    if (n <= 0 || descs == nullptr || phase == nullptr) return -2;
    int P = 0;
    for (int i = 0; i < n; ++i) {
        if (phase[i] < 0 || phase[i] >= n) return -2;
        P = std::max(P, phase[i] + 1);
    }
    std::vector<std::vector<int>> members(P);
    for (int i = 0; i < n; ++i) members[phase[i]].push_back(i);
    for (int p = 0; p < P; ++p)
        if (members[p].empty()) return -2;   // phases are numbered 0..P-1 without gaps
    L.mats.clear();
    if (count_chunks(descs, n, R, &L.mats, kChainTiles) < 0) return -2;
    int64_t ncounters = 0, npartials = 0;
    L.parent.resize(n);
    for (int i = 0; i < n; ++i) L.parent[i] = i;
    L.head_rb.assign(n, -1);
    std::vector<std::vector<int>> tails(P);     // per phase: the fine decompositions (indices into mats)
    const int64_t W = split_target();
    for (int p = 0; p < P; ++p) {
        // each phase runs on the whole GPU by itself: plan it like one launch
        std::vector<MatDev> g;
        for (int i : members[p]) g.push_back(L.mats[i]);
        plan_group(g, R, ncounters, npartials, kChainTiles);
        int64_t items = 0;
        for (size_t k = 0; k < g.size(); ++k) {
            L.mats[members[p][k]] = g[k];
            items += g[k].nitems;
        }
        if (items <= W) continue;
        // A phase of several waves ends in a partly filled last wave of whole
        // items, and the next phase cannot start before it ends.  Its last
        // wave's worth of row blocks (about W / items of every matrix) is
        // therefore decoded as items of half as many tiles (one pass each),
        // handed out after everything else: a second decomposition of the
        // same matrix covering the tail's row blocks only (its chunks select
        // those items).  (One-tile items measured slower: their staging,
        // reduction and global partial sums cost more than the tail saved.)
        const double f = std::min(0.5, (double)W / (double)items);
        for (int i : members[p]) {
            const MatDev& d = L.mats[i];
            int kf = 0;
            for (int t = d.cbs / 2; t >= 1 && kf == 0; --t)
                if (d.ncb % t == 0) kf = t;
            if (kf == 0 || kf >= d.kcol) continue;            // nothing finer with fewer streams
            const int tail = std::min(d.nrb, std::max(1, (int)std::ceil(f * d.nrb)));
            MatDev fd = d;
            fd.kcol = kf;
            fd.nseg = d.ncb / kf;
            fd.cbs = kf;
            fd.nitems = d.nrb * fd.nseg;
            fd.accumulate = 0;
            fd.combine = fd.nseg <= kWarps ? 1 : 0;
            fd.counters = nullptr;
            fd.partials = nullptr;
            if (!fd.combine) {
                ncounters += fd.nrb;
                npartials += (int64_t)fd.nrb * fd.nseg * R;
            }
            L.head_rb[i] = d.nrb - tail;
            L.mats.push_back(fd);
            L.parent.push_back(i);
            L.head_rb.push_back(d.nrb - tail);             // the fine one starts there
            tails[p].push_back((int)L.mats.size() - 1);
        }
    }
    // prescale jobs and x' buffers of the bf16-activation matrices
    L.jobs.clear();
    L.job_mat.clear();
    L.xprime.assign(n, 0);
    std::vector<int> job_of(n, -1);
    size_t xbytes = 0;
    for (int i = 0; i < n; ++i) {
        if (L.mats[i].step == nullptr) continue;
        job_of[i] = (int)L.jobs.size();
        PrescaleJob jb;
        jb.x = static_cast<const __nv_bfloat16*>(L.mats[i].x);
        jb.step = L.mats[i].step;
        jb.out = nullptr;
        jb.cols = L.mats[i].cols;
        jb.pad_ = 0;
        L.jobs.push_back(jb);
        L.job_mat.push_back(i);
        L.xprime[i] = xbytes;              // relative to xprime_off until the offsets are known
        xbytes = align16(xbytes + sizeof(float) * (size_t)L.mats[i].cols);
    }
    auto prescale_chunks = [&](int p, int kphase) {
        for (int i : members[p]) {
            if (job_of[i] < 0) continue;
            for (int c0 = 0; c0 < L.mats[i].cols; c0 += kPrescaleCols) {
                const int cnt = std::min(kPrescaleCols, L.mats[i].cols - c0);
                L.chunks.push_back(Chunk{job_of[i], c0, -cnt, kphase});
            }
        }
    };
    auto item_cost = [&](const MatDev& d) -> int64_t { return (int64_t)R * d.cbs * d.C; };
    bool front = false;
    for (int i : members[0]) front = front || job_of[i] >= 0;
    const int shift = front ? 1 : 0;
    L.chunks.clear();
    L.phase_end.clear();
    if (front) {
        prescale_chunks(0, 0);
        L.phase_end.push_back((int)L.chunks.size());
    }
    for (int p = 0; p < P; ++p) {
        const int kp = p + shift;
        if (p + 1 < P) prescale_chunks(p + 1, kp);
        // items [i0, i1) of decomposition k (row blocks split at head_rb)
        auto emit = [&](int k, int i0, int i1) {
            const int cs = chunk_items(L.mats[k]);
            for (int it = i0; it < i1; it += cs) L.chunks.push_back(Chunk{k, it, std::min(cs, i1 - it), kp});
        };
        auto by_cost = [&](size_t c0) {
            // longest chunks first: the last CTAs to start run the shortest
            std::stable_sort(L.chunks.begin() + c0, L.chunks.end(), [&](const Chunk& a, const Chunk& b) {
                return item_cost(L.mats[a.desc]) > item_cost(L.mats[b.desc]);
            });
        };
        size_t c0 = L.chunks.size();
        for (int i : members[p]) {
            const MatDev& d = L.mats[i];
            emit(i, 0, L.head_rb[i] < 0 ? d.nitems : L.head_rb[i] * d.nseg);
        }
        by_cost(c0);
        c0 = L.chunks.size();
        for (int k : tails[p]) emit(k, L.head_rb[k] * L.mats[k].nseg, L.mats[k].nitems);
        by_cost(c0);
        L.phase_end.push_back((int)L.chunks.size());
    }
    L.nphases = P + shift;
    L.shift = shift;
    const size_t nch = L.chunks.size();
    L.jobs_off = align16(sizeof(ChainHeader) + sizeof(MatDev) * L.mats.size() + sizeof(Chunk) * nch);
    L.phase_off = align16(L.jobs_off + sizeof(PrescaleJob) * L.jobs.size());
    L.ctl_off = align16(L.phase_off + sizeof(int) * (size_t)L.nphases);
    L.counters_off = align16(L.ctl_off + sizeof(ChainCtl) + sizeof(uint32_t) * kDoneStride * (size_t)L.nphases);
    L.partials_off = align16(L.counters_off + sizeof(uint32_t) * (size_t)ncounters);
    L.xprime_off = align16(L.partials_off + sizeof(float) * (size_t)npartials);
    L.bytes = L.xprime_off + xbytes;
    return 0;
}

extern "C" int64_t rans_gemv_chain_workspace_bytes(const RansGemvDesc* descs, const int* phase, int n, int R) {
    if (!valid_R(R)) return -1;
    ChainLayout L;
    if (layout_chain(descs, phase, n, R, L) != 0) return -2;
    return (int64_t)L.bytes;
}

extern "C" int64_t rans_gemv_chain_describe(const RansGemvDesc* descs, const int* phase, int n, int R,
                                            int32_t* out, int64_t max_chunks) {
    if (!valid_R(R)) return -1;
    ChainLayout L;
    if (layout_chain(descs, phase, n, R, L) != 0) return -2;
    const int64_t nc = (int64_t)L.chunks.size();
    for (int64_t c = 0; out != nullptr && c < nc && c < max_chunks; ++c) {
        const Chunk& ch = L.chunks[c];
        int32_t* o = out + 8 * c;
        o[0] = ch.phase;
        if (ch.nitems < 0) {               // activation prescale: columns [item0, item0 - nitems)
            o[1] = L.job_mat[ch.desc];
            o[2] = 1;
            o[3] = ch.item0;
            o[4] = -ch.nitems;
            o[5] = o[6] = o[7] = 0;
        } else {
            const MatDev& d = L.mats[ch.desc];
            o[1] = L.parent[ch.desc];
            o[2] = 0;
            o[3] = ch.item0;
            o[4] = ch.nitems;
            o[5] = d.cbs;
            o[6] = d.kcol;
            o[7] = d.nseg;
        }
    }
    return nc;
}

template <int R>
static int chain_grid_t(int64_t nchunks) {
    static unsigned long long done = 0;
    static int resident[64] = {};
    if (!set_smem_attr((const void*)gemv_chain_kernel<R>, &done)) return -1;
    return (int)std::min<int64_t>(nchunks, resident_blocks((const void*)gemv_chain_kernel<R>, resident));
}

static int chain_grid(int R, int64_t nchunks) {
    switch (R) {
        case 1: return chain_grid_t<1>(nchunks);
        case 2: return chain_grid_t<2>(nchunks);
        case 4: return chain_grid_t<4>(nchunks);
        case 8: return chain_grid_t<8>(nchunks);
        case 16: return chain_grid_t<16>(nchunks);
        default: return -1;
    }
}

extern "C" int rans_gemv_chain_plan(const RansGemvDesc* descs, const int* phase, int n, int R,
                                    const RansChainSync* sync, int timeout_ms, void* workspace,
                                    size_t workspace_bytes, int* grid_out, cudaStream_t stream) {
    if (!valid_R(R)) return -1;
    if (timeout_ms <= 0) return -2;
    if (sync != nullptr && (sync->nranks < 1 || sync->nranks > kMaxPeers || sync->rank < 0 ||
                            sync->rank >= sync->nranks || sync->arrive == nullptr ||
                            sync->arrive_peer == nullptr || sync->peer_y == nullptr))
        return -2;
    ChainLayout L;
    if (layout_chain(descs, phase, n, R, L) != 0) return -2;
    if (L.bytes > workspace_bytes) return -3;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int64_t coff = 0, poff = 0;
    const int nm = (int)L.mats.size();     // the caller's matrices, then the fine tails
    for (int k = 0; k < nm; ++k) {
        MatDev& d = L.mats[k];
        const int i = L.parent[k];
        if (d.nseg > 1 && !d.accumulate && !d.combine) {
            d.counters = reinterpret_cast<uint32_t*>(ws + L.counters_off) + coff;
            d.partials = reinterpret_cast<float*>(ws + L.partials_off) + poff;
            coff += d.nrb;
            poff += (int64_t)d.nrb * d.nseg * R;
        }
        if (d.step != nullptr) {
            // decode reads the prescaled copy written by the prescale chunks
            d.x = ws + L.xprime_off + L.xprime[i];
            d.step = nullptr;
        }
        if (sync != nullptr) {
            if (d.accumulate) return -2;   // atomically accumulated rows cannot be exchanged by stores
            d.npeer = sync->nranks;
            for (int p = 0; p < sync->nranks; ++p)
                d.ypeer[p] = static_cast<float*>(const_cast<void*>(sync->peer_y[(size_t)i * sync->nranks + p]));
        }
    }
    for (size_t j = 0; j < L.jobs.size(); ++j)
        L.jobs[j].out = reinterpret_cast<float*>(ws + L.xprime_off + L.xprime[L.job_mat[j]]);
    // host image up to the partials (header, descriptors, chunks, prescale
    // jobs, phase ends, zeroed control block and segment counters)
    std::vector<uint8_t> host(L.partials_off, 0);
    ChainHeader* h = reinterpret_cast<ChainHeader*>(host.data());
    h->ndesc = nm;
    h->nchunks = (int)L.chunks.size();
    h->R = R;
    h->nphases = L.nphases;
    h->npeer = sync ? sync->nranks : 0;
    h->rank = sync ? sync->rank : 0;
    h->phase_off = (int64_t)L.phase_off;
    h->ctl_off = (int64_t)L.ctl_off;
    h->timeout_ns = (int64_t)timeout_ms * 1000000ll;
    h->jobs_off = (int64_t)L.jobs_off;
    h->shift = L.shift;
    if (sync) {
        h->arrive = static_cast<uint32_t*>(sync->arrive);
        for (int p = 0; p < sync->nranks; ++p) h->arrive_peer[p] = static_cast<uint32_t*>(sync->arrive_peer[p]);
    }
    MatDev* md = reinterpret_cast<MatDev*>(h + 1);
    for (int k = 0; k < nm; ++k) md[k] = L.mats[k];
    std::memcpy(md + nm, L.chunks.data(), sizeof(Chunk) * L.chunks.size());
    if (!L.jobs.empty()) std::memcpy(host.data() + L.jobs_off, L.jobs.data(), sizeof(PrescaleJob) * L.jobs.size());
    int* pe = reinterpret_cast<int*>(host.data() + L.phase_off);
    for (int p = 0; p < L.nphases; ++p) pe[p] = L.phase_end[p];
    const int grid = chain_grid(R, (int64_t)L.chunks.size());
    if (grid <= 0) return (int)cudaErrorInvalidConfiguration;
    {
        // chunks followed by at least a full wave of their own phase may be
        // taken one chunk ahead
        Chunk* chw = reinterpret_cast<Chunk*>(md + nm);
        for (size_t c = 0; c < L.chunks.size(); ++c)
            if ((int64_t)c + grid < L.phase_end[chw[c].phase]) chw[c].phase |= kChainAhead;
    }
    cudaError_t e = cudaMemcpyAsync(workspace, host.data(), host.size(), cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return (int)e;
    if (sync != nullptr) {
        // this rank's arrival counters start at zero; the caller makes every
        // rank finish planning (a host barrier) before any rank launches
        e = cudaMemsetAsync(sync->arrive, 0, sizeof(uint32_t) * (size_t)L.nphases, stream);
        if (e != cudaSuccess) return (int)e;
    }
    // the pageable source must stay valid until the copy has been staged
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return (int)e;
    if (grid_out) *grid_out = grid;
    return 0;
}

template <int R>
static int launch_chain_t(const void* ws, int grid, cudaStream_t stream) {
    static unsigned long long done = 0;
    set_smem_attr((const void*)gemv_chain_kernel<R>, &done);
    gemv_chain_kernel<R><<<grid, kThreads, kSmemBytes, stream>>>(static_cast<const ChainHeader*>(ws));
    return (int)cudaGetLastError();
}

extern "C" int rans_gemv_chain_launch(int R, const void* workspace, int grid, cudaStream_t stream) {
    if (grid <= 0) return 0;
    switch (R) {
        case 1: return launch_chain_t<1>(workspace, grid, stream);
        case 2: return launch_chain_t<2>(workspace, grid, stream);
        case 4: return launch_chain_t<4>(workspace, grid, stream);
        case 8: return launch_chain_t<8>(workspace, grid, stream);
        case 16: return launch_chain_t<16>(workspace, grid, stream);
        default: return -1;
    }
}

extern "C" int rans_gemv_chain_status(void* workspace, int* phase_out, cudaStream_t stream) {
    if (workspace == nullptr) return -2;
    ChainHeader h;
    ChainCtl ctl;
    cudaError_t e = cudaMemcpyAsync(&h, workspace, sizeof(h), cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return (int)e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return (int)e;
    uint8_t* ctl_dev = static_cast<uint8_t*>(workspace) + h.ctl_off;
    e = cudaMemcpyAsync(&ctl, ctl_dev, sizeof(ctl), cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return (int)e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return (int)e;
    // the caller's phase (kernel phases count an up-front prescale phase)
    if (phase_out) *phase_out = ctl.status != 0 ? ctl.where - h.shift : -1;
    if (ctl.status == 0) return 0;
    // read and cleared: the next launch runs again
    e = cudaMemsetAsync(ctl_dev + offsetof(ChainCtl, status), 0, 2 * sizeof(int32_t), stream);
    if (e != cudaSuccess) return (int)e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return (int)e;
    return -5;
}

}  // namespace rb200

// ------------------------------------------------- step launcher, no allocation
// Some callers cannot allocate device memory at the point where they run a
// decoder step: a framework whose caching allocator owns the whole pool (a
// private cudaMalloc behind its back fragments it, or fails under memory
// pressure), an inference loop that forbids allocation after start-up to keep
// its latency predictable, or a runtime with no allocator handle to give us.
// rans_gemv_step_noalloc serves them: its work plan lives in a fixed-size
// file-scope device array instead of a caller-allocated workspace.  The plan
// is the simple one (whole row blocks per warp, eight warps per CTA, longest
// chunks first): it needs no segment partials, counters or prescaled
// activations, so the array holds nothing but descriptors and chunks.  The
// latency-bound split plans of rans_gemv_step_plan are not used here; results
// are the same, small launches run slower.
// Plan bytes = 32 + 200 * n + 16 * sum over matrices of ceil(rows / (8 R)).
static_assert(sizeof(StepHeader) == 32 && sizeof(MatDev) == 200 && sizeof(Chunk) == 16,
              "the plan-size formula of rans_gemv_step_noalloc (include/rans_b200.h)");
constexpr size_t kNoAllocScratchBytes = 256 * 1024;   // the plan's maximum size
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint8_t g_step_scratch[kNoAllocScratchBytes];

// The plan reaches the device inside kernel launch parameters, a piece of at
// most kPlanPieceBytes per launch (the parameter space of a launch is 32,764
// bytes on sm_70 and later with CUDA 12.1+).  A launch copies its parameters
// when it is issued, so nothing on the host has to outlive the call: no
// pageable or pinned staging buffer is read later by the device.
constexpr int kPlanPieceBytes = 32000;
struct PlanPiece {
    uint32_t offset, nbytes;             // destination offset in g_step_scratch, bytes (multiple of 16)
    uint4 bytes[kPlanPieceBytes / 16];
};
static_assert(sizeof(PlanPiece) <= 32764, "plan piece exceeds the kernel parameter space");

__global__ void __launch_bounds__(256) write_plan_kernel(const __grid_constant__ PlanPiece piece) {
    uint4* dst = reinterpret_cast<uint4*>(g_step_scratch + piece.offset);
    for (uint32_t i = threadIdx.x; i < piece.nbytes / 16; i += blockDim.x) dst[i] = piece.bytes[i];
}

// Host staging of the plan (static: no heap), the parameter block of one
// piece, and, per device, the device address of g_step_scratch (the
// host-side name is only a stand-in).
static uint8_t g_noalloc_host[kNoAllocScratchBytes];
static PlanPiece g_noalloc_piece;
static void* g_noalloc_dev[kNoAllocMaxDevices];
static std::mutex g_noalloc_mu;

extern "C" int rans_gemv_step_noalloc(const RansGemvDesc* descs, int n, int R, cudaStream_t stream) {
    if (!valid_R(R)) return -1;
    if (n <= 0 || descs == nullptr) return -2;
    // size check from the shapes alone, before touching any device state
    int64_t nchunks = 0;
    for (int i = 0; i < n; ++i) {
        const RansGemvDesc& s = descs[i];
        if (!shape_ok(R, s.rows, s.cols, s.C)) return -2;
        MatDev d = make_desc(s.words, s.offs, s.table, s.x, s.step, s.y, s.rows, s.cols, s.C, s.nwords);
        plan_matrix(d, R, 0);
        nchunks += (d.nitems + kWarps - 1) / kWarps;
    }
    const size_t bytes = step_bytes(n, nchunks);
    if (bytes > kNoAllocScratchBytes) return -3;   // plan larger than the static scratch
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= kNoAllocMaxDevices) return -2;
    if (g_noalloc_dev[dev] == nullptr) {
        // once per device, with that device current
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_step_scratch);
        if (e != cudaSuccess) return (int)e;
        g_noalloc_dev[dev] = p;
    }
    StepHeader* h = reinterpret_cast<StepHeader*>(g_noalloc_host);
    h->ndesc = n;
    h->nchunks = (int)nchunks;
    h->R = R;
    h->ahead = 0;         // no span table here: no L2 prefetch
    h->spans_off = 0;
    h->pad_ = 0;
    MatDev* md = reinterpret_cast<MatDev*>(h + 1);
    Chunk* ch = reinterpret_cast<Chunk*>(md + n);
    int64_t c = 0;
    for (int i = 0; i < n; ++i) {
        const RansGemvDesc& s = descs[i];
        md[i] = make_desc(s.words, s.offs, s.table, s.x, s.step, s.y, s.rows, s.cols, s.C, s.nwords);
        plan_matrix(md[i], R, 0);
        for (int it = 0; it < md[i].nitems; it += kWarps) {
            ch[c].desc = i;
            ch[c].item0 = it;
            ch[c].nitems = md[i].nitems - it < kWarps ? md[i].nitems - it : kWarps;
            ch[c].phase = 0;
            ++c;
        }
    }
    // same order as rans_gemv_step_plan (longest chunks first, ties in input
    // order), with an in-place sort
    auto item_cost = [&](const MatDev& d) -> int64_t {
        return (int64_t)R * d.cbs * d.C;
    };
    std::sort(ch, ch + nchunks, [&](const Chunk& a, const Chunk& b) {
        const int64_t ca = item_cost(md[a.desc]), cb = item_cost(md[b.desc]);
        if (ca != cb) return ca > cb;
        if (a.desc != b.desc) return a.desc < b.desc;
        return a.item0 < b.item0;
    });
    // Upload through launch parameters, piece by piece, in stream order before
    // the step kernel that reads the plan.
    const size_t padded = (bytes + 15) & ~size_t(15);
    for (size_t off = 0; off < padded; off += kPlanPieceBytes) {
        const size_t nb = std::min<size_t>(kPlanPieceBytes, padded - off);
        g_noalloc_piece.offset = (uint32_t)off;
        g_noalloc_piece.nbytes = (uint32_t)nb;
        std::memcpy(g_noalloc_piece.bytes, g_noalloc_host + off, nb);
        write_plan_kernel<<<1, 256, 0, stream>>>(g_noalloc_piece);
        e = cudaGetLastError();
        if (e != cudaSuccess) return (int)e;
    }
    return rans_gemv_step_launch(R, g_noalloc_dev[dev], (int)nchunks, stream);
}

extern "C" int rans_b200_abi_version(void) { return RANS_B200_ABI_VERSION; }
