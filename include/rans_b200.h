/*
 * rans_b200.h -- C ABI of the B200 (sm_100a) entropy-coded weight GEMV library
 * (librans_b200.so).  Plain pointers, sizes and an int status; no C++ or
 * framework types cross this boundary.
 *
 * Bitstream ("tile-interleaved rANS", unchanged from the reference
 * snuri00/vram-compression, kernel/rans_gemv.cu:1-15 and kernel/rans.py:55-98):
 *   - W (rows x cols) holds integer codes; W_real[r,c] = code[r,c] * step[c].
 *   - The matrix is cut into tiles of R rows x C columns; tile t = rb*ncb + cb
 *     (ncb = cols / C).  Lane l (0..31) of a tile owns columns l, l+32, ... and
 *     stores them as one rANS stream s = t*32 + l in the order
 *       for k in 0..C/32-1: for r in 0..R-1: code[rb*R + r][cb*C + l + 32k].
 *   - 32-bit state in [2^16, 2^32), 16-bit renormalisation words, 12-bit
 *     probabilities, one static table per matrix:
 *       table[slot] = sym | freq << 8 | (slot - cum[sym]) << 20,  sym = code + 128.
 *   - words: uint16, each stream = [state >> 16, state & 0xffff, payload...],
 *     followed by 8 zero pad words after the last stream; offs: uint32 word
 *     offset of every stream (rows*cols*32/(R*C) entries).
 *
 * All launchers are asynchronous on `stream`, allocate nothing unless stated,
 * and return 0 on success, a CUDA error code (as int) after a failed launch,
 * -1 for an unsupported R, or -2 for a shape the tiling cannot describe
 * (rows % R, cols % C or C % 32 non-zero).
 */
#ifndef RANS_B200_H
#define RANS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef __CUDA_RUNTIME_H__
typedef struct CUstream_st* cudaStream_t;
#endif

#define RANS_B200_ABI_VERSION 3   /* 2: escape-code entry points, rans_gemv_step_kernels; 3: chain launcher */

/* ---------------------------------------------------------------- drop-in
 * The three entry points of the reference library, same names, argument
 * meaning and error convention, so a ctypes/cffi/cgo binding written for the
 * reference's librans.so loads this library unchanged.                    */

/* y[rows] (fp32) = code . x  where x (fp32[cols]) is already multiplied by
 * the per-column step.  When cols != C the caller zero-fills y first (the
 * reference accumulates column blocks with atomic adds); when cols == C y is
 * overwritten.  R in {1,2,4,8,16}.
 * Replaces kernel/rans_gemv.cu:146-153 (launch_rans_gemv). */
int launch_rans_gemv(int R, const void* words, const void* offs, const void* table,
                     const void* x, void* y, int rows, int cols, int C,
                     cudaStream_t stream);

/* out (bf16, rows x cols row-major) = bf16(code * step[col]).
 * Replaces kernel/rans_gemv.cu:155-162 (launch_rans_decode). */
int launch_rans_decode(int R, const void* words, const void* offs, const void* table,
                       const void* step, void* out, int rows, int cols, int C,
                       cudaStream_t stream);

/* Fixed-rate 4-bit baseline: w = uint32[rows][cols/8], nibble b of word j
 * holds code+8 of column 8j+b; y[rows] = sum (q-8) * x[col]; cols % 32 == 0.
 * Replaces kernel/rans_gemv.cu:164-170 (launch_int4_gemv). */
int launch_int4_gemv(const void* w, const void* x, void* y, int rows, int cols,
                     cudaStream_t stream);

/* ---------------------------------------------------------------- additive */

/* Same GEMV with the step folded inside the kernel: x is bf16[cols], step is
 * fp32[cols]; y (fp32[rows]) is overwritten (no zero-fill needed).
 * nwords = total length of `words` in words (including the 8 pad words), or
 * -1 when unknown (the final pass is then staged up to the end of the device
 * memory region holding `words`, as for the drop-in entry points).
 * Additive variant of kernel/rans.py:140-152 (RansMatrix.gemv), whose host
 * multiply x.float()*step (rans.py:141) moves into the kernel. */
int rans_gemv_bf16(int R, const void* words, const void* offs, const void* table,
                   const void* x_bf16, const void* step, void* y, int rows, int cols,
                   int C, int64_t nwords, cudaStream_t stream);

/* One encoded matrix (one linear projection) for the step launcher.
 * Device pointers.  x is bf16[cols] when step != NULL, else fp32[cols]
 * already multiplied by the step.  y (fp32[rows]) is overwritten. */
typedef struct RansGemvDesc {
    const void* words;   /* uint16 stream words                     */
    const void* offs;    /* uint32 word offset per stream           */
    const void* table;   /* uint32[4096] slot table (layout above)  */
    const void* x;       /* activation                              */
    const void* step;    /* fp32 per-column step or NULL            */
    void* y;             /* fp32 output                             */
    int64_t nwords;      /* words length incl. pad, or -1 if unknown */
    int32_t rows, cols, C;
    int32_t reserved;    /* must be 0                               */
} RansGemvDesc;

/* Bytes of device workspace the step launcher needs for these n descriptors
 * (all tiled with the same R); negative on a bad R (-1) or shape (-2). */
int64_t rans_gemv_step_workspace_bytes(const RansGemvDesc* descs, int n, int R);

/* Encode the work plan of n matrices (HOST array `descs`) into the caller's
 * device `workspace` and return the launch grid in *grid_out.  Call once, and
 * again whenever a descriptor changes; it synchronises `stream`.  Returns -3
 * when workspace_bytes is too small. */
int rans_gemv_step_plan(const RansGemvDesc* descs, int n, int R, void* workspace,
                        size_t workspace_bytes, int* grid_out, cudaStream_t stream);

/* Row-sharded multi-GPU variant of rans_gemv_step_plan: descs[i] describes
 * this rank's row shard of projection i, and peer_y[i*npeers + p] is the
 * device address (valid on this GPU: NVLink peer mapping / symmetric memory)
 * of the first row of that shard inside rank p's FULL output buffer of
 * projection i, this rank included.  The kernel then stores every output row
 * to all npeers buffers (the all-gather of the outputs is fused into the
 * epilogue; npeers <= 8, one node); the caller
 * runs one cross-GPU barrier after the launch before reading outputs.
 * Replaces the reference's (absent) exchange; no counterpart there. */
int rans_gemv_step_plan_peers(const RansGemvDesc* descs, const void* const* peer_y, int npeers,
                              int n, int R, void* workspace, size_t workspace_bytes,
                              int* grid_out, cudaStream_t stream);

/* Run every projection of a decoder step from ONE grid (capturable in a
 * CUDA graph).  Each CTA loads the slot table of its matrix and its warps
 * decode whole row blocks, so y is stored without atomics.  A plan of two or
 * more waves of work with bf16 activations first runs one small kernel that
 * writes x*step (fp32) into the workspace; rans_gemv_step_kernels tells how
 * many kernels a launch of a planned workspace runs (1 or 2).  No counterpart
 * in the reference: its harness launches one kernel per matrix
 * (kernel/bench.py:104-107, kernel/rans.py:147-151). */
int rans_gemv_step_launch(int R, const void* workspace, int grid, cudaStream_t stream);
int rans_gemv_step_kernels(const void* workspace);

/* ------------------------------------------------------------ chain launcher
 * A decoder step as a chain of dependent phases (per layer {q,k,v} -> o ->
 * {gate,up} -> down: phase p+1 reads what phase p wrote), run from ONE
 * persistent grid.  phase[i] (0..P-1, every phase non-empty) is descriptor
 * i's phase; chunks of phase p start only after every chunk of phase p-1 has
 * finished (and, with `sync`, after every rank has signalled phase p-1).
 * Weights are independent of the previous phase: the table load and each
 * warp's staging of its words overlap it; a warp waits right before its first
 * activation load.  Activations are read with coherent loads after the wait,
 * so phase p+1's x may be phase p's y (the fp32 pre-scaled convention: step
 * NULL).  A bf16 x (step given) must be written before the launch: the kernel
 * turns it into fp32 x*step in the workspace one phase ahead of its use.  No
 * counterpart in the reference, whose harness launches one kernel per matrix
 * (kernel/bench.py:104-107, kernel/rans.py:147-151); this is the layer-level
 * launcher of its survey. */

/* Row-sharded chain over the GPUs of one node (one process per GPU).
 * arrive: this rank's uint32[P+1] arrival counters (the chain may add one
 * phase in front of the caller's for activation prescaling) in memory every
 * rank can write (NVLink peer mapping / symmetric memory); arrive_peer[r]: the address,
 * valid on this GPU, of rank r's counters (this rank included); peer_y as for
 * rans_gemv_step_plan_peers.  Every rank plans (which zeroes its counters),
 * then all ranks pass a host barrier, then every rank launches the same number
 * of times.  A phase's output rows are stored into every rank's buffer, and
 * the phase is complete on a rank once all ranks have added 1 to its counter
 * there.  A faster rank may already run the next launch's first phase while
 * a slower one runs this launch's last, so phase 0's outputs must not be
 * read by the last phase; and nothing waits for the last phase inside the
 * kernel, so its rows from other ranks are complete on this rank only once
 * every rank's launch has ended (synchronise and pass a host barrier). */
typedef struct RansChainSync {
    int32_t nranks;                  /* <= 8 */
    int32_t rank;
    void* arrive;
    void* const* arrive_peer;        /* [nranks] */
    const void* const* peer_y;       /* [n * nranks] */
} RansChainSync;

/* Device workspace bytes for this chain; -1 bad R, -2 bad shape or phases. */
int64_t rans_gemv_chain_workspace_bytes(const RansGemvDesc* descs, const int* phase, int n, int R);

/* The chain's work list as the planner hands it out, without a GPU (no
 * counterpart in the reference: plan introspection for tests and tuning).
 * Writes up to max_chunks records of 8 int32 to `out` (may be NULL), in
 * hand-out order: kernel phase (the caller's phase, plus 1 when an activation
 * prescale phase runs in front); the caller's matrix index; kind (0 decode,
 * 1 activation prescale); then for decode the first item, the item count
 * (at most one per warp of a CTA), tiles per item, streams interleaved per
 * lane and segments per row block (item i covers row block i / segments,
 * tiles [(i % segments) * tiles, ... + tiles) clipped to the matrix), and for
 * prescale the first column and the column count.  Returns the number of
 * chunks, -1 bad R, -2 bad shape or phases. */
int64_t rans_gemv_chain_describe(const RansGemvDesc* descs, const int* phase, int n, int R,
                                 int32_t* out, int64_t max_chunks);

/* Plan the chain into `workspace` (HOST arrays descs, phase; sync NULL on one
 * GPU).  timeout_ms bounds every dependency wait of the kernel.  Returns the
 * launch grid (the CTAs resident at once, at most the number of chunks) in
 * *grid_out.  Synchronises `stream`; -3 when workspace_bytes is too small. */
int rans_gemv_chain_plan(const RansGemvDesc* descs, const int* phase, int n, int R,
                         const RansChainSync* sync, int timeout_ms, void* workspace,
                         size_t workspace_bytes, int* grid_out, cudaStream_t stream);

/* One launch of a planned chain (one kernel). */
int rans_gemv_chain_launch(int R, const void* workspace, int grid, cudaStream_t stream);

/* Synchronises `stream` and reports the chain's state: 0 when every wait of
 * the launches so far ended in time, -5 when one ran out (*phase_out = the
 * phase it waited for, -1 for the activation prescale in front of phase 0;
 * outputs of that launch are incomplete).  Reading -5
 * clears it; until then launches return at once without work.  A multi-GPU
 * chain must then be planned again on every rank. */
int rans_gemv_chain_status(void* workspace, int* phase_out, cudaStream_t stream);

/* The same decoder step for callers that cannot allocate device memory when
 * they run it: a framework whose caching allocator owns the whole pool (a
 * private cudaMalloc would fragment it or fail under pressure), an inference
 * loop that forbids allocation after start-up, a runtime without an allocator
 * handle to hand over.  It plans and launches in one call and allocates
 * nothing: the plan goes to a 256 KB file-scope device array that every GPU
 * loading this library holds until exit, uploaded through kernel launch
 * parameters (no host buffer is read after the call returns).  `descs` is a
 * HOST array of device pointers, as for rans_gemv_step_plan.  The plan is the
 * simple one (whole row blocks per warp), without the split planning of
 * rans_gemv_step_plan: same results, slower small launches.
 * Plan bytes = 32 + 200*n + 16 * sum_i ceil(rows_i / (8*R)); above 256 KB it
 * returns -3 before any GPU work.  At R = 8 a whole 28-layer Qwen2.5-1.5B step
 * (196 matrices, 10,080 chunks) takes about 200 KB; at R = 1 one layer takes
 * about 47 KB, so split such a step into calls of at most five layers.
 * The first call on a device looks up the array's device address with that
 * device current; make that first call before any stream capture.  All calls
 * share the one array, which keeps the last call's plan: calls whose work
 * overlaps on the GPU (for example on different streams) race.  No
 * counterpart in the reference. */
int rans_gemv_step_noalloc(const RansGemvDesc* descs, int n, int R, cudaStream_t stream);

/* ------------------------------------------------------------ host encoder
 * Bit-exact C++ restatement of the reference producer kernel/rans.py:34-98
 * (build_table, lane_order, encode), multithreaded over tiles.            */

/* table[4096] and freq/cum[256] (int32) from int8 codes.  Returns 0, or 1
 * for a single-symbol distribution (kernel/rans.py:45). */
int rans_build_table_host(const int8_t* codes, int64_t n, uint32_t* table,
                          int32_t* freq, int32_t* cum, int nthreads);

/* Upper bound of the words array length for a shape (streams*(n+2)+8). */
int64_t rans_encode_bound(int rows, int cols, int R, int C);

/* Encode int8 codes (row-major rows x cols) with `table`.  Writes offs
 * (one per stream), words (*nwords_out including the 8 pad words, at most
 * words_cap) and per-stream lengths are implied by offs.  Returns 0, -2 for
 * a bad shape, -3 when words_cap is too small. */
int rans_encode_host(const int8_t* codes, int rows, int cols, int R, int C,
                     const uint32_t* table, uint16_t* words, int64_t words_cap,
                     uint32_t* offs, int64_t* nwords_out, int nthreads);

/* ------------------------------------------------------------ escape codes
 * Codes outside [-128, 127] (the reference's encoder rejects them,
 * kernel/rans.py:65-66; "escape codes" are listed as future work in its
 * README) are stored in the stream as an in-range fill code and kept in a
 * sparse list of n (row, col) pairs, int32 each.  No counterpart in the
 * reference.  Both launch one thread per escape on `stream` and return 0, a
 * CUDA error, or -2 for bad arguments. */

/* y[rows[i]] += delta[i] * x'[cols[i]] (atomicAdd), delta = code - fill as
 * fp32.  x' = x (fp32, pre-scaled, the launch_rans_gemv convention) when
 * step is NULL, else bf16 x times fp32 step (the rans_gemv_bf16 convention).
 * Run after the GEMV that wrote y. */
int rans_escape_gemv(const void* rows, const void* cols, const void* delta, int n,
                     const void* x, const void* step, void* y, cudaStream_t stream);

/* out[rows[i] * ncols + cols[i]] = bf16(codes[i] * step[cols[i]]), codes
 * int32.  Run after launch_rans_decode wrote out. */
int rans_escape_decode(const void* rows, const void* cols, const void* codes, int n,
                       const void* step, void* out, int ncols, cudaStream_t stream);

/* ABI version (RANS_B200_ABI_VERSION). */
int rans_b200_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* RANS_B200_H */
