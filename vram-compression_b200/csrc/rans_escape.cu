// Escape codes: integer codes outside the 8-bit alphabet of the rANS tables.
//
// The reference encoder accepts codes in [-128, 127] only (kernel/rans.py:65-66
// asserts) and lists escape codes as future work (README.md "Next").  Here an
// out-of-range code is stored in the stream as a fill code (any in-range value,
// normally the most frequent one, so it costs few bits) and kept exactly in a
// sparse side list (row, col, code).  Results are then completed by two small
// kernels that run after the fused GEMV / the decode on the same stream:
//
//   GEMV:   y[row] += (code - fill) * x'[col]          (x' = x * step)
//   decode: out[row, col] = bf16(code * step[col])
//
// so the dense result equals the one of the unclipped codes (GEMV up to fp32
// summation order).  Escapes are rare (outliers), one thread each.
#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/rans_b200.h"

namespace {

constexpr int kEscThreads = 256;

__global__ void escape_gemv_kernel(const int32_t* __restrict__ rows, const int32_t* __restrict__ cols,
                                   const float* __restrict__ delta, int n, const void* __restrict__ x,
                                   const float* __restrict__ step, float* __restrict__ y) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int c = cols[i];
    float xv;
    if (step != nullptr) {
        xv = __bfloat162float(static_cast<const __nv_bfloat16*>(x)[c]) * step[c];
    } else {
        xv = static_cast<const float*>(x)[c];
    }
    atomicAdd(y + rows[i], delta[i] * xv);
}

__global__ void escape_decode_kernel(const int32_t* __restrict__ rows, const int32_t* __restrict__ cols,
                                     const int32_t* __restrict__ codes, int n, const float* __restrict__ step,
                                     __nv_bfloat16* __restrict__ out, int ncols) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int c = cols[i];
    out[(int64_t)rows[i] * ncols + c] = __float2bfloat16(static_cast<float>(codes[i]) * step[c]);
}

}  // namespace

extern "C" int rans_escape_gemv(const void* rows, const void* cols, const void* delta, int n, const void* x,
                                const void* step, void* y, cudaStream_t stream) {
    if (n < 0) return -2;
    if (n == 0) return 0;
    if (rows == nullptr || cols == nullptr || delta == nullptr || x == nullptr || y == nullptr) return -2;
    escape_gemv_kernel<<<(n + kEscThreads - 1) / kEscThreads, kEscThreads, 0, stream>>>(
        static_cast<const int32_t*>(rows), static_cast<const int32_t*>(cols), static_cast<const float*>(delta), n,
        x, static_cast<const float*>(step), static_cast<float*>(y));
    return (int)cudaGetLastError();
}

extern "C" int rans_escape_decode(const void* rows, const void* cols, const void* codes, int n, const void* step,
                                  void* out, int ncols, cudaStream_t stream) {
    if (n < 0 || ncols <= 0) return -2;
    if (n == 0) return 0;
    if (rows == nullptr || cols == nullptr || codes == nullptr || step == nullptr || out == nullptr) return -2;
    escape_decode_kernel<<<(n + kEscThreads - 1) / kEscThreads, kEscThreads, 0, stream>>>(
        static_cast<const int32_t*>(rows), static_cast<const int32_t*>(cols), static_cast<const int32_t*>(codes), n,
        static_cast<const float*>(step), static_cast<__nv_bfloat16*>(out), ncols);
    return (int)cudaGetLastError();
}
