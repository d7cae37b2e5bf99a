// The x-prep workspace shared by the dequant-GEMV (rw4_gemv_tma.cu) and the tcgen05 decode GEMM
// (rw4_gemm_skinny.cu): each activation row converted to fp16 with its own power of two, in the
// fragment order of rw4_gemv_frag.cuh, plus per-group sums (rw4_xprep_kernel).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstddef>

namespace rw4 {

// Byte offsets of the x-prep arrays inside a workspace (each 256-byte aligned).
struct XPrepLayout {
  int64_t Mpad = 0;         // rows padded to even (the side box is 16 bytes wide per row pair)
  size_t xf = 0;            // fp16 [M, K], fragment order within each 16-value chunk
  size_t side = 0;          // fp32 pairs [K/64][Mpad]: (2^e * sum x, -1024 * sum fp16(x 2^e))
  size_t row_exp = 0;       // int32 [Mpad]: e per row
  size_t bytes = 0;         // total
};

XPrepLayout xprep_layout(int64_t M, int64_t K);

// An RMSNorm applied to each row before its conversion: x -> bf16(w * bf16(x * rsqrt(mean(x^2) +
// eps))), the rounding sequence (and summation order) of rw4_rmsnorm.
struct XNorm {
  const void* weight;   // bf16 [K], 16-byte aligned
  float eps;
};

// Launch the conversion of x [M, K] bf16 (RMS-normalised first when `norm` is given) into the
// workspace `ws` laid out as `l` (programmatic dependent launch; the kernel after it may start and
// must wait before reading the workspace).
int xprep_launch(const void* x, int M, int K, const XPrepLayout& l, uint8_t* ws,
                 cudaStream_t stream, const XNorm* norm = nullptr);

}  // namespace rw4
