// Register-fragment helpers shared by the RW4 GEMV kernels (mma.sync m16n8k16, bf16 in, fp32
// accumulate).  See rw4_gemv.cu for the K-permutation argument: the 16 K-slots of one MMA are the
// 16 codes of one thread's 8-byte slice of a row, in the order a shift + LOP3 extracts them, and the
// activation fragment is permuted identically.
#pragma once

#include "rw4_common.cuh"

namespace rw4 {
namespace frag {

constexpr uint32_t kMagic = 0x43004300u;   // bf16 pair (128, 128)
constexpr uint32_t kOnes = 0x3F803F80u;    // bf16 pair (1, 1)

// Codes of nibbles (p, p+4) of `word` as a bf16 pair (128 + c_p, 128 + c_{p+4}).
__device__ __forceinline__ uint32_t nib_pair(uint32_t word, int shift) {
  uint32_t r;
  const uint32_t v = word >> shift;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "n"(0x000F000F), "n"(kMagic));
  return r;
}

// x fragment for one group: 16 bf16 values x[16t .. 16t+16) of the thread's batch row, permuted
// to the K order the code extraction produces.  b[j][0..1] are the two B registers of MMA step j.
__device__ __forceinline__ void load_x_frag(const __nv_bfloat16* xrow, bool valid,
                                            uint32_t (&b)[4][2]) {
  uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
  if (valid) {
    lo = ldg_u4(xrow);
    hi = ldg_u4(xrow + 8);
  }
  // natural pairs: lo = (x0,x1)(x2,x3)(x4,x5)(x6,x7); hi = (x8,x9)..(x14,x15)
  b[0][0] = __byte_perm(lo.x, lo.z, 0x5410);  // (x0, x4)
  b[0][1] = __byte_perm(lo.x, lo.z, 0x7632);  // (x1, x5)
  b[1][0] = __byte_perm(lo.y, lo.w, 0x5410);  // (x2, x6)
  b[1][1] = __byte_perm(lo.y, lo.w, 0x7632);  // (x3, x7)
  b[2][0] = __byte_perm(hi.x, hi.z, 0x5410);  // (x8, x12)
  b[2][1] = __byte_perm(hi.x, hi.z, 0x7632);  // (x9, x13)
  b[3][0] = __byte_perm(hi.y, hi.w, 0x5410);  // (x10, x14)
  b[3][1] = __byte_perm(hi.y, hi.w, 0x7632);  // (x11, x15)
}

// A operand of MMA step j for the thread's two rows (g: word wa, g+8: word wb).
//   reg0 = row g,   logical k (2t, 2t+1)   <- nibbles (p,   p+4)
//   reg1 = row g+8, logical k (2t, 2t+1)   <- nibbles (p,   p+4)
//   reg2 = row g,   logical k (2t+8, 2t+9) <- nibbles (p+1, p+5)
//   reg3 = row g+8, logical k (2t+8, 2t+9) <- nibbles (p+1, p+5)
// with p = 2 (j & 1) inside word j >> 1 of the thread's 8-byte slice.
__device__ __forceinline__ void a_frag(uint2 wa, uint2 wb, int j, uint32_t (&a)[4]) {
  const uint32_t xa = (j < 2) ? wa.x : wa.y;
  const uint32_t xb = (j < 2) ? wb.x : wb.y;
  const int p = (j & 1) * 2;
  a[0] = nib_pair(xa, 4 * p);
  a[1] = nib_pair(xb, 4 * p);
  a[2] = nib_pair(xa, 4 * p + 4);
  a[3] = nib_pair(xb, 4 * p + 4);
}


}  // namespace frag
}  // namespace rw4
