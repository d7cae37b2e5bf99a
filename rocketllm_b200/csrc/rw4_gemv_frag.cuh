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


// ---- fp16 variant for one activation row ------------------------------------------------------
// The two nibbles of a byte feed the tensor cores without a shift between them: under the fp16
// pattern 0x6400 (1024, ulp 1) the low nibble gives 1024 + c and the high nibble, masked in place,
// 1024 + 16 c.  The activation of every high-nibble (odd-k) slot is pre-scaled by 2^-12 and every
// low-nibble (even-k) slot by 2^-8, so both classes contribute 2^-8 * c * x; one shift by 8
// serves the two nibbles of the byte above.  Four codes per shift instead of two per shift.
constexpr uint32_t kMagicF16 = 0x64006400u;   // f16 pair (1024, 1024)
constexpr uint32_t kF16_1 = 0x3C003C00u;      // f16 pair (1, 1): 1 * x 2^-8 = 2^-8 x
constexpr uint32_t kF16_16 = 0x4C004C00u;     // f16 pair (16, 16): 16 * x 2^-12 = 2^-8 x

__device__ __forceinline__ uint32_t nib_lo_f16(uint32_t v) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "n"(0x000F000F), "n"(kMagicF16));
  return r;
}
__device__ __forceinline__ uint32_t nib_hi_f16(uint32_t v) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "n"(0x00F000F0), "n"(kMagicF16));
  return r;
}

// A operand of MMA step j (same slot assignment as a_frag: slots 2t, 2t+1 take nibbles (p, p+4),
// slots 2t+8, 2t+9 nibbles (p+1, p+5), p = 2 (j & 1) of word j >> 1).
__device__ __forceinline__ void a_frag_f16(uint2 wa, uint2 wb, int j, uint32_t (&a)[4]) {
  uint32_t xa = (j < 2) ? wa.x : wa.y;
  uint32_t xb = (j < 2) ? wb.x : wb.y;
  if (j & 1) {
    xa >>= 8;
    xb >>= 8;
  }
  a[0] = nib_lo_f16(xa);
  a[1] = nib_lo_f16(xb);
  a[2] = nib_hi_f16(xa);
  a[3] = nib_hi_f16(xb);
}

// 16 bf16 activations -> the 8 f16 pair registers b[j][0..1] in the K order above, even-k values
// times 2^-8, odd-k values times 2^-12 (exact for |x| >= 2^-6 resp. 2^-2; smaller values keep
// fp16's subnormal spacing 2^-24, i.e. an absolute error below 2^-12 resp. 2^-16).
__device__ __forceinline__ uint32_t f16_pair(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ void x16_to_f16_frag(uint4 lo, uint4 hi, uint32_t (&o)[8]) {
  const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  auto ev = [](uint32_t v) { return __uint_as_float(v << 16) * 0.00390625f; };       // 2^-8
  auto od = [](uint32_t v) { return __uint_as_float(v & 0xFFFF0000u) * 0.000244140625f; };
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    // values 8h .. 8h+7 sit in w[4h .. 4h+3] as (x0 x1)(x2 x3)(x4 x5)(x6 x7)
    o[4 * h + 0] = f16_pair(ev(w[4 * h + 0]), ev(w[4 * h + 2]));  // (x0, x4)
    o[4 * h + 1] = f16_pair(od(w[4 * h + 0]), od(w[4 * h + 2]));  // (x1, x5)
    o[4 * h + 2] = f16_pair(ev(w[4 * h + 1]), ev(w[4 * h + 3]));  // (x2, x6)
    o[4 * h + 3] = f16_pair(od(w[4 * h + 1]), od(w[4 * h + 3]));  // (x3, x7)
  }
}

}  // namespace frag
}  // namespace rw4
