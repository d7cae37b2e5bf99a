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


// ---- fp16 variant (dense path: activations converted per row, rw4_gemv_tma.cu) -------------
// The two nibbles of a byte feed the tensor cores without a shift between them: under the fp16
// pattern 0x6400 (1024, ulp 1) the low nibble gives 1024 + c and the high nibble, masked in place,
// 1024 + 16 c.  The activation of every high-nibble (odd-k) slot therefore carries an extra 2^-4
// relative to the low-nibble (even-k) slots, so both classes contribute c * x times the row's
// common power of two; one shift by 8 serves the two nibbles of the byte above.  Four codes per
// shift instead of two per shift.
constexpr uint32_t kMagicF16 = 0x64006400u;   // f16 pair (1024, 1024)

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

__device__ __forceinline__ uint32_t f16_pair(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// 16 bf16 activations (natural order, two 16-byte words) -> the 8 fp16 pair registers
// o[2j], o[2j+1] = B operand of MMA step j in the K order of a_frag_f16, even-k values times
// 2^e and odd-k values times 2^(e-4).  The power of two is applied as two exact multiplications
// (p1 * p2 = 2^e, p1 and p2 normal fp32 for any exponent a bf16 row can need), so the result is
// x * 2^e rounded once to fp16 -- exact whenever that value is an fp16 normal.
// Also returns the chunk's two sums, each added in natural order: xs = sum of x * 2^e (exact
// products) and hs = sum of the 16 fp16 values as the tensor cores will see them.
__device__ __forceinline__ void x16_to_f16_frag(uint4 lo, uint4 hi, float p1, float p2,
                                                uint32_t (&o)[8], float& xs, float& hs) {
  const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  const float p2o = p2 * 0.0625f;  // odd slots: 2^(e-4)
  auto ev = [&](uint32_t v) { return (__uint_as_float(v << 16) * p1) * p2; };
  auto od = [&](uint32_t v) { return (__uint_as_float(v & 0xFFFF0000u) * p1) * p2o; };
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    // values 8h .. 8h+7 sit in w[4h .. 4h+3] as (x0 x1)(x2 x3)(x4 x5)(x6 x7)
    o[4 * h + 0] = f16_pair(ev(w[4 * h + 0]), ev(w[4 * h + 2]));  // (x0, x4)
    o[4 * h + 1] = f16_pair(od(w[4 * h + 0]), od(w[4 * h + 2]));  // (x1, x5)
    o[4 * h + 2] = f16_pair(ev(w[4 * h + 1]), ev(w[4 * h + 3]));  // (x2, x6)
    o[4 * h + 3] = f16_pair(od(w[4 * h + 1]), od(w[4 * h + 3]));  // (x3, x7)
  }
  xs = 0.f;
  hs = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {  // 2^e * x exactly (power-of-two scaling of a bf16 value)
    xs += ev(w[i]);
    xs += (__uint_as_float(w[i] & 0xFFFF0000u) * p1) * p2;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __half2 h2 = *reinterpret_cast<const __half2*>(&o[i]);
    hs += __low2float(h2);
    hs += __high2float(h2);
  }
}

// Sums of a group of 64 from its four chunks, held by lanes 4j .. 4j+3 of a warp (every lane of the
// warp must call this): one butterfly, the same order on every lane and in every kernel.
__device__ __forceinline__ void group_sums(float& xs, float& hs) {
  xs += __shfl_xor_sync(0xFFFFFFFFu, xs, 1);
  xs += __shfl_xor_sync(0xFFFFFFFFu, xs, 2);
  hs += __shfl_xor_sync(0xFFFFFFFFu, hs, 1);
  hs += __shfl_xor_sync(0xFFFFFFFFu, hs, 2);
}

// Largest |x| of 8 bf16 values as a bit pattern (bf16 magnitudes order like their bit patterns).
__device__ __forceinline__ uint32_t absmax8(uint4 v) {
  const uint32_t m2 = __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                               __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
  return max(m2 & 0xFFFFu, m2 >> 16);
}

// The row's exponent e: its largest magnitude (bf16 bits) times 2^e lies in [2^14, 2^15), so every
// even-k value x 2^e and odd-k value x 2^(e-4) fits fp16.  An all-zero row, or one holding inf or
// NaN, keeps e = 0.
__device__ __forceinline__ int row_exponent(uint32_t maxbits) {
  return (maxbits != 0 && maxbits < 0x7F80u) ? 14 - ilogbf(__uint_as_float(maxbits << 16)) : 0;
}

// 2^e as two fp32 normals (|e| <= 147 for any bf16 row).
__device__ __forceinline__ void exp_factors(int e, float& p1, float& p2) {
  const int e1 = e >> 1, e2 = e - e1;
  p1 = __int_as_float((127 + e1) << 23);
  p2 = __int_as_float((127 + e2) << 23);
}

// bf16(w * bf16(x * r)) for 8 values: RMSNorm's scaling, rounded as rw4_rmsnorm rounds it.
__device__ __forceinline__ uint4 norm8(uint4 xv, uint4 wv, float r) {
  const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w}, ws[4] = {wv.x, wv.y, wv.z, wv.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float a = __bfloat162float(__float2bfloat16_rn(__uint_as_float(xs[j] << 16) * r));
    const float b = __bfloat162float(__float2bfloat16_rn(__uint_as_float(xs[j] & 0xFFFF0000u) * r));
    const __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(ws[j] << 16) * a,
                                                  __uint_as_float(ws[j] & 0xFFFF0000u) * b);
    o[j] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// RMSNorm's 1 / rms of one row of K values, summed in rw4_rmsnorm's order: 256 threads (tid) each
// take elements tid, tid + 256, ... in turn, then the warp butterfly, then the 8 warps' sums in
// order.  `part` is 8 floats of shared memory; `sync` a barrier over exactly those 256 threads.
template <typename Sync>
__device__ __forceinline__ float rms_scale(const __nv_bfloat16* __restrict__ xr, int K, float eps,
                                           int tid, float* part, Sync sync) {
  float ss = 0.f;
  for (int i = tid; i < K; i += 256) {
    const float v = __bfloat162float(xr[i]);
    ss = fmaf(v, v, ss);
  }
  ss += __shfl_xor_sync(0xFFFFFFFFu, ss, 16);
  ss += __shfl_xor_sync(0xFFFFFFFFu, ss, 8);
  ss += __shfl_xor_sync(0xFFFFFFFFu, ss, 4);
  ss += __shfl_xor_sync(0xFFFFFFFFu, ss, 2);
  ss += __shfl_xor_sync(0xFFFFFFFFu, ss, 1);
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  sync();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += part[w];
  return rsqrtf(tot / (float)K + eps);
}

}  // namespace frag
}  // namespace rw4
