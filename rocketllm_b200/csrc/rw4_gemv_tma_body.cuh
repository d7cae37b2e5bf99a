// Body of the TMA-fed RW4 dequant-GEMV, shared by the dense entry point (rw4_gemv_tma.cu) and the
// grouped routed-expert entry point (rw4_moe.cu).
//
//   producer warp (one elected lane)      S-stage ring in shared memory          8 consumer warps
//   wait empty[s] ---------------------> codes  [2 boxes x 16R rows x 128 B]  --> wait full[s]
//   expect_tx(full[s]); TMA loads        scales [16R rows x 8 fp16]              copy 2x8 B codes +
//   (cp.async.bulk.tensor.2d, L2        zeros  [16R rows x 8 fp16]              scales + 32 B of x
//    evict-first hint on weights)        x      [2 boxes x BM rows x 256 bf16]   to registers
//                                                                                 arrive empty[s]
//                                                                                 MMA + epilogue
//
// A stage is 512 values of K (8 groups) of the CTA's 16R rows together with the same 512 values of
// the slice's BM activation rows (x travels in the ring with the weights, so no consumer ever
// waits on a global load); consumer warp w always takes group w of the stage, accumulates over all stages, and the 8 partial sums are combined in shared memory
// at the end (deterministic, no atomics, no scratch memory).  Arithmetic: codes enter the tensor
// cores as bf16 (128 + c) (rw4_gemv_frag.cuh), each group's fp32 accumulator is scaled by its
// fp16 scale and the zero term uses the group's sum of x from an all-ones MMA.  The code boxes use
// the 128-byte TMA swizzle (16-byte chunk index XOR row % 8), which keeps the consumers' 8-byte
// shared loads within the two wavefronts 256 bytes need.  Rows past the weight's end are
// zero-filled by the TMA unit and never stored.
//
// SWIGLU variant (R == 2): tile 0 holds rows [r0, r0+16) of the gate half of a stacked gate/up
// weight and tile 1 the matching up rows [r0+I, r0+I+16); the epilogue writes
// bf16(bf16(silu(bf16(g))) * bf16(u)), the rounding sequence of the bf16 model's own
// act_fn(gate) * up (transformers models/mixtral/modeling_mixtral.py:84-91).
//
// K split over a thread-block cluster (KS > 1): the KS CTAs of a cluster take contiguous thirds /
// quarters / halves of the stages of the same rows; every CTA reduces its 8 warps in its own shared
// memory, the CTAs of rank > 0 write their partial sums into rank 0's shared memory through the
// cluster's distributed shared memory, and after one cluster barrier rank 0 adds them and stores.
// More CTAs (and shorter K loops) for short, narrow projections, with no global scratch and no
// atomics.
//
// Every mbarrier wait is bounded (rw4_tma.cuh); on a timeout the CTA drains its own copies, writes
// nothing and sets the library's device status word.
#pragma once

#include <cooperative_groups.h>

#include "rw4_gemv_frag.cuh"
#include "rw4_tma.cuh"

namespace rw4 {
namespace gemv_tma {

constexpr int kConsumers = 8;                 // consumer warps = groups per stage
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kStageK = 64 * kConsumers;      // 512 values of K per stage

template <int R, int S>
struct Layout {
  static constexpr int BR = 16 * R;                   // rows per CTA
  static constexpr int kCodeBox = BR * 128;           // one box: BR rows x 128 bytes (256 k)
  static constexpr int kCodeStage = 2 * kCodeBox;
  static constexpr int kScaleStage = BR * 16;         // BR rows x 8 fp16
  static constexpr int kCodes = 0;
  static constexpr int kScales = S * kCodeStage;
  static constexpr int kZeros = kScales + S * kScaleStage;
  static constexpr int kBars = kZeros + S * kScaleStage;
  static constexpr int kBytes = kBars + 2 * S * 8;
  static constexpr int kStageTx = kCodeStage + 2 * kScaleStage;
  // x ring after the weights: S stages of two [bm rows x 256 bf16] boxes (bm = activation rows
  // of one slice, <= 16, chosen per launch)
  static constexpr int kX = (kBytes + 1023) / 1024 * 1024;
  __host__ __device__ static constexpr int x_stage(int bm) { return bm * 1024; }
  __host__ __device__ static constexpr int dyn_smem(int bm) { return kX + S * x_stage(bm) + 1024; }
};

// Shared-memory loads by shared-window address (always LDS, never a generic load).
__device__ __forceinline__ uint2 lds_v2(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ float lds_half(uint32_t a) {
  unsigned short h;
  asm volatile("ld.shared.b16 %0, [%1];" : "=h"(h) : "r"(a));
  return __half2float(__ushort_as_half(h));
}

// 16 bf16 x values from shared memory (two 16-byte loads), permuted like load_x_frag.
__device__ __forceinline__ void x_frag_smem(uint32_t a, bool valid, uint32_t (&b)[4][2]) {
  uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
  if (valid) {
    lo = lds_v4(a);
    hi = lds_v4(a + 16);
  }
  b[0][0] = __byte_perm(lo.x, lo.z, 0x5410);
  b[0][1] = __byte_perm(lo.x, lo.z, 0x7632);
  b[1][0] = __byte_perm(lo.y, lo.w, 0x5410);
  b[1][1] = __byte_perm(lo.y, lo.w, 0x7632);
  b[2][0] = __byte_perm(hi.x, hi.z, 0x5410);
  b[2][1] = __byte_perm(hi.x, hi.z, 0x7632);
  b[3][0] = __byte_perm(hi.y, hi.w, 0x5410);
  b[3][1] = __byte_perm(hi.y, hi.w, 0x7632);
}

// XT (x by TMA): tm_x maps the activations [rows, K] bf16 with a [bm, 256] box; this slice is its
// rows [x_row0, x_row0 + Ml) (Ml <= bm <= 16; box rows past the tensor's end arrive as zeros, rows
// of the box past Ml are ignored).  Without XT (the routed-expert kernel, whose row count lives on
// the device) the consumers read rows [x_row0, x_row0 + Ml) of x (row stride K) from global memory.
// y: output rows (stride ldy).
// Plain: writes y[m, r0 + r] for r0 + r < n_out.  SWIGLU: writes y[m, r0 + r] for r0 + r < n_out
// (= I) from weight rows r0 + r (gate) and r0 + I + r (up).
// M1: the launch has exactly one activation row (NT == 1, M == 1).
// XF (with M1, without XT): the consumers first convert the CTA's activation row into fp16 pair
// registers in shared memory (x16_to_f16_frag, 1 KB per stage) and the MMAs run in fp16
// (a_frag_f16: one shift per four codes); requires nstages * 1 KB of shared memory at kX.
template <int NT, int R, int S, bool SWIGLU, int KS = 1, bool XT = true, bool M1 = false,
          bool XF = false>
__device__ __forceinline__ void body(const CUtensorMap* tm_codes, const CUtensorMap* tm_scale,
                                     const CUtensorMap* tm_zero, const CUtensorMap* tm_x,
                                     const __nv_bfloat16* __restrict__ x, int x_row0, int bm,
                                     int Ml, int K,
                                     __nv_bfloat16* __restrict__ y, int64_t ldy, int r0,
                                     int n_out, int up_offset, unsigned int* status) {
  using namespace rw4::frag;
  using L = Layout<R, S>;
  static_assert(!SWIGLU || R == 2, "the SwiGLU epilogue pairs one gate tile with one up tile");
  static_assert(!M1 || NT == 1, "one activation row fits one MMA column tile");
  static_assert(!XF || (M1 && !XT), "the fp16 path is the one-row GEMV");
  if (M1) Ml = min(Ml, 1);  // a one-row launch never computes or stores a second row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ int aborted;
  const uint32_t sbase = smem_addr(smem);
  const uint32_t full0 = sbase + L::kBars;
  const uint32_t empty0 = full0 + 8 * S;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // this CTA's range of stages (the whole K unless the cluster splits it)
  int crank = 0;
  if (KS > 1) asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  const int nst_all = K / kStageK;
  const int per = (nst_all + KS - 1) / KS;
  const int s_begin = min(nst_all, crank * per);
  const int nstages = min(nst_all, s_begin + per) - s_begin;

  if (threadIdx.x == 0) {
    aborted = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kConsumers);
    }
    fence_barrier_init();
  }
  __syncthreads();

  float out[R][NT][4];
#pragma unroll
  for (int rt = 0; rt < R; ++rt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) out[rt][nt][e] = 0.f;

  // let the next kernel on the stream begin launching (its CTAs start as ours retire)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == kConsumers) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tensormap(tm_codes);
      prefetch_tensormap(tm_scale);
      prefetch_tensormap(tm_zero);
      if (XT) prefetch_tensormap(tm_x);
      const uint64_t pol = policy_evict_first();
      // Before the dependency on the previous kernel resolves, only pull the first stages' weights
      // into L2 (coherent: if that kernel wrote them, the loads below still see its writes).
      for (int s = 0; s < min(S, nstages); ++s) {
        const int kx = (s_begin + s) * (kStageK / 2);
        tma_prefetch_2d(tm_codes, kx, r0);
        tma_prefetch_2d(tm_codes, kx + 128, r0);
        if (SWIGLU) {
          tma_prefetch_2d(tm_codes, kx, r0 + up_offset);
          tma_prefetch_2d(tm_codes, kx + 128, r0 + up_offset);
        }
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      int issued = 0;
      for (int s = 0; s < nstages; ++s) {
        const int st = s % S;
        const uint32_t par = ((s / S) & 1) ^ 1;
        if (!mbar_wait(empty0 + 8 * st, par, status)) {
          aborted = 1;
          break;
        }
        const uint32_t fb = full0 + 8 * st;
        mbar_arrive_expect_tx(fb, L::kStageTx + (XT ? L::x_stage(bm) : 0));
        const uint32_t cdst = sbase + L::kCodes + st * L::kCodeStage;
        const uint32_t sdst = sbase + L::kScales + st * L::kScaleStage;
        const uint32_t zdst = sbase + L::kZeros + st * L::kScaleStage;
        const int kx = (s_begin + s) * (kStageK / 2);
        const int gx = (s_begin + s) * kConsumers;
        if (XT) {
          const uint32_t xdst = sbase + L::kX + st * L::x_stage(bm);
          tma_load_2d(xdst, tm_x, (s_begin + s) * kStageK, x_row0, fb);
          tma_load_2d(xdst + bm * 512, tm_x, (s_begin + s) * kStageK + 256, x_row0, fb);
        }
        if (SWIGLU) {
          // 16-row boxes: gate tile then up tile (2048 bytes apart, swizzle phase unchanged).
          const int ru = r0 + up_offset;
          tma_load_2d_hint(cdst, tm_codes, kx, r0, fb, pol);
          tma_load_2d_hint(cdst + 2048, tm_codes, kx, ru, fb, pol);
          tma_load_2d_hint(cdst + L::kCodeBox, tm_codes, kx + 128, r0, fb, pol);
          tma_load_2d_hint(cdst + L::kCodeBox + 2048, tm_codes, kx + 128, ru, fb, pol);
          tma_load_2d_hint(sdst, tm_scale, gx, r0, fb, pol);
          tma_load_2d_hint(sdst + 256, tm_scale, gx, ru, fb, pol);
          tma_load_2d_hint(zdst, tm_zero, gx, r0, fb, pol);
          tma_load_2d_hint(zdst + 256, tm_zero, gx, ru, fb, pol);
        } else {
          tma_load_2d_hint(cdst, tm_codes, kx, r0, fb, pol);
          tma_load_2d_hint(cdst + L::kCodeBox, tm_codes, kx + 128, r0, fb, pol);
          tma_load_2d_hint(sdst, tm_scale, gx, r0, fb, pol);
          tma_load_2d_hint(zdst, tm_zero, gx, r0, fb, pol);
        }
        issued = s + 1;
      }
      // Drain: never leave the CTA with copies still landing in its shared memory.
      for (int s = max(0, issued - S); s < issued; ++s)
        mbar_wait(full0 + 8 * (s % S), (s / S) & 1, status);
    }
  } else {
    // ---------------- consumers ----------------
    // The producer loads x only after the previous grid completed; waiting here as well keeps this
    // warp's stores of y behind that grid too (a no-op without a programmatic dependency).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int g = lane >> 2, t = lane & 3;
    const int w = warp;              // group of the stage this warp owns
    const int half = w >> 2, q = w & 3;
    const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    // Shared-window byte offsets that do not change from stage to stage.  Rows 16 rt + g and
    // 16 rt + g + 8 share the swizzle phase g, so every tile's codes sit at a constant stride.
    const uint32_t code_off = L::kCodes + half * L::kCodeBox + g * 128 +
                              (((2 * q + (t >> 1)) ^ g) << 4) + 8 * (t & 1);
    const uint32_t scale_off = L::kScales + g * 16 + 2 * w;
    const uint32_t zero_off = L::kZeros + g * 16 + 2 * w;
    const uint32_t x_off = L::kX + half * bm * 512 + (64 * q + 16 * t) * 2;
    if (XF) {
      // the CTA's activation row -> fp16 pair registers, 32 bytes per 16 values, in shared memory
      const __nv_bfloat16* xr = x + (int64_t)x_row0 * K + (int64_t)s_begin * kStageK;
      const int chunks = nstages * (kStageK / 16);
      for (int c = threadIdx.x; c < chunks; c += kConsumers * 32) {
        uint32_t o[8];
        x16_to_f16_frag(ldg_u4(xr + 16 * c), ldg_u4(xr + 16 * c + 8), o);
        const uint32_t a = sbase + L::kX + 32 * c;
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(o[0]), "r"(o[1]),
                     "r"(o[2]), "r"(o[3]) : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a + 16), "r"(o[4]),
                     "r"(o[5]), "r"(o[6]), "r"(o[7]) : "memory");
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");  // consumers only
    }
    for (int s = 0; s < nstages; ++s) {
      const int st = s % S;
      if (!mbar_wait(full0 + 8 * st, (s / S) & 1, status)) {
        aborted = 1;
        break;
      }
      const uint32_t cb = sbase + code_off + st * L::kCodeStage;
      const uint32_t sb = sbase + scale_off + st * L::kScaleStage;
      const uint32_t zb = sbase + zero_off + st * L::kScaleStage;
      uint2 wa[R], wb[R];
      float s_a[R], s_b[R], z_a[R], z_b[R];
#pragma unroll
      for (int rt = 0; rt < R; ++rt) {
        wa[rt] = lds_v2(cb + rt * 2048);
        wb[rt] = lds_v2(cb + rt * 2048 + 1024);
        s_a[rt] = lds_half(sb + rt * 256);
        s_b[rt] = lds_half(sb + rt * 256 + 128);
        z_a[rt] = lds_half(zb + rt * 256);
        z_b[rt] = lds_half(zb + rt * 256 + 128);
      }
      // x fragment of group (s * 8 + w) (box w / 4 of the stage), then release the slot
      uint32_t b[NT][4][2];
      if (XF) {
        const uint32_t xa = sbase + L::kX + 32 * (32 * s + 4 * w + t);
        const uint4 v0 = lds_v4(xa), v1 = lds_v4(xa + 16);
        b[0][0][0] = v0.x; b[0][0][1] = v0.y; b[0][1][0] = v0.z; b[0][1][1] = v0.w;
        b[0][2][0] = v1.x; b[0][2][1] = v1.y; b[0][3][0] = v1.z; b[0][3][1] = v1.w;
      } else if (XT) {
        const uint32_t xb = sbase + x_off + st * L::x_stage(bm);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int m = nt * 8 + g;
          x_frag_smem(xb + m * 512, m < Ml && m < bm, b[nt]);
        }
      } else {
        const int kofs = (s_begin + s) * kStageK + 64 * w + 16 * t;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int m = nt * 8 + g;
          load_x_frag(x + (int64_t)(x_row0 + min(m, Ml - 1)) * K + kofs, m < Ml, b[nt]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * st);

      // sums of x over the group; the code MMAs start from -128 * sum(x), which removes the
      // +128 of the bf16 code encoding: acc = sum(x * c)
      float xs[NT][4], c0[NT][4];
      if (XF) {
        // 2^-8 sum(x) (A = 1 on even-k slots, 16 on odd-k slots) and the code offset
        // sum(1024 * scaled x) that the code MMAs start from (negated); everything accumulated is
        // then 2^-8 times the true value, undone once per output in the epilogue
        const uint32_t unscale[4] = {kF16_1, kF16_1, kF16_16, kF16_16};
        const uint32_t k1024[4] = {kMagicF16, kMagicF16, kMagicF16, kMagicF16};
        float off[4];
        mma_f16_16816(xs[0], unscale, b[0][0][0], b[0][0][1], zero4);
        mma_f16_16816(off, k1024, b[0][0][0], b[0][0][1], zero4);
#pragma unroll
        for (int j = 1; j < 4; ++j) {
          mma_f16_16816(xs[0], unscale, b[0][j][0], b[0][j][1], xs[0]);
          mma_f16_16816(off, k1024, b[0][j][0], b[0][j][1], off);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) c0[0][e] = -off[e];
      } else {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_bf16_16816(xs[nt], ones, b[nt][0][0], b[nt][0][1], zero4);
#pragma unroll
          for (int j = 1; j < 4; ++j)
            mma_bf16_16816(xs[nt], ones, b[nt][j][0], b[nt][j][1], xs[nt]);
#pragma unroll
          for (int e = 0; e < 4; ++e) c0[nt][e] = -128.f * xs[nt][e];
        }
      }
#pragma unroll
      for (int rt = 0; rt < R; ++rt) {
        float acc[NT][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a[4];
          if (XF) {
            a_frag_f16(wa[rt], wb[rt], j, a);
            mma_f16_16816(acc[0], a, b[0][j][0], b[0][j][1], j == 0 ? c0[0] : acc[0]);
            continue;
          }
          a_frag(wa[rt], wb[rt], j, a);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            if (j == 0)
              mma_bf16_16816(acc[nt], a, b[nt][j][0], b[nt][j][1], c0[nt]);
            else
              mma_bf16_16816(acc[nt], a, b[nt][j][0], b[nt][j][1], acc[nt]);
          }
        }

#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          // one activation row (M1): only column 0 of the MMA tile carries data
          out[rt][nt][0] = fmaf(s_a[rt], acc[nt][0], fmaf(z_a[rt], xs[nt][0], out[rt][nt][0]));
          if (!M1)
            out[rt][nt][1] = fmaf(s_a[rt], acc[nt][1], fmaf(z_a[rt], xs[nt][1], out[rt][nt][1]));
          out[rt][nt][2] = fmaf(s_b[rt], acc[nt][2], fmaf(z_b[rt], xs[nt][2], out[rt][nt][2]));
          if (!M1)
            out[rt][nt][3] = fmaf(s_b[rt], acc[nt][3], fmaf(z_b[rt], xs[nt][3], out[rt][nt][3]));
        }
      }
    }
  }

  // ---- combine the consumer warps' partial sums (ring memory reused) and write bf16 -----------
  __syncthreads();
  constexpr int kCols = 16 * NT + 1;
  constexpr int kRowsOut = SWIGLU ? 16 : L::BR;
  constexpr int kOut = kRowsOut * (M1 ? 1 : 16 * NT);  // one row: only MMA column 0 carries data
  float* red = reinterpret_cast<float*>(smem);  // [kConsumers][BR][kCols]
  if (!aborted && warp < kConsumers) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int rt = 0; rt < R; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float* base = red + (warp * L::BR + 16 * rt + g) * kCols + nt * 8 + 2 * t;
        base[0] = out[rt][nt][0];
        base[1] = out[rt][nt][1];
        base[8 * kCols] = out[rt][nt][2];
        base[8 * kCols + 1] = out[rt][nt][3];
      }
  }
  __syncthreads();
  // per-output partial sums of this CTA (SWIGLU keeps gate and up apart until the final value)
  constexpr int kPer = (kOut + kThreads - 1) / kThreads;
  float part[kPer][SWIGLU ? 2 : 1];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int o = threadIdx.x + i * kThreads;
    const int r = o % kRowsOut, m = o / kRowsOut;
    float a0 = 0.f, a1 = 0.f;
    if (!aborted && o < kOut) {
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        a0 += red[(w * L::BR + r) * kCols + m];
        if (SWIGLU) a1 += red[(w * L::BR + 16 + r) * kCols + m];
      }
    }
    part[i][0] = a0;
    if (SWIGLU) part[i][SWIGLU ? 1 : 0] = a1;
  }
  if (KS > 1) {
    // ranks > 0 deposit their partials in rank 0's shared memory; one cluster barrier
    __shared__ float xred[KS > 1 ? (KS - 1) : 1][kOut][SWIGLU ? 2 : 1];
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    if (crank > 0 && !aborted) {
      float(*dst)[kOut][SWIGLU ? 2 : 1] = cluster.map_shared_rank(xred, 0);
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int o = threadIdx.x + i * kThreads;
        if (o < kOut) {
          dst[crank - 1][o][0] = part[i][0];
          if (SWIGLU) dst[crank - 1][o][SWIGLU ? 1 : 0] = part[i][SWIGLU ? 1 : 0];
        }
      }
    }
    cluster.sync();
    if (crank > 0) return;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int o = threadIdx.x + i * kThreads;
      if (o < kOut) {
#pragma unroll
        for (int j = 0; j < KS - 1; ++j) {
          part[i][0] += xred[j][o][0];
          if (SWIGLU) part[i][SWIGLU ? 1 : 0] += xred[j][o][SWIGLU ? 1 : 0];
        }
      }
    }
  }
  if (aborted) return;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int o = threadIdx.x + i * kThreads;
    const int r = o % kRowsOut, m = o / kRowsOut;
    const int n = r0 + r;
    if (o < kOut && n < n_out && m < Ml) {
      float v;
      if (SWIGLU) {
        const float unit = XF ? 256.f : 1.f;
        const float gb = __bfloat162float(__float2bfloat16_rn(part[i][0] * unit));
        const float ub = __bfloat162float(__float2bfloat16_rn(part[i][SWIGLU ? 1 : 0] * unit));
        const float act = __bfloat162float(__float2bfloat16_rn(gb / (1.f + expf(-gb))));
        v = act * ub;
      } else {
        v = XF ? part[i][0] * 256.f : part[i][0];
      }
      y[(int64_t)m * ldy + n] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace gemv_tma
}  // namespace rw4
