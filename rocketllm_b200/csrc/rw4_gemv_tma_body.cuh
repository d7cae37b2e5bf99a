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
// waits on a global load); consumer warp w always takes group w of the stage, accumulates over all
// stages, and the 8 partial sums are combined in shared memory at the end (deterministic, no
// atomics).  Arithmetic of the routed-expert path (bf16 activations): codes enter the tensor cores
// as bf16 (128 + c) (rw4_gemv_frag.cuh), each group's fp32 accumulator is scaled by its fp16 scale
// and the zero term uses the group's sum of x from an all-ones MMA.  The dense path (XP / XQ,
// below) multiplies fp16 codes by pre-converted activations instead.  The code boxes use
// the 128-byte TMA swizzle (16-byte chunk index XOR row % 8), which keeps the consumers' 8-byte
// shared loads within the two wavefronts 256 bytes need.  Rows past the weight's end are
// zero-filled by the TMA unit and never stored.
//
// SWIGLU variant (R even): tiles 0 .. R/2-1 hold rows [r0, r0+8R) of the gate half of a stacked
// gate/up weight and tiles R/2 .. R-1 the matching up rows [r0+I, r0+I+8R); the epilogue writes
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
// XP (the dense decode path): the activations arrive already converted by the x-prep kernel
// (rw4_gemv_tma.cu) -- fp16, each row scaled by its own power of two 2^e so that its largest
// magnitude lies in [2^14, 2^15), even-k values by 2^e and odd-k values by 2^(e-4), every 16-value
// chunk permuted into MMA fragment order -- together with two fp32 numbers per (group, row): the
// group's sum of x times 2^e and minus 1024 times the sum of its fp16 values (the code offset).
// The codes then enter the tensor cores as fp16 (1024 + c) and (1024 + 16 c) straight from one LOP3
// each (a_frag_f16), the accumulator starts from the offset, and the row's 2^-e is applied once
// when the output is stored.  Every row is converted the same way whatever the batch, so a row's
// output does not depend on the rows beside it or on the launch's M, and scaling x by a power of
// two scales the output by exactly that power (no fixed pre-scale, no fp16 underflow of small
// activations).  XQ does the same conversion inside the GEMV for a one-row launch.
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
  // XP: per-(group, row) fp32 pairs of the stage's 8 groups for the slice's rows padded to even
  __host__ __device__ static constexpr int side_rows(int bm) { return (bm + 1) & ~1; }
  __host__ __device__ static constexpr int side_stage(int bm) { return 64 * side_rows(bm); }
  __host__ __device__ static constexpr int side_base(int bm) { return kX + S * x_stage(bm); }
  __host__ __device__ static constexpr int dyn_smem_xp(int bm) {
    return kX + S * (x_stage(bm) + side_stage(bm)) + 1024;
  }
  // XQ: the CTA's converted activation row (1 KB per stage) and its (sum, -offset) pairs (64 B per
  // stage) for up to kXQMaxStages stages
  static constexpr int kXQMaxStages = 32;
  static constexpr int kXQSide = kX + kXQMaxStages * 1024;
  __host__ __device__ static constexpr int dyn_smem_xq(int nstages) {
    return kXQSide + nstages * 64 + 1024;
  }
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
// XP (implies the TMA ring): tm_x maps the x-prep output [rows, K] fp16 with the same box, tm_side
// its per-(group, row) pairs [K/64, 2 * padded rows] fp32 with an [8, 2 * side_rows(bm)] box, and
// row_exp[x_row0 + m] is row m's exponent e (the output is scaled by 2^-e).
// XQ (one activation row, M1, without the ring): the consumers convert the row themselves before
// the first stage -- its exponent from the whole row's largest magnitude, then this CTA's K range
// into fp16 fragments and (sum, -offset) pairs in shared memory -- with the same helpers, in the
// same order, as the x-prep kernel, so the output has the same bits as the XP path's.  x is the
// bf16 activations (row x_row0, stride K).
// nw, eps (XQ only; nw may be null): the row is first normalised as rw4_rmsnorm does it --
// bf16(nw * bf16(x * r)), r from the row's mean square summed in that kernel's order -- so the
// output has the bits of rw4_rmsnorm followed by the GEMV.
// y: output rows (stride ldy); res (XP / XQ only, may be null): rows added to the output in the
// model's bf16 order, bf16(bf16(x . W^T) + res) -- a decoder layer's residual connection.
// Plain: writes y[m, r0 + r] for r0 + r < n_out.  SWIGLU: writes y[m, r0 + r] for r0 + r < n_out
// (= I) from weight rows r0 + r (gate) and r0 + up_offset + r (up): bf16(bf16(silu(bf16(gate))) *
// bf16(up)), the bits of the plain GEMV over both followed by rw4_silu_mul.
// M1: the launch has exactly one activation row (NT == 1, M == 1).
template <int NT, int R, int S, bool SWIGLU, int KS = 1, bool XT = true, bool M1 = false,
          bool XP = false, bool XQ = false>
__device__ __forceinline__ void body(const CUtensorMap* tm_codes, const CUtensorMap* tm_scale,
                                     const CUtensorMap* tm_zero, const CUtensorMap* tm_x,
                                     const CUtensorMap* tm_side, const int* __restrict__ row_exp,
                                     const __nv_bfloat16* __restrict__ x, int x_row0, int bm,
                                     int Ml, int K,
                                     __nv_bfloat16* __restrict__ y, int64_t ldy, int r0,
                                     int n_out, int up_offset, unsigned int* status,
                                     const __nv_bfloat16* __restrict__ res = nullptr,
                                     const __nv_bfloat16* __restrict__ nw = nullptr,
                                     float eps = 0.f) {
  using namespace rw4::frag;
  using L = Layout<R, S>;
  static_assert(!SWIGLU || R % 2 == 0, "the SwiGLU epilogue pairs gate tiles with up tiles");
  static_assert(!M1 || NT == 1, "one activation row fits one MMA column tile");
  static_assert(!XP || XT, "the pre-converted activations come through the ring");
  static_assert(!XQ || (M1 && !XT && !XP), "XQ converts one activation row");
  if (M1) Ml = min(Ml, 1);  // a one-row launch never computes or stores a second row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ int aborted;
  __shared__ int xq_exp;  // XQ: the row's exponent, for every thread of the final store
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
    xq_exp = 0;
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
      if (XP) prefetch_tensormap(tm_side);
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
        mbar_arrive_expect_tx(fb, L::kStageTx + (XT ? L::x_stage(bm) : 0) +
                                      (XP ? L::side_stage(bm) : 0));
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
        if (XP)  // the stage's 8 groups x the slice's rows: (sum of x, -offset) pairs
          tma_load_2d(sbase + L::side_base(bm) + st * L::side_stage(bm), tm_side, 2 * x_row0, gx,
                      fb);
        if (SWIGLU) {
          // 8R-row boxes: gate rows then up rows (2048 R/2 bytes apart, swizzle phase unchanged).
          const int ru = r0 + up_offset;
          constexpr int kUp = 2048 * (R / 2), kUpS = 256 * (R / 2);
          tma_load_2d_hint(cdst, tm_codes, kx, r0, fb, pol);
          tma_load_2d_hint(cdst + kUp, tm_codes, kx, ru, fb, pol);
          tma_load_2d_hint(cdst + L::kCodeBox, tm_codes, kx + 128, r0, fb, pol);
          tma_load_2d_hint(cdst + L::kCodeBox + kUp, tm_codes, kx + 128, ru, fb, pol);
          tma_load_2d_hint(sdst, tm_scale, gx, r0, fb, pol);
          tma_load_2d_hint(sdst + kUpS, tm_scale, gx, ru, fb, pol);
          tma_load_2d_hint(zdst, tm_zero, gx, r0, fb, pol);
          tma_load_2d_hint(zdst + kUpS, tm_zero, gx, ru, fb, pol);
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
    // warp's reads of x and stores of y behind that grid too (a no-op without a programmatic
    // dependency).
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
    const int srows = L::side_rows(bm);
    const uint32_t side_off = L::side_base(bm) + w * srows * 8;
    if (XQ) {
      // One pass over the row: this CTA's K range is loaded once into registers (at most 4
      // chunks of 16 per thread) and its largest magnitude taken there; with a K split the rest of
      // the row is read only for its maximum.  Then the range is converted from the registers.
      constexpr int kPer = L::kXQMaxStages * (kStageK / 16) / (kConsumers * 32);
      const int tid = threadIdx.x;
      const __nv_bfloat16* xr = x + (int64_t)x_row0 * K;
      const __nv_bfloat16* xk = xr + (int64_t)s_begin * kStageK;
      const int chunks = nstages * (kStageK / 16);
      static_assert(kConsumers == 8, "rms_scale sums over 256 threads");
      float r = 1.f;
      if (nw) {
        __shared__ float wss[kConsumers];
        r = rms_scale(xr, K, eps, tid, wss, [] {
          asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
        });
      }
      const __nv_bfloat16* nwk = nw ? nw + (int64_t)s_begin * kStageK : nullptr;
      uint4 lo[kPer], hi[kPer];
      uint32_t mx = 0;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int c = tid + kConsumers * 32 * i;
        lo[i] = make_uint4(0, 0, 0, 0);
        hi[i] = lo[i];
        if (c < chunks) {
          lo[i] = ldg_u4(xk + 16 * c);
          hi[i] = ldg_u4(xk + 16 * c + 8);
          if (nw) {
            lo[i] = norm8(lo[i], ldg_u4(nwk + 16 * c), r);
            hi[i] = norm8(hi[i], ldg_u4(nwk + 16 * c + 8), r);
          }
          mx = max(mx, max(absmax8(lo[i]), absmax8(hi[i])));
        }
      }
      if (KS > 1) {
        const int k0 = s_begin * kStageK, k1 = (s_begin + nstages) * kStageK;
        for (int i = tid; i < K / 8; i += kConsumers * 32)
          if (8 * i < k0 || 8 * i >= k1) {
            uint4 v = ldg_u4(xr + 8 * i);
            if (nw) v = norm8(v, ldg_u4(nw + 8 * i), r);
            mx = max(mx, absmax8(v));
          }
      }
      mx = __reduce_max_sync(0xFFFFFFFFu, mx);
      __shared__ uint32_t wmax[kConsumers];
      if (lane == 0) wmax[warp] = mx;
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");  // consumers only
      uint32_t a = 0;
#pragma unroll
      for (int i = 0; i < kConsumers; ++i) a = max(a, wmax[i]);
      const int e = row_exponent(a);
      if (tid == 0) xq_exp = e;
      float p1, p2;
      exp_factors(e, p1, p2);
      // this CTA's K range -> fp16 fragments (32 bytes per 16 values) and per-group pairs; the
      // 4 chunks of a group sit on 4 consecutive lanes, as in the x-prep kernel
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        if (kConsumers * 32 * i >= chunks) break;   // uniform over the CTA
        const int c = tid + kConsumers * 32 * i;
        float xs_c = 0.f, hs_c = 0.f;
        if (c < chunks) {
          uint32_t o[8];
          x16_to_f16_frag(lo[i], hi[i], p1, p2, o, xs_c, hs_c);
          const uint32_t a0 = sbase + L::kX + 32 * c;
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a0), "r"(o[0]), "r"(o[1]),
                       "r"(o[2]), "r"(o[3]) : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a0 + 16), "r"(o[4]),
                       "r"(o[5]), "r"(o[6]), "r"(o[7]) : "memory");
        }
        group_sums(xs_c, hs_c);
        if (c < chunks && (c & 3) == 0) {
          float* sd = reinterpret_cast<float*>(smem + L::kXQSide) + 2 * (c >> 2);
          sd[0] = xs_c;
          sd[1] = -1024.f * hs_c;
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
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
      // x fragment of group (s * 8 + w) (box w / 4 of the stage)
      uint32_t b[NT][4][2];
      float xs[NT][4], c0[NT][4];
      if (XQ) {
        // column 0 (g == 0) carries the row, the others zeros -- as the XP ring delivers it
        uint4 v0 = make_uint4(0, 0, 0, 0), v1 = make_uint4(0, 0, 0, 0);
        if (g == 0) {
          const uint32_t xa = sbase + L::kX + 32 * (32 * s + 4 * w + t);
          v0 = lds_v4(xa);
          v1 = lds_v4(xa + 16);
        }
        b[0][0][0] = v0.x; b[0][0][1] = v0.y; b[0][1][0] = v0.z; b[0][1][1] = v0.w;
        b[0][2][0] = v1.x; b[0][2][1] = v1.y; b[0][3][0] = v1.z; b[0][3][1] = v1.w;
        float sx = 0.f, so = 0.f;
        if (t == 0) {
          const float* sd = reinterpret_cast<const float*>(smem + L::kXQSide) + 2 * (8 * s + w);
          sx = sd[0];
          so = sd[1];
        }
        xs[0][0] = xs[0][2] = sx;
        xs[0][1] = xs[0][3] = 0.f;
        c0[0][0] = c0[0][2] = so;
        c0[0][1] = c0[0][3] = 0.f;
      } else if (XP) {
        const uint32_t xb = sbase + x_off + st * L::x_stage(bm);
        const uint32_t sd = sbase + side_off + st * L::side_stage(bm);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          // fp16 pairs already in fragment order: two 16-byte loads, no permutes
          const int m = nt * 8 + g;
          uint4 v0 = make_uint4(0, 0, 0, 0), v1 = make_uint4(0, 0, 0, 0);
          if (m < Ml && m < bm) {
            v0 = lds_v4(xb + m * 512);
            v1 = lds_v4(xb + m * 512 + 16);
          }
          b[nt][0][0] = v0.x; b[nt][0][1] = v0.y; b[nt][1][0] = v0.z; b[nt][1][1] = v0.w;
          b[nt][2][0] = v1.x; b[nt][2][1] = v1.y; b[nt][3][0] = v1.z; b[nt][3][1] = v1.w;
          // (sum of x, -offset) of this group for accumulator columns 2t and 2t + 1
          const int col = nt * 8 + 2 * t;
          uint4 sv = make_uint4(0, 0, 0, 0);
          if (col < srows) sv = lds_v4(sd + col * 8);
          xs[nt][0] = xs[nt][2] = __uint_as_float(sv.x);
          xs[nt][1] = xs[nt][3] = __uint_as_float(sv.z);
          c0[nt][0] = c0[nt][2] = __uint_as_float(sv.y);
          c0[nt][1] = c0[nt][3] = __uint_as_float(sv.w);
        }
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

      if (!XP && !XQ) {
        // sums of x over the group; the code MMAs start from -128 * sum(x), which removes the
        // +128 of the bf16 code encoding: acc = sum(x * c)
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
          if (XP || XQ)
            a_frag_f16(wa[rt], wb[rt], j, a);
          else
            a_frag(wa[rt], wb[rt], j, a);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            if (XP || XQ)
              mma_f16_16816(acc[nt], a, b[nt][j][0], b[nt][j][1], j == 0 ? c0[nt] : acc[nt]);
            else
              mma_bf16_16816(acc[nt], a, b[nt][j][0], b[nt][j][1], j == 0 ? c0[nt] : acc[nt]);
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
      // Release the slot only now: every value this thread read from it has been consumed by the
      // MMAs and FMAs above, so its shared-memory reads are complete before the producer's TMA
      // (async proxy) can refill the slot.  (Released right after the reads, a refill could
      // overtake reads still in flight -- the tcgen05 GEMM's codes ring showed exactly that.)
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * st);
    }
  }

  // ---- combine the consumer warps' partial sums (ring memory reused) and write bf16 -----------
  __syncthreads();
  constexpr int kCols = 16 * NT + 1;
  constexpr int kRowsOut = SWIGLU ? L::BR / 2 : L::BR;
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
        if (SWIGLU) a1 += red[(w * L::BR + kRowsOut + r) * kCols + m];
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
  const int xq_e = XQ ? xq_exp : 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int o = threadIdx.x + i * kThreads;
    const int r = o % kRowsOut, m = o / kRowsOut;
    const int n = r0 + r;
    if (o < kOut && n < n_out && m < Ml) {
      float v;
      if (SWIGLU) {
        // gate and up as the plain GEMV rounds them (after the row's 2^-e on the fp16 paths),
        // then act_fn(gate) * up as the model rounds it
        float gv = part[i][0], uv = part[i][SWIGLU ? 1 : 0];
        if (XP || XQ) {
          const int e = XQ ? xq_e : row_exp[x_row0 + m];
          gv = ldexpf(gv, -e);
          uv = ldexpf(uv, -e);
        }
        const float gb = __bfloat162float(__float2bfloat16_rn(gv));
        const float ub = __bfloat162float(__float2bfloat16_rn(uv));
        const float act = __bfloat162float(__float2bfloat16_rn(gb / (1.f + expf(-gb))));
        v = act * ub;
      } else if (XP || XQ) {
        // undo the row's 2^e (exact)
        v = ldexpf(part[i][0], XQ ? -xq_e : -row_exp[x_row0 + m]);
        // residual (same layout as y): the model's bf16 `residual + linear(x)`, i.e. the product
        // rounded to bf16 first, then the sum
        if (res) v = __bfloat162float(__float2bfloat16_rn(v)) +
                     __bfloat162float(res[(int64_t)m * ldy + n]);
      } else {
        v = part[i][0];
      }
      y[(int64_t)m * ldy + n] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace gemv_tma
}  // namespace rw4
