// Decode attention straight over the int4 (KIVI-layout) KV cache.
//
// The reference keeps K quantized per channel over groups of 64 tokens and V per token over
// groups of 64 channels (rocketllm/quant/kv_cache.py:146-221), plus a window of the most recent
// tokens in the compute dtype, and before every attention call it expands the whole history back
// to the compute dtype (kv_cache.py:308-316).  This kernel reads the packed history directly.
//
// Device layout of one (batch, kv head) "head slot" hs (all arrays contiguous):
//   k_codes [hs][gcap][D][32]  u8   group-major: the 64 tokens of group g, channel c, two per byte
//   k_sz    [hs][gcap][D][2]   f16  (scale, zero) of channel c over group g
//   v_codes [hs][gcap*64][D/2] u8   token-major, two channels per byte
//   v_sz    [hs][gcap*64][D/64][2] f16 (scale, zero) of a token's 64-channel group
//   k_res / v_res [hs][rcap][D] bf16  the residual window, rlen tokens valid
// The reference's block tensors are views of these (a permutation of the group axis for K).
//
// Work: one item = one 64-token group (or 64-token chunk of the window).  A (rank, kv head)
// thread-block cluster of S CTAs x 8 warps shares the items of one head slot round-robin; each
// warp streams its groups through a private two-stage shared-memory ring fed by 1-D bulk copies
// (cp.async.bulk, completion on an mbarrier, every wait bounded) and keeps its own online-softmax
// state; warps combine in shared memory, CTAs through distributed shared memory (no global
// scratch).
//
// Math per group (head dim D, query heads of the kv head as the n8 columns, tokens / channels as
// the m16 rows of mma.sync m16n8k16):
//   S^T[t, j] = sum_c K[t, c] q'[j, c],  K[t, c] = code * s_c + z_c
//            = sum_c code[t, c] (q'[j, c] s_c) + sum_c q'[j, c] z_c
// so the per-channel scale folds into the fp16 B operand (q' s), the codes enter the A operand as
// exact fp16 integers, and the zero term is an fp32 dot product per head.  Likewise for V, whose
// per-token scale folds into the B operand P s_t after the probabilities are transposed into B
// fragments (movmatrix), and sum_t P z_t is accumulated in fp32.  Codes are widened with one
// byte_perm per pair of rows plus a mask-or-subtract per two codes; the high nibble of a byte is
// used in place (16 x code), its rows carry a factor 16 that the epilogue removes.  The residual
// window runs through bf16 MMAs into the same accumulators.  Softmax is in the log2 domain.
#include <cooperative_groups.h>

#include <atomic>
#include <cstdlib>

#include "rw4_common.cuh"
#include "rw4_tma.cuh"

namespace cg = cooperative_groups;
using namespace rw4;

namespace {

constexpr int kTok = 64;
constexpr int kStages = 2;
// warps per CTA (one CTA per SM: 255 registers a thread).  12 warps at 168 registers measured
// no faster at batch 16 and slower at batch 1 (more warps without items, a longer combine).
template <int NT>
struct KvWarps {
  static constexpr int value = 8;
};
constexpr float kNegBig = -1.0e30f;

template <int D>
struct KvLayout {
  static constexpr int VG = D / 64;          // V scale groups per token
  static constexpr int kK = 32 * D;          // K codes of one group
  static constexpr int kKsz = 4 * D;         // K (scale, zero) of one group
  static constexpr int kVRow = D / 2;        // V codes of one token
  static constexpr int kVBlk = 16 * kVRow + 32;  // 16 tokens + 32 bytes of bank padding
  static constexpr int kVsz = kTok * VG * 4;
  static constexpr int oK = 0;
  static constexpr int oKsz = oK + kK;
  static constexpr int oV = oKsz + kKsz;
  static constexpr int oVsz = oV + 4 * kVBlk;
  static constexpr int kStage = (oVsz + kVsz + 127) / 128 * 128;
  static constexpr uint32_t kTx = kK + kKsz + kTok * kVRow + kVsz;
};

struct KvArgs {
  const __nv_bfloat16* q;
  int64_t q_sb, q_sh, q_sq;
  const uint8_t* kc;
  const uint8_t* ksz;
  const uint8_t* vc;
  const uint8_t* vsz;
  int64_t gcap, groups;
  const __nv_bfloat16* kr;
  const __nv_bfloat16* vr;
  int64_t rcap, rlen;
  int KVH, G;
  int Q;         // query positions: the last Q window tokens, each attending causally
  float qscale;  // softmax scaling * log2(e)
  __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_sq;
  unsigned int* status;
};

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ uint32_t lds_u32(const uint8_t* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// two codes (bits 0-3 or 4-7 of each half, selected by `mask`) -> fp16 pair 1024 + code (or
// 1024 + 16 code): exact, with an offset of 1024 that an all-ones MMA removes per chunk
__device__ __forceinline__ uint32_t codes_f16(uint32_t x, uint32_t mask) {
  return (x & mask) | 0x64006400u;
}

constexpr uint32_t kOnesF16 = 0x3C003C00u;  // (1.0, 1.0)

__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
  __half2 h = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t bf16x2_times16(uint32_t x) {
  __nv_bfloat162 h = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&x),
                             __nv_bfloat162(__float2bfloat16(16.f), __float2bfloat16(16.f)));
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t movtrans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float half_lo(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
}
__device__ __forceinline__ float half_hi(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}

// Online-softmax step over one item's scores s[nt][mt][4] (C fragments of S^T: rows = tokens
// 8n+2mt / 8n+2mt+1, columns = heads nt*8 + 2qd + {0, 1}); s is replaced by the probabilities.
template <int NT, int VM, int VG>
__device__ __forceinline__ void softmax_step(float (&s)[NT][4][4], float (&m_run)[NT][2],
                                             float (&l_run)[NT][2], float (&zp)[NT][VG][2],
                                             float (&o)[NT][VM][4], float (&offv)[NT][VG][4]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float mx = kNegBig;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) mx = fmaxf(mx, fmaxf(s[nt][mt][j], s[nt][mt][j + 2]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mnew = fmaxf(m_run[nt][j], mx);
      const float alpha = ex2(m_run[nt][j] - mnew);
      m_run[nt][j] = mnew;
      float l = l_run[nt][j] * alpha;
#pragma unroll
      for (int g = 0; g < VG; ++g) {
        zp[nt][g][j] *= alpha;
        offv[nt][g][j] *= alpha;
        offv[nt][g][j + 2] *= alpha;
      }
#pragma unroll
      for (int vm = 0; vm < VM; ++vm) {
        o[nt][vm][j] *= alpha;
        o[nt][vm][j + 2] *= alpha;
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const float p0 = ex2(s[nt][mt][j] - mnew);
        const float p1 = ex2(s[nt][mt][j + 2] - mnew);
        s[nt][mt][j] = p0;
        s[nt][mt][j + 2] = p1;
        l += p0 + p1;
      }
      l_run[nt][j] = l;
    }
  }
}

template <int D, int NT, int kWarps = KvWarps<NT>::value>
__global__ void __launch_bounds__(kWarps * 32, 1) rw4_kv_attn_kernel(const KvArgs a) {
  constexpr int kThreads = kWarps * 32;
  using L = KvLayout<D>;
  constexpr int KC = D / 16;  // 16-channel chunks of the QK^T reduction
  constexpr int VG = L::VG;
  constexpr int VM = D / 16;  // 16-channel m-tiles of O^T
  constexpr int QH = 8 * NT;  // query-head columns (zero beyond G)
  extern __shared__ __align__(128) uint8_t smem[];
  float* qs = reinterpret_cast<float*>(smem);  // [QH][D] query * qscale
  uint8_t* stages = smem + QH * D * 4;
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + kWarps * kStages * L::kStage);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = lane >> 2, qd = lane & 3;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = static_cast<int>(cluster.block_rank());
  const int csize = static_cast<int>(cluster.num_blocks());
  const int hs = blockIdx.y;
  const int b = hs / a.KVH, kvh = hs % a.KVH;

  // column h of the MMAs = (query position h / G, query head kvh * G + h % G)
  for (int i = threadIdx.x; i < QH * D; i += kThreads) {
    const int h = i / D, c = i % D;
    float v = 0.f;
    if (h < a.Q * a.G)
      v = __bfloat162float(a.q[b * a.q_sb + static_cast<int64_t>(kvh * a.G + h % a.G) * a.q_sh +
                               static_cast<int64_t>(h / a.G) * a.q_sq + c]) *
          a.qscale;
    qs[i] = v;
  }
  const uint32_t bar0 = smem_addr(bars + warp * kStages);
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_barrier_init();
  }
  __syncthreads();

  // query fragment of the quantized path as fp16 pairs: head nt*8 + n, channels
  // (16kc + qd, 16kc + qd + 4) and (16kc + qd + 8, 16kc + qd + 12)
  uint32_t qh[NT][KC][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
      const float* qr = qs + (nt * 8 + n) * D + 16 * kc + qd;
      qh[nt][kc][0] = pack_f16(qr[0], qr[4]);
      qh[nt][kc][1] = pack_f16(qr[8], qr[12]);
    }

  const int64_t nw = static_cast<int64_t>(csize) * kWarps;
  const int64_t wg = static_cast<int64_t>(crank) * kWarps + warp;
  const int64_t nq = a.groups;
  const int64_t total = nq + (a.rlen + kTok - 1) / kTok;
  const int64_t nq_w = wg < nq ? (nq - 1 - wg) / nw + 1 : 0;
  const int64_t tcap = a.gcap * kTok;
  const uint8_t* kc_hs = a.kc + static_cast<int64_t>(hs) * a.gcap * L::kK;
  const uint8_t* ksz_hs = a.ksz + static_cast<int64_t>(hs) * a.gcap * L::kKsz;
  const uint8_t* vc_hs = a.vc + static_cast<int64_t>(hs) * tcap * L::kVRow;
  const uint8_t* vsz_hs = a.vsz + static_cast<int64_t>(hs) * tcap * VG * 4;
  const __nv_bfloat16* kr = a.kr + static_cast<int64_t>(hs) * a.rcap * D;
  const __nv_bfloat16* vr = a.vr + static_cast<int64_t>(hs) * a.rcap * D;
  uint8_t* my = stages + warp * kStages * L::kStage;

  auto issue = [&](int64_t j) {  // lane 0: group wg + j*nw into stage j % kStages
    const int64_t g = wg + j * nw;
    const int s = static_cast<int>(j % kStages);
    const uint32_t dst = smem_addr(my + s * L::kStage);
    const uint32_t bar = bar0 + 8 * s;
    mbar_arrive_expect_tx(bar, L::kTx);
    bulk_load(dst + L::oK, kc_hs + g * L::kK, L::kK, bar);
    bulk_load(dst + L::oKsz, ksz_hs + g * L::kKsz, L::kKsz, bar);
    const uint8_t* v = vc_hs + g * kTok * L::kVRow;
#pragma unroll
    for (int blk = 0; blk < 4; ++blk)
      bulk_load(dst + L::oV + blk * L::kVBlk, v + blk * 16 * L::kVRow, 16 * L::kVRow, bar);
    bulk_load(dst + L::oVsz, vsz_hs + g * kTok * VG * 4, L::kVsz, bar);
  };
  if (lane == 0)
    for (int64_t j = 0; j < kStages && j < nq_w; ++j) issue(j);
  __syncwarp();

  float m_run[NT][2], l_run[NT][2], zp[NT][VG][2], o[NT][VM][4];
  float offv[NT][VG][4];  // sum_t B[t, head] of the V MMAs: their 1024 offset, per head
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      m_run[nt][j] = kNegBig;
      l_run[nt][j] = 0.f;
#pragma unroll
      for (int g = 0; g < VG; ++g) zp[nt][g][j] = 0.f;
    }
#pragma unroll
    for (int g = 0; g < VG; ++g)
#pragma unroll
      for (int i = 0; i < 4; ++i) offv[nt][g][i] = 0.f;
#pragma unroll
    for (int vm = 0; vm < VM; ++vm)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[nt][vm][i] = 0.f;
  }

  int64_t consumed = 0;  // quantized groups this warp has finished with
  bool ok = true;
  for (int64_t item = wg; item < total; item += nw) {
    float s[NT][4][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) s[nt][mt][i] = 0.f;

    if (item < nq) {
      // ---------------- a quantized group ----------------
      const int st = static_cast<int>(consumed % kStages);
      const bool got = mbar_wait(bar0 + 8 * st, static_cast<uint32_t>((consumed / kStages) & 1),
                                 a.status);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      const uint8_t* sb = my + st * L::kStage;
      const uint8_t* kcs = sb + L::oK;
      const uint8_t* kss = sb + L::oKsz;
      // offk: sum_c B'[c, head] (the 1024 offset of the codes); zk: sum_c q'[head, c] z_c
      float offk[NT][4], zk[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) offk[nt][i] = zk[nt][i] = 0.f;
      const uint32_t ones[4] = {kOnesF16, kOnesF16, kOnesF16, kOnesF16};
#pragma unroll
      for (int kc = 0; kc < KC; ++kc) {
        uint32_t w[4], sz[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 16 * kc + qd + 4 * e;
          w[e] = lds_u32(kcs + 32 * c + 4 * n);
          sz[e] = lds_u32(kss + 4 * c);
        }
        const uint32_t s01 = __byte_perm(sz[0], sz[1], 0x5410);
        const uint32_t s23 = __byte_perm(sz[2], sz[3], 0x5410);
        const uint32_t z01 = __byte_perm(sz[0], sz[1], 0x7632);
        const uint32_t z23 = __byte_perm(sz[2], sz[3], 0x7632);
        uint32_t bq[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          bq[nt][0] = hmul2_u(qh[nt][kc][0], s01);
          bq[nt][1] = hmul2_u(qh[nt][kc][1], s23);
          mma_f16_16816(offk[nt], ones, bq[nt][0], bq[nt][1], offk[nt]);
          mma_f16_16816(zk[nt], ones, hmul2_u(qh[nt][kc][0], z01), hmul2_u(qh[nt][kc][1], z23),
                        zk[nt]);
        }
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          const uint32_t sel = mt | (mt << 4) | ((4 + mt) << 8) | ((4 + mt) << 12);
          const uint32_t x01 = __byte_perm(w[0], w[1], sel);
          const uint32_t x23 = __byte_perm(w[2], w[3], sel);
          const uint32_t af[4] = {codes_f16(x01, 0x000F000Fu), codes_f16(x01, 0x00F000F0u),
                                  codes_f16(x23, 0x000F000Fu), codes_f16(x23, 0x00F000F0u)};
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_f16_16816(s[nt][mt], af, bq[nt][0], bq[nt][1], s[nt][mt]);
        }
      }
      // S = (acc - 1024 offk) [/ 16 on the high-nibble rows] + zk; the all-ones MMAs leave the
      // per-head sums in every row, columns 2qd and 2qd + 1 as the scores' own fragment
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float ce0 = fmaf(-1024.f, offk[nt][0], zk[nt][0]);
        const float ce1 = fmaf(-1024.f, offk[nt][1], zk[nt][1]);
        const float co0 = fmaf(-64.f, offk[nt][0], zk[nt][0]);
        const float co1 = fmaf(-64.f, offk[nt][1], zk[nt][1]);
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          s[nt][mt][0] += ce0;
          s[nt][mt][1] += ce1;
          s[nt][mt][2] = fmaf(s[nt][mt][2], 0.0625f, co0);
          s[nt][mt][3] = fmaf(s[nt][mt][3], 0.0625f, co1);
        }
      }
      softmax_step<NT, VM, VG>(s, m_run, l_run, zp, o, offv);

      // P V: scales of this thread's tokens 8n..8n+7 (C-fragment rows)
      const uint8_t* vcs = sb + L::oV;
      const uint32_t* vss = reinterpret_cast<const uint32_t*>(sb + L::oVsz) + 8 * VG * n;
      uint32_t vz[8 * VG];
#pragma unroll
      for (int i = 0; i < 2 * VG; ++i) {
        const uint4 t4 = *reinterpret_cast<const uint4*>(vss + 4 * i);
        vz[4 * i] = t4.x;
        vz[4 * i + 1] = t4.y;
        vz[4 * i + 2] = t4.z;
        vz[4 * i + 3] = t4.w;
      }
      const uint8_t* blk = vcs + qd * L::kVBlk;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t bv[NT][VG][2], pe[NT], po[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          pe[nt] = pack_f16(s[nt][mt][0], s[nt][mt][1]);
          po[nt] = pack_f16(s[nt][mt][2], s[nt][mt][3]);
        }
#pragma unroll
        for (int g = 0; g < VG; ++g) {
          const uint32_t e = vz[(2 * mt) * VG + g], od = vz[(2 * mt + 1) * VG + g];
          const float ze = half_hi(e), zo = half_hi(od);
          const uint32_t se2 = __byte_perm(e, e, 0x1010), so2 = __byte_perm(od, od, 0x1010);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            zp[nt][g][0] = fmaf(s[nt][mt][0], ze, fmaf(s[nt][mt][2], zo, zp[nt][g][0]));
            zp[nt][g][1] = fmaf(s[nt][mt][1], ze, fmaf(s[nt][mt][3], zo, zp[nt][g][1]));
            bv[nt][g][0] = movtrans(hmul2_u(pe[nt], se2));
            bv[nt][g][1] = movtrans(hmul2_u(po[nt], so2));
            const uint32_t ones[4] = {kOnesF16, kOnesF16, kOnesF16, kOnesF16};
            mma_f16_16816(offv[nt][g], ones, bv[nt][g][0], bv[nt][g][1], offv[nt][g]);
          }
        }
#pragma unroll
        for (int g = 0; g < VG; ++g) {
          const uint8_t* rowp = blk + 32 * g + 4 * n;
          const uint32_t wA = lds_u32(rowp + (2 * mt) * L::kVRow);
          const uint32_t wB = lds_u32(rowp + (2 * mt + 8) * L::kVRow);
          const uint32_t wC = lds_u32(rowp + (2 * mt + 1) * L::kVRow);
          const uint32_t wD = lds_u32(rowp + (2 * mt + 9) * L::kVRow);
#pragma unroll
          for (int mm = 0; mm < 4; ++mm) {
            const uint32_t sel = mm | (mm << 4) | ((4 + mm) << 8) | ((4 + mm) << 12);
            const uint32_t x = __byte_perm(wA, wB, sel);
            const uint32_t y = __byte_perm(wC, wD, sel);
            const uint32_t af[4] = {codes_f16(x, 0x000F000Fu), codes_f16(x, 0x00F000F0u),
                                    codes_f16(y, 0x000F000Fu), codes_f16(y, 0x00F000F0u)};
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              mma_f16_16816(o[nt][4 * g + mm], af, bv[nt][g][0], bv[nt][g][1], o[nt][4 * g + mm]);
          }
        }
      }
      // every lane orders its generic reads of the stage before the bulk refill (async proxy)
      fence_proxy_async_smem();
      __syncwarp();
      const int64_t next = consumed + kStages;
      if (lane == 0 && next < nq_w) issue(next);
      ++consumed;
    } else {
      // ---------------- a 64-token chunk of the bf16 window ----------------
      const int64_t t0 = (item - nq) * kTok;
      const int64_t last = a.rlen - 1;
#pragma unroll
      for (int kc = 0; kc < KC; ++kc) {
        uint32_t bq[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 f = *reinterpret_cast<const float4*>(qs + (nt * 8 + n) * D +
                                                            (D / 4) * qd + 4 * kc);
          bq[nt][0] = pack_bf16(f.x, f.y);
          bq[nt][1] = pack_bf16(f.z, f.w);
        }
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          const int64_t te = min(t0 + 8 * n + 2 * mt, last), to = min(te + 1, last);
          const uint2 ke = ldg_u2(kr + te * D + (D / 4) * qd + 4 * kc);
          const uint2 ko = ldg_u2(kr + to * D + (D / 4) * qd + 4 * kc);
          const uint32_t af[4] = {ke.x, ko.x, ke.y, ko.y};
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma_bf16_16816(s[nt][mt], af, bq[nt][0], bq[nt][1], s[nt][mt]);
        }
      }
      // window token t is visible to query position qi iff t <= rlen - Q + qi (the query tokens
      // are the window's last Q); padding columns see the whole window
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const int64_t te = t0 + 8 * n + 2 * mt;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int col = nt * 8 + 2 * qd + (i & 1);
            const int64_t limit =
                col < a.Q * a.G ? a.rlen - a.Q + 1 + col / a.G : a.rlen;
            if (te + (i >> 1) >= limit) s[nt][mt][i] = -INFINITY;
          }
      }
      softmax_step<NT, VM, VG>(s, m_run, l_run, zp, o, offv);
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t bv[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          bv[nt][0] = movtrans(pack_bf16(s[nt][mt][0], s[nt][mt][1]));
          bv[nt][1] = movtrans(pack_bf16(s[nt][mt][2], s[nt][mt][3]));
        }
        const int64_t tA = min(t0 + 16 * qd + 2 * mt, last), tB = min(tA + 8, last),
                      tC = min(tA + 1, last), tD = min(tA + 9, last);
#pragma unroll
        for (int g = 0; g < VG; ++g) {
          const int64_t col = 64 * g + 8 * n;
          const uint4 vA = ldg_u4(vr + tA * D + col), vB = ldg_u4(vr + tB * D + col);
          const uint4 vC = ldg_u4(vr + tC * D + col), vD = ldg_u4(vr + tD * D + col);
          const uint32_t wa[4] = {vA.x, vA.y, vA.z, vA.w}, wb[4] = {vB.x, vB.y, vB.z, vB.w};
          const uint32_t wc[4] = {vC.x, vC.y, vC.z, vC.w}, wd[4] = {vD.x, vD.y, vD.z, vD.w};
#pragma unroll
          for (int mm = 0; mm < 4; ++mm) {
            const uint32_t af[4] = {__byte_perm(wa[mm], wb[mm], 0x5410),
                                    bf16x2_times16(__byte_perm(wa[mm], wb[mm], 0x7632)),
                                    __byte_perm(wc[mm], wd[mm], 0x5410),
                                    bf16x2_times16(__byte_perm(wc[mm], wd[mm], 0x7632))};
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              mma_bf16_16816(o[nt][4 * g + mm], af, bv[nt][0], bv[nt][1], o[nt][4 * g + mm]);
          }
        }
      }
    }
  }
  if (!ok) {
    // a copy did not land in time: give the outstanding ones a bounded chance to finish before
    // the shared memory is reused
    if (lane == 0) atomicOr(a.status, RW4_DEVERR_TIMEOUT);
    const int64_t issued = nq_w < consumed + kStages ? nq_w : consumed + kStages;
    for (int64_t j = consumed; j < issued; ++j)
      mbar_wait(bar0 + 8 * static_cast<int>(j % kStages), static_cast<uint32_t>((j / kStages) & 1),
                a.status);
  }

  // ---------------- per-warp partials ----------------
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float l = l_run[nt][j];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      l_run[nt][j] = l;
#pragma unroll
      for (int g = 0; g < VG; ++g) {
        float z = zp[nt][g][j];
        z += __shfl_xor_sync(0xffffffffu, z, 4);
        z += __shfl_xor_sync(0xffffffffu, z, 8);
        z += __shfl_xor_sync(0xffffffffu, z, 16);
        zp[nt][g][j] = z;
      }
    }
  __syncthreads();  // every warp is past its ring: the stage area becomes the partials area
  constexpr int kPart = QH * (D + 2);  // floats: O[QH][D], m[QH], l[QH]
  float* part = reinterpret_cast<float*>(stages);
  float* mine = part + warp * kPart;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int vm = 0; vm < VM; ++vm) {
      const int g = vm / 4, mm = vm % 4;
      const int ch = 64 * g + 8 * n + 2 * mm;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = i & 1;
        const int h = nt * 8 + 2 * qd + j;
        const float a = fmaf(-1024.f, offv[nt][g][j], o[nt][vm][i]);
        const float v = (i < 2 ? a : a * 0.0625f) + zp[nt][g][j];
        mine[h * D + ch + (i >> 1)] = v;
      }
    }
  if (n == 0) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int h = nt * 8 + 2 * qd + j;
        mine[QH * D + h] = m_run[nt][j];
        mine[QH * D + QH + h] = l_run[nt][j];
      }
  }
  __syncthreads();
  float* cpart = part + kWarps * kPart;  // this CTA's combination of its warps
  for (int i = threadIdx.x; i < QH * D; i += kThreads) {
    const int h = i / D;
    float mx = kNegBig;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, part[w * kPart + QH * D + h]);
    float acc = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = ex2(part[w * kPart + QH * D + h] - mx);
      acc = fmaf(part[w * kPart + i], f, acc);
      l = fmaf(part[w * kPart + QH * D + QH + h], f, l);
    }
    cpart[i] = acc;
    if (i % D == 0) {
      cpart[QH * D + h] = mx;
      cpart[QH * D + QH + h] = l;
    }
  }
  cluster.sync();
  if (crank == 0) {
    for (int i = threadIdx.x; i < a.Q * a.G * D; i += kThreads) {
      const int h = i / D, c = i % D;
      float mx = kNegBig;
      for (int r = 0; r < csize; ++r) {
        const float* rp = cluster.map_shared_rank(cpart, r);
        mx = fmaxf(mx, rp[QH * D + h]);
      }
      float acc = 0.f, l = 0.f;
      for (int r = 0; r < csize; ++r) {
        const float* rp = cluster.map_shared_rank(cpart, r);
        const float f = ex2(rp[QH * D + h] - mx);
        acc = fmaf(rp[h * D + c], f, acc);
        l = fmaf(rp[QH * D + QH + h], f, l);
      }
      a.out[b * a.o_sb + static_cast<int64_t>(h / a.G) * a.o_sq +
            static_cast<int64_t>(kvh * a.G + h % a.G) * a.o_sh + c] = __float2bfloat16(acc / l);
    }
  }
  cluster.sync();  // rank 0 has read every CTA's partials
}

template <int D, int NT>
size_t kv_smem() {
  using L = KvLayout<D>;
  constexpr int kWarps = KvWarps<NT>::value;
  return static_cast<size_t>(8 * NT * D * 4) + kWarps * kStages * L::kStage + kWarps * kStages * 8;
}

template <int D, int NT>
int launch_kv(const KvArgs& args, int hs_count, int csize, cudaStream_t stream) {
  using L = KvLayout<D>;
  constexpr int kWarps = KvWarps<NT>::value;
  static_assert(kWarps * (8 * NT * (D + 2)) * 4 + 8 * NT * (D + 2) * 4 <=
                    kWarps * kStages * L::kStage,
                "partials must fit the stage area");
  auto kern = rw4_kv_attn_kernel<D, NT>;
  const size_t smem = kv_smem<D, NT>();
  static std::atomic<uint32_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set.load() & (1u << dev))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
            cudaSuccess)
      return fail(RW4_ECUDA, "kv_attention: cannot set the kernel's launch attributes");
    attr_set.fetch_or(1u << dev);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(csize, hs_count);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kern, args);
  if (err != cudaSuccess) return cuda_status(err, "rw4 kv_attention launch");
  return launch_status("rw4 kv_attention launch");
}

}  // namespace

namespace rw4 {

// CTAs per head slot: enough to give every SM one CTA when the batch is small, at most a portable
// cluster of 8, and no more than the items keep busy (at least one per warp).
int kv_cluster_size(int64_t head_slots, int64_t items, int warps) {
  int s = 1;
  while (s < 8 && head_slots * (2 * s) <= sm_count() &&
         static_cast<int64_t>(2 * s) * warps <= items)
    s *= 2;
  return s;
}

}  // namespace rw4

extern "C" int rw4_kv_attention(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                int64_t q_stride_q, int32_t batch, int32_t heads,
                                int32_t kv_heads, int32_t head_dim, int32_t q_len,
                                const uint8_t* k_codes, const void* k_sz, const uint8_t* v_codes,
                                const void* v_sz, int64_t groups_cap, int64_t groups,
                                const void* k_res, const void* v_res, int64_t res_cap,
                                int64_t res_len, float scaling, void* out, int64_t out_stride_b,
                                int64_t out_stride_h, int64_t out_stride_q, void* stream) {
  using namespace rw4;
  if (!q || !out || batch <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads)
    return fail(RW4_EINVAL, "kv_attention: bad query / head arguments (%d heads, %d kv heads)",
                heads, kv_heads);
  const int G = heads / kv_heads;
  if (G > 16) return fail(RW4_EUNSUPPORTED, "kv_attention: %d query heads per kv head (max 16)", G);
  if (q_len < 1 || q_len * G > 16)
    return fail(RW4_EUNSUPPORTED,
                "kv_attention: %d query positions x %d heads per kv head (at most 16 columns)",
                q_len, G);
  if (head_dim != 64 && head_dim != 128)
    return fail(RW4_EUNSUPPORTED, "kv_attention: head_dim %d (64 or 128 supported)", head_dim);
  if (groups < 0 || groups > groups_cap || res_len < 0 || res_len > res_cap)
    return fail(RW4_EINVAL, "kv_attention: %lld groups of %lld, %lld window tokens of %lld",
                (long long)groups, (long long)groups_cap, (long long)res_len, (long long)res_cap);
  if (groups + res_len == 0) return fail(RW4_EINVAL, "kv_attention: empty cache");
  if (res_len < q_len)
    return fail(RW4_EINVAL, "kv_attention: the %d query tokens must be the window's last (%lld)",
                q_len, (long long)res_len);
  if (groups_cap > 0 && (!k_codes || !k_sz || !v_codes || !v_sz || !aligned(k_codes, 16) ||
                         !aligned(k_sz, 16) || !aligned(v_codes, 16) || !aligned(v_sz, 16)))
    return fail(RW4_EINVAL, "kv_attention: packed arrays must be non-null and 16-byte aligned");
  if (res_cap > 0 && (!k_res || !v_res || !aligned(k_res, 16) || !aligned(v_res, 16)))
    return fail(RW4_EINVAL, "kv_attention: window arrays must be non-null and 16-byte aligned");
  const int64_t hs_count = static_cast<int64_t>(batch) * kv_heads;
  if (hs_count > 65535) return fail(RW4_EINVAL, "kv_attention: %lld head slots", (long long)hs_count);
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "kv_attention: device status word unavailable");
  KvArgs args;
  args.q = static_cast<const __nv_bfloat16*>(q);
  args.q_sb = q_stride_b;
  args.q_sh = q_stride_h;
  args.q_sq = q_stride_q;
  args.kc = k_codes;
  args.ksz = static_cast<const uint8_t*>(k_sz);
  args.vc = v_codes;
  args.vsz = static_cast<const uint8_t*>(v_sz);
  args.gcap = groups_cap;
  args.groups = groups;
  args.kr = static_cast<const __nv_bfloat16*>(k_res);
  args.vr = static_cast<const __nv_bfloat16*>(v_res);
  args.rcap = res_cap;
  args.rlen = res_len;
  args.KVH = kv_heads;
  args.G = G;
  args.Q = q_len;
  args.qscale = scaling * 1.4426950408889634f;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.o_sb = out_stride_b;
  args.o_sh = out_stride_h;
  args.o_sq = out_stride_q;
  args.status = status;
  const int cols = q_len * G;
  const int64_t items = groups + (res_len + kTok - 1) / kTok;
  int cs = kv_cluster_size(hs_count, items, cols <= 8 ? KvWarps<1>::value : KvWarps<2>::value);
  // launch-shape switch for measurements, read once per process
  static const char* const forced = getenv("RW4_KV_CLUSTER");
  if (forced) {
    const int f = atoi(forced);
    if (f != 1 && f != 2 && f != 4 && f != 8 && f != 16)
      return fail(RW4_EINVAL, "RW4_KV_CLUSTER=%s (1, 2, 4, 8 or 16)", forced);
    cs = f;
  }
  cudaStream_t st = as_stream(stream);
  const int hsc = static_cast<int>(hs_count);
  if (head_dim == 128)
    return cols <= 8 ? launch_kv<128, 1>(args, hsc, cs, st) : launch_kv<128, 2>(args, hsc, cs, st);
  return cols <= 8 ? launch_kv<64, 1>(args, hsc, cs, st) : launch_kv<64, 2>(args, hsc, cs, st);
}

extern "C" int rw4_kv_attention_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                       int32_t batch, int32_t heads, int32_t kv_heads,
                                       int32_t head_dim, const uint8_t* k_codes, const void* k_sz,
                                       const uint8_t* v_codes, const void* v_sz,
                                       int64_t groups_cap, int64_t groups, const void* k_res,
                                       const void* v_res, int64_t res_cap, int64_t res_len,
                                       float scaling, void* out, int64_t out_stride_b,
                                       int64_t out_stride_h, void* stream) {
  return rw4_kv_attention(q, q_stride_b, q_stride_h, 0, batch, heads, kv_heads, head_dim, 1,
                          k_codes, k_sz, v_codes, v_sz, groups_cap, groups, k_res, v_res, res_cap,
                          res_len, scaling, out, out_stride_b, out_stride_h, 0, stream);
}
