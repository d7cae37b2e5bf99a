// RW4 dequant-GEMV for decode (M <= 16): y[M, N] = x[M, K] . W[N, K]^T with W in RW4.
//
// Roofline: HBM.  Algorithmic bytes per call = N*K/2 (codes) + 4*N*K/64 (fp16 scale + zero)
// + 2*M*K (x) + 2*M*N (y); at M=1 that is 0.5625 B per weight and 3.6 flop/B, far left of the
// ridge.  On B200 the HBM rate (~6.5 TB/s) delivers ~11.6 G weights/ms while the four schedulers
// of 148 SMs issue ~36 T lane-ops/s, so a per-weight "unpack, convert, scale, FMA" sequence on the
// CUDA cores (~5 ops/weight) cannot keep up.  This kernel therefore:
//
//  * multiplies raw codes, not dequantized weights.  Per group g of 64 along K,
//        sum_k x_k (c_k s_g + z_g) = s_g * sum_k x_k c_k + z_g * sum_k x_k,
//    so the inner product runs on integer codes and the per-group scale/zero are applied once
//    per 64 weights in fp32 (exact weights, no bf16 rounding of W at all);
//  * turns codes into bf16 with one LOP3 per pair: (w >> 4p) & 0x000F000F | 0x43004300 gives the
//    bf16 pair (128 + c_p, 128 + c_{p+4}); the 128 offset is folded into the zero term
//    (z' = z - 128 s), so there is no subtraction per weight;
//  * feeds (128 + c) and x to the tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate) with a
//    per-group accumulator, and gets sum_k x_k of every group from one more MMA against an all-ones
//    A operand (no CUDA-core reduction of x);
//  * permutes K inside each MMA: the 16 K-slots of one MMA map to the 16 codes of one thread's
//    8-byte slice in the order the LOP3 extraction produces them, and x is loaded naturally and
//    permuted with two PRMTs per register pair to match.  The reduction is over K, so any
//    permutation applied identically to A and B leaves the result unchanged.
//
// Work split: a CTA owns 16*R consecutive output rows and the full K; its 8 warps take interleaved
// chunks of 4 groups (256 k) and combine partial sums through shared memory at the end, so every
// output is written once, deterministically, with no atomics and no scratch memory.  Codes are
// fetched with 8-byte L1-bypassing loads (each quad of lanes reads 32 contiguous bytes = one
// sector of a row); scales, zeros and x go through the read-only cache.
//
// Exactness: the group partial sum of (128 + c) x is formed by the tensor core in fp32; the later
// subtraction of 128 * sum(x) cancels ~7 bits, leaving ~2^-17 relative error per group, far below
// the bf16 output rounding (2^-9).
#include "rw4_gemv_frag.cuh"
#include "rw4_xprep.cuh"

namespace {

using namespace rw4::frag;

constexpr int kWarps = 8;
constexpr int kGroupsPerChunk = 4;  // 256 values of K per warp iteration

// Registers holding one chunk (4 groups) of codes and scales for the thread's 2R rows.
template <int R>
struct ChunkRegs {
  uint2 wa[R][kGroupsPerChunk], wb[R][kGroupsPerChunk];  // 8 code bytes per row and group
  uint2 sa[R], sb[R], za[R], zb[R];                      // 4 fp16 scales / zeros per row
};

__device__ __forceinline__ uint2 pack4h(__half a, __half b, __half c, __half d) {
  __half2 lo = __halves2half2(a, b), hi = __halves2half2(c, d);
  return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

template <int R>
__device__ __forceinline__ void load_chunk(ChunkRegs<R>& r, int c, int G, bool vec_scales,
                                           const uint8_t* const (&wrow_a)[R],
                                           const uint8_t* const (&wrow_b)[R],
                                           const __half* const (&srow_a)[R],
                                           const __half* const (&srow_b)[R],
                                           const __half* const (&zrow_a)[R],
                                           const __half* const (&zrow_b)[R]) {
  const int gbase = c * kGroupsPerChunk;
#pragma unroll
  for (int i = 0; i < kGroupsPerChunk; ++i) {
    const bool in = gbase + i < G;
#pragma unroll
    for (int rt = 0; rt < R; ++rt) {
      r.wa[rt][i] = in ? ldg_stream_u2(wrow_a[rt] + (gbase + i) * 32) : make_uint2(0, 0);
      r.wb[rt][i] = in ? ldg_stream_u2(wrow_b[rt] + (gbase + i) * 32) : make_uint2(0, 0);
    }
  }
#pragma unroll
  for (int rt = 0; rt < R; ++rt) {
    if (vec_scales) {
      r.sa[rt] = ldg_u2(srow_a[rt] + gbase);
      r.sb[rt] = ldg_u2(srow_b[rt] + gbase);
      r.za[rt] = ldg_u2(zrow_a[rt] + gbase);
      r.zb[rt] = ldg_u2(zrow_b[rt] + gbase);
    } else {
      const int g0 = min(gbase, G - 1), g1 = min(gbase + 1, G - 1);
      const int g2 = min(gbase + 2, G - 1), g3 = min(gbase + 3, G - 1);
      r.sa[rt] = pack4h(srow_a[rt][g0], srow_a[rt][g1], srow_a[rt][g2], srow_a[rt][g3]);
      r.sb[rt] = pack4h(srow_b[rt][g0], srow_b[rt][g1], srow_b[rt][g2], srow_b[rt][g3]);
      r.za[rt] = pack4h(zrow_a[rt][g0], zrow_a[rt][g1], zrow_a[rt][g2], zrow_a[rt][g3]);
      r.zb[rt] = pack4h(zrow_b[rt][g0], zrow_b[rt][g1], zrow_b[rt][g2], zrow_b[rt][g3]);
    }
  }
}

// fp16 element i (0..3) of four packed in a uint2.
__device__ __forceinline__ float h4(uint2 v, int i) {
  const uint32_t w = (i < 2) ? v.x : v.y;
  const __half2 h = *reinterpret_cast<const __half2*>(&w);
  return __half2float((i & 1) ? __high2half(h) : __low2half(h));
}

template <int NT, int R>
__device__ __forceinline__ void compute_chunk(const ChunkRegs<R>& r, int c, int G, int K, int Ml,
                                              int g, int t, const __nv_bfloat16* __restrict__ x,
                                              float (&out)[R][NT][4]) {
  const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
  const int gbase = c * kGroupsPerChunk;
#pragma unroll
  for (int i = 0; i < kGroupsPerChunk; ++i) {
    if (gbase + i >= G) break;
    const int kofs = (gbase + i) * 64 + 16 * t;
    uint32_t b[NT][4][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int m = nt * 8 + g;
      load_x_frag(x + (int64_t)min(m, Ml - 1) * K + kofs, m < Ml, b[nt]);
    }
    // sum of x over the group, for batch columns (2t, 2t+1) of each batch tile
    float xs[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      mma_bf16_16816(xs[nt], ones, b[nt][0][0], b[nt][0][1], zero4);
#pragma unroll
      for (int j = 1; j < 4; ++j) mma_bf16_16816(xs[nt], ones, b[nt][j][0], b[nt][j][1], xs[nt]);
    }
#pragma unroll
    for (int rt = 0; rt < R; ++rt) {
      float acc[NT][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t a[4];
        a_frag(r.wa[rt][i], r.wb[rt][i], j, a);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (j == 0)
            mma_bf16_16816(acc[nt], a, b[nt][j][0], b[nt][j][1], zero4);
          else
            mma_bf16_16816(acc[nt], a, b[nt][j][0], b[nt][j][1], acc[nt]);
        }
      }
      const float s_a = h4(r.sa[rt], i), s_b = h4(r.sb[rt], i);
      const float z_a = fmaf(-128.f, s_a, h4(r.za[rt], i));
      const float z_b = fmaf(-128.f, s_b, h4(r.zb[rt], i));
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        out[rt][nt][0] = fmaf(s_a, acc[nt][0], fmaf(z_a, xs[nt][0], out[rt][nt][0]));
        out[rt][nt][1] = fmaf(s_a, acc[nt][1], fmaf(z_a, xs[nt][1], out[rt][nt][1]));
        out[rt][nt][2] = fmaf(s_b, acc[nt][2], fmaf(z_b, xs[nt][2], out[rt][nt][2]));
        out[rt][nt][3] = fmaf(s_b, acc[nt][3], fmaf(z_b, xs[nt][3], out[rt][nt][3]));
      }
    }
  }
}

// NT: number of 8-wide batch tiles (1 for M <= 8, 2 for M <= 16).  R: 16-row tiles per CTA.
template <int NT, int R>
__global__ void __launch_bounds__(kWarps * 32)
    rw4_gemv_kernel(const __nv_bfloat16* __restrict__ x, int M, int K,
                    const uint8_t* __restrict__ wq, const __half* __restrict__ sc,
                    const __half* __restrict__ zr, int N, __nv_bfloat16* __restrict__ y) {
  __shared__ float red[kWarps][16 * R][16 * NT + 1];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;  // MMA group id: A rows g, g+8; B column g; C columns 2t, 2t+1
  const int t = lane & 3;

  // Slice of the batch handled by this CTA row (grid.y walks 16-row slices of a larger M).
  const int m0 = blockIdx.y * 16;
  x += (int64_t)m0 * K;
  y += (int64_t)m0 * N;
  const int Ml = min(16, M - m0);

  const int G = K / 64;
  const int64_t row_bytes = K / 2;
  const int r0 = blockIdx.x * (16 * R);

  // Row pointers (clamped so rows past N read valid memory; their results are discarded).
  const uint8_t* wrow_a[R];
  const uint8_t* wrow_b[R];
  const __half* srow_a[R];
  const __half* srow_b[R];
  const __half* zrow_a[R];
  const __half* zrow_b[R];
#pragma unroll
  for (int rt = 0; rt < R; ++rt) {
    const int ra = min(r0 + 16 * rt + g, N - 1);
    const int rb = min(r0 + 16 * rt + g + 8, N - 1);
    wrow_a[rt] = wq + (int64_t)ra * row_bytes + 8 * t;
    wrow_b[rt] = wq + (int64_t)rb * row_bytes + 8 * t;
    srow_a[rt] = sc + (int64_t)ra * G;
    srow_b[rt] = sc + (int64_t)rb * G;
    zrow_a[rt] = zr + (int64_t)ra * G;
    zrow_b[rt] = zr + (int64_t)rb * G;
  }

  float out[R][NT][4];
#pragma unroll
  for (int rt = 0; rt < R; ++rt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) out[rt][nt][e] = 0.f;

  const int chunks = (G + kGroupsPerChunk - 1) / kGroupsPerChunk;
  const bool vec_scales = (G & 3) == 0;

  // Register-staged fallback for K not a multiple of 512 (the TMA kernel's scale-box alignment):
  // each chunk is loaded into registers and then computed.
  for (int c = warp; c < chunks; c += kWarps) {
    ChunkRegs<R> cur;
    load_chunk<R>(cur, c, G, vec_scales, wrow_a, wrow_b, srow_a, srow_b, zrow_a, zrow_b);
    compute_chunk<NT, R>(cur, c, G, K, Ml, g, t, x, out);
  }

  // ---- combine the warps' partial sums and write bf16 -----------------------------------------
#pragma unroll
  for (int rt = 0; rt < R; ++rt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      red[warp][16 * rt + g][nt * 8 + 2 * t] = out[rt][nt][0];
      red[warp][16 * rt + g][nt * 8 + 2 * t + 1] = out[rt][nt][1];
      red[warp][16 * rt + g + 8][nt * 8 + 2 * t] = out[rt][nt][2];
      red[warp][16 * rt + g + 8][nt * 8 + 2 * t + 1] = out[rt][nt][3];
    }
  __syncthreads();
  constexpr int kOut = 16 * R * 16 * NT;
  for (int o = threadIdx.x; o < kOut; o += kWarps * 32) {
    const int r = o % (16 * R);   // consecutive threads -> consecutive output rows (coalesced)
    const int m = o / (16 * R);
    const int n = r0 + r;
    if (n < N && m < Ml) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) v += red[w][r][m];
      y[(int64_t)m * N + n] = __float2bfloat16_rn(v);
    }
  }
}

template <int NT, int R>
void launch(const __nv_bfloat16* x, int M, int K, const uint8_t* wq, const __half* sc,
            const __half* zr, int N, __nv_bfloat16* y, cudaStream_t s) {
  dim3 grid((N + 16 * R - 1) / (16 * R), (M + 15) / 16);
  rw4_gemv_kernel<NT, R><<<grid, kWarps * 32, 0, s>>>(x, M, K, wq, sc, zr, N, y);
}

int rows_per_cta_override() {
  static int v = [] {
    const char* e = getenv("RW4_GEMV_ROW_TILES");
    return e ? atoi(e) : 0;
  }();
  return v;
}

}  // namespace

namespace rw4 {

// y = x W^T for any M via 16-row batch slices (M <= 16: one slice).
bool gemv_tma_supported(int64_t K);
size_t gemv_tma_workspace(int64_t M, int64_t K, int64_t N);
int gemv_tma_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                    const void* zr, int64_t N, void* y, cudaStream_t s, int row_tiles, void* ws,
                    size_t ws_bytes, const void* res = nullptr, const XNorm* norm = nullptr);

// Workspace bytes the GEMV needs for (M, K, N): the TMA kernel's x-prep arrays (none for a row it
// converts itself); the register-staged kernel needs none.
size_t gemv_workspace(int64_t M, int64_t K, int64_t N) {
  static const bool no_tma = getenv("RW4_GEMV_NO_TMA") != nullptr;
  return (!no_tma && gemv_tma_supported(K)) ? gemv_tma_workspace(M, K, N) : 0;
}

int gemv_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                const void* zr, int64_t N, void* y, cudaStream_t s, void* ws, size_t ws_bytes) {
  const int nt = (M <= 8) ? 1 : 2;
  const int forced = rows_per_cta_override();
  static const bool no_tma = getenv("RW4_GEMV_NO_TMA") != nullptr;
  // the TMA kernel picks its own CTA shape (gemv_tma_policy) unless RW4_GEMV_ROW_TILES forces one
  if (!no_tma && gemv_tma_supported(K))
    return gemv_tma_launch(x, M, K, wq, sc, zr, N, y, s, forced, ws, ws_bytes);
  // register-staged kernel (K % 512 != 0): 32-row CTAs from N >= 18944, else 16
  const int R = (forced == 1 || forced == 2) ? forced : (N >= 16 * 2 * 148 * 4) ? 2 : 1;
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* yb = static_cast<__nv_bfloat16*>(y);
  const auto* s16 = static_cast<const __half*>(sc);
  const auto* z16 = static_cast<const __half*>(zr);
  const int Mi = (int)M, Ki = (int)K, Ni = (int)N;
  if (nt == 1) {
    if (R == 1) launch<1, 1>(xb, Mi, Ki, wq, s16, z16, Ni, yb, s);
    else launch<1, 2>(xb, Mi, Ki, wq, s16, z16, Ni, yb, s);
  } else {
    if (R == 1) launch<2, 1>(xb, Mi, Ki, wq, s16, z16, Ni, yb, s);
    else launch<2, 2>(xb, Mi, Ki, wq, s16, z16, Ni, yb, s);
  }
  return launch_status("rw4 gemv launch");
}

}  // namespace rw4
