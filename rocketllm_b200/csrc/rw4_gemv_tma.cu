// RW4 dequant-GEMV, TMA-fed (K a multiple of 512): y[M, N] = x[M, K] . W[N, K]^T for decode
// batches, one 16-row batch slice per grid row.  The pipeline itself lives in
// rw4_gemv_tma_body.cuh; this file converts the activations and launches it.
//
// The activations are multiplied as fp16 values of x * 2^e, one power of two per row chosen from
// the row's largest magnitude, so that a row's conversion depends on that row alone: the GEMV then
// gives every row the same bits whether it runs alone (M = 1), in a decode batch or in a 16-row
// slice of a larger M, and x scaled by a power of two gives y scaled by exactly that power.
//
//  * one row whose CTA K range fits 32 KB of shared memory: the GEMV converts it in its own
//    prologue (XQ) -- one launch, no workspace;
//  * otherwise two launches: the x-prep kernel (rw4_xprep_kernel, one CTA per activation row)
//    writes the converted rows in MMA fragment order, per group of 64 the sum of x times 2^e and
//    minus 1024 times the sum of the fp16 values, and e, into a caller-provided workspace
//    (xprep_layout); the GEMV (XP) reads them through its TMA ring.  The pass reads and writes
//    M*K*2 bytes once per call; the GEMV is launched with programmatic dependent launch, so its
//    weight prefetch overlaps the pass.
// Both paths use the same conversion helpers in the same order (rw4_gemv_frag.cuh), so they give
// the same bits.
#include <atomic>

#include "rw4_gemv_tma_body.cuh"
#include "rw4_xprep.cuh"

namespace rw4 {

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

XPrepLayout xprep_layout(int64_t M, int64_t K) {
  XPrepLayout l;
  l.Mpad = (M + 1) & ~int64_t(1);
  l.xf = 0;
  l.side = align256((size_t)M * K * 2);
  l.row_exp = l.side + align256((size_t)(K / 64) * l.Mpad * 8);
  l.bytes = l.row_exp + align256((size_t)l.Mpad * 4);
  return l;
}

}  // namespace rw4

namespace {

using namespace rw4;
using namespace rw4::gemv_tma;

constexpr int kPrepThreads = 256;

// One CTA per row m < Mpad; rows M..Mpad-1 only zero their side pairs and exponent.
__global__ void __launch_bounds__(kPrepThreads)
    rw4_xprep_kernel(const __nv_bfloat16* __restrict__ x, int M, int K, int Mpad,
                     uint4* __restrict__ xf, float2* __restrict__ side, int* __restrict__ row_exp,
                     const __nv_bfloat16* __restrict__ nw, float eps) {
  const int m = blockIdx.x;
  const int G = K / 64;
  // x comes from the previous kernel on the stream; the GEMV after us may start launching now (it
  // reads nothing of ours before its own griddepcontrol.wait, which waits for this grid)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (m >= M) {
    for (int g = threadIdx.x; g < G; g += kPrepThreads)
      side[(int64_t)g * Mpad + m] = make_float2(0.f, 0.f);
    if (threadIdx.x == 0) row_exp[m] = 0;
    return;
  }
  const __nv_bfloat16* xr = x + (int64_t)m * K;
  // 0. with a norm: the row's scale, summed in rw4_rmsnorm's order (strided per thread, the warp
  //    butterfly, the warps in order)
  static_assert(kPrepThreads == 256, "rms_scale sums over 256 threads");
  float r = 1.f;
  if (nw) {
    __shared__ float wss[kPrepThreads / 32];
    r = frag::rms_scale(xr, K, eps, threadIdx.x, wss, [] { __syncthreads(); });
  }
  auto load8 = [&](int i) {   // 8 values of the (normalised) row starting at 8 i
    const uint4 v = ldg_u4(xr + 8 * i);
    return nw ? frag::norm8(v, ldg_u4(nw + 8 * i), r) : v;
  };
  // 1. largest magnitude
  uint32_t mx = 0;
  for (int i = threadIdx.x; i < K / 8; i += kPrepThreads)
    mx = max(mx, frag::absmax8(load8(i)));
  mx = __reduce_max_sync(0xFFFFFFFFu, mx);
  __shared__ uint32_t wmax[kPrepThreads / 32];
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = mx;
  __syncthreads();
  uint32_t a = 0;
#pragma unroll
  for (int w = 0; w < kPrepThreads / 32; ++w) a = max(a, wmax[w]);
  const int e = frag::row_exponent(a);
  if (threadIdx.x == 0) row_exp[m] = e;
  float p1, p2;
  frag::exp_factors(e, p1, p2);
  // 2. convert, 16 values per thread; the 4 chunks of a group sit on 4 consecutive lanes
  const int chunks = K / 16;
  for (int base = 0; base < chunks; base += kPrepThreads) {
    const int c = base + threadIdx.x;
    float xs = 0.f, hs = 0.f;
    if (c < chunks) {
      uint32_t o[8];
      frag::x16_to_f16_frag(load8(2 * c), load8(2 * c + 1), p1, p2, o, xs, hs);
      uint4* dst = xf + ((int64_t)m * K + 16 * c) / 8;
      dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
      dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
    frag::group_sums(xs, hs);
    if (c < chunks && (c & 3) == 0)
      side[(int64_t)(c >> 2) * Mpad + m] = make_float2(xs, -1024.f * hs);
  }
}

// Two CTAs per SM: the register cap this implies (<= 113 per thread) measurably improves the
// schedule (16 consumer warps per SM sharing the ALU pipe with the producers).  KS > 1 splits K
// over a (1, 1, KS) thread-block cluster (grid.z = KS) reduced through distributed shared memory.
// M1: one activation row.  XQ (with M1): the CTA converts that row itself (no x-prep launch, no
// workspace); otherwise the x-prep output arrives through the TMA ring.  SW: W is [gate; up] (N
// rows, gate first) and y [M, N / 2] = act_fn(gate) * up; a CTA takes BR / 2 gate rows and the
// matching up rows.
template <int NT, int R, int S, int KS, bool M1, bool XQ, bool SW = false>
__global__ void __cluster_dims__(1, 1, KS) __launch_bounds__(kThreads, 2)
    rw4_gemv_tma_kernel(const __grid_constant__ CUtensorMap tm_codes,
                        const __grid_constant__ CUtensorMap tm_scale,
                        const __grid_constant__ CUtensorMap tm_zero,
                        const __grid_constant__ CUtensorMap tm_x,
                        const __grid_constant__ CUtensorMap tm_side, const int* row_exp,
                        const __nv_bfloat16* __restrict__ x, int bm, int M, int K, int N,
                        __nv_bfloat16* __restrict__ y, unsigned int* status,
                        const __nv_bfloat16* __restrict__ res,
                        const __nv_bfloat16* __restrict__ nw, float eps) {
  // batch slices are the fastest grid dimension: the CTAs of all slices of one row tile run
  // together, so the slices after the first find the tile's weights in L2
  const int m0 = blockIdx.x * 16;
  const int n_out = SW ? N / 2 : N;   // output columns (= the row stride of y)
  body<NT, R, S, SW, KS, !XQ, M1, !XQ, XQ>(&tm_codes, &tm_scale, &tm_zero, &tm_x, &tm_side,
                                           row_exp, x, m0, bm, min(16, M - m0), K,
                                           y + (int64_t)m0 * n_out, n_out,
                                           blockIdx.y * (SW ? Layout<R, S>::BR / 2
                                                            : Layout<R, S>::BR),
                                           n_out, SW ? N / 2 : 0, status,
                                           res ? res + (int64_t)m0 * n_out : nullptr,
                                           XQ ? nw : nullptr, eps);
}

bool pdl_enabled() {
  static const bool off = getenv("RW4_NO_PDL") != nullptr;
  return !off;
}

// Smallest dynamic shared memory request that keeps a third CTA off an SM (228 KB per SM, 1 KB
// reserved per CTA).
constexpr int kTwoPerSmSmem = 228 * 1024 / 3 + 1024;

cudaLaunchAttribute pdl_attr() {
  cudaLaunchAttribute a;
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  return a;
}

int launch_xprep(const void* x, int M, int K, const XPrepLayout& l, uint8_t* ws,
                 cudaStream_t stream, const XNorm* norm = nullptr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)l.Mpad);
  cfg.blockDim = dim3(kPrepThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1] = {pdl_attr()};
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(
      &cfg, rw4_xprep_kernel, static_cast<const __nv_bfloat16*>(x), M, K, (int)l.Mpad,
      reinterpret_cast<uint4*>(ws + l.xf), reinterpret_cast<float2*>(ws + l.side),
      reinterpret_cast<int*>(ws + l.row_exp),
      norm ? static_cast<const __nv_bfloat16*>(norm->weight) : nullptr, norm ? norm->eps : 0.f);
  if (err != cudaSuccess) return cuda_status(err, "rw4 x-prep launch");
  return launch_status("rw4 x-prep launch");
}

}  // namespace

namespace rw4 {
int xprep_launch(const void* x, int M, int K, const XPrepLayout& l, uint8_t* ws,
                 cudaStream_t stream, const XNorm* norm) {
  return launch_xprep(x, M, K, l, ws, stream, norm);
}
}  // namespace rw4

namespace {

// One activation row whose CTA K range fits the in-kernel conversion's shared memory: the GEMV
// converts it itself (XQ).  Everything else goes through the x-prep pass.
bool one_row_in_kernel(int64_t M, int64_t K, int ks) {
  return M == 1 && ((K / kStageK) + ks - 1) / ks <= Layout<1, 1>::kXQMaxStages;
}

template <int NT, int R, int S, int KS = 1, bool SW = false>
int launch_tma(const void* x, int M, int K, const uint8_t* wq, const void* sc, const void* zr,
               int N, void* y, const XPrepLayout& l, uint8_t* ws, cudaStream_t stream,
               const void* res, const XNorm* norm) {
  using L = Layout<R, S>;
  static_assert(L::kBars >= kConsumers * L::BR * (16 * NT + 1) * 4,
                "reduction buffer must fit in the ring below the barriers");
  static_assert(!SW || R % 2 == 0, "SwiGLU pairs gate and up row tiles");
  if (SW && (N % 2 || res)) return fail(RW4_EINVAL, "gemv_tma: SwiGLU takes [gate; up], no residual");
  // weight rows per box and per CTA: BR, or BR / 2 gate rows + BR / 2 up rows
  const int box_rows = SW ? L::BR / 2 : L::BR;
  CUtensorMap tc, ts, tz, tx, tside;
  const int G = K / 64;
  // activation rows per slice: the whole batch for M <= 8 (NT = 1), 16-row slices above
  const int bm = M < 16 ? M : 16;
  if (bm > 8 * NT) return fail(RW4_EINVAL, "gemv_tma: %d activation rows for NT=%d", M, NT);
  const bool xq = NT == 1 && one_row_in_kernel(M, K, KS);
  if (norm && !xq) return fail(RW4_EINVAL, "gemv_tma: the norm belongs to the x-prep pass here");
  int st = make_tensor_map_2d(&tc, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K / 2, K / 2,
                              box_rows, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&ts, sc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, N, G, (uint64_t)G * 2,
                            box_rows, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&tz, zr, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, N, G, (uint64_t)G * 2,
                            box_rows, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st != RW4_OK) return st;
  if (xq) {
    tx = tz;  // not read by the in-kernel conversion
    tside = tz;
  } else {
    st = make_tensor_map_2d(&tx, ws + l.xf, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, M, K,
                            (uint64_t)K * 2, bm, 256, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st == RW4_OK)
      st = make_tensor_map_2d(&tside, ws + l.side, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, G,
                              2 * l.Mpad, (uint64_t)l.Mpad * 8, 8, 2 * L::side_rows(bm),
                              CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != RW4_OK) return st;
  }
  const bool m1 = NT == 1 && M == 1;
  const int variant = xq ? 2 : m1 ? 1 : 0;
  auto kern = xq ? rw4_gemv_tma_kernel<NT, R, S, KS, NT == 1, NT == 1, SW>
              : m1 ? rw4_gemv_tma_kernel<NT, R, S, KS, NT == 1, false, SW>
                   : rw4_gemv_tma_kernel<NT, R, S, KS, false, false, SW>;
  // The dynamic shared memory limit is a per-device function attribute: set it once per device
  // and kernel variant (this function is instantiated once per launch shape).
  static std::atomic<uint32_t> attr_set[3];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set[variant].load() & (1u << dev))) {
    const int largest = xq ? L::dyn_smem_xq(L::kXQMaxStages) : L::dyn_smem_xp(8 * NT);
    const int most = largest > kTwoPerSmSmem ? largest : kTwoPerSmSmem;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, most) !=
        cudaSuccess)
      return fail(RW4_ECUDA, "gemv_tma: cannot set dynamic shared memory size");
    attr_set[variant].fetch_or(1u << dev);
  }
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "gemv_tma: device status word unavailable");
  const int64_t tiles = ((SW ? N / 2 : N) + box_rows - 1) / box_rows;
  if (tiles > 65535) return fail(RW4_EINVAL, "gemv_tma: N=%d needs more than 65535 row tiles", N);
  dim3 grid((M + 15) / 16, (unsigned)tiles, KS);
  // Programmatic dependent launch: this grid may start while the kernel before it (the x-prep pass,
  // or whatever produced x) runs; it streams its weights at once and waits (griddepcontrol.wait)
  // only before it reads x.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  // At most two CTAs per SM: with smaller rings the block scheduler may stack three or four CTAs
  // of a one-wave grid on some SMs and leave others idle (measured: M=1 slower than M=8 on the
  // 4096-row shapes until the shared-memory request made a third CTA impossible).
  const int cta_stages = ((K / kStageK) + KS - 1) / KS;
  const int smem_need = xq ? L::dyn_smem_xq(cta_stages) : L::dyn_smem_xp(bm);
  cfg.dynamicSmemBytes = smem_need > kTwoPerSmSmem ? smem_need : kTwoPerSmSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1] = {pdl_attr()};
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kern, tc, ts, tz, tx, tside,
                                       reinterpret_cast<const int*>(ws + l.row_exp),
                                       static_cast<const __nv_bfloat16*>(x), bm, M, K, N,
                                       static_cast<__nv_bfloat16*>(y), status,
                                       static_cast<const __nv_bfloat16*>(res),
                                       norm ? static_cast<const __nv_bfloat16*>(norm->weight)
                                            : nullptr,
                                       norm ? norm->eps : 0.f);
  if (err != cudaSuccess) return cuda_status(err, "rw4 gemv_tma launch");
  return launch_status("rw4 gemv_tma launch");
}

}  // namespace

namespace rw4 {

bool gemv_tma_supported(int64_t K) { return K % kStageK == 0; }

// Launch shape policy (measured on the isolated sweep and the Llama / Mixtral projection shapes).
// The K split is a function of the weight's shape alone, taken from the one-row launch: every
// batch size then adds a row's partial sums in the same order, so a row's output has the same bits
// at every M.  Wider CTAs amortise the per-stage work (x fragment, barrier) over more weight rows
// and win whenever they still give about 1.3 CTAs per SM (>= 192 of the 296 two-per-SM slots;
// measured: 4096 x 6144 at one row runs 6.5 us as 192 unsplit 32-row CTAs against 8.9 us as 384
// CTAs with K split in two, and 11.7 against 15.3 us at 16 rows):
// 64-row CTAs from N >= 12288, then 32-row CTAs, then 16-row CTAs, each with K split over a
// cluster of up to 4 CTAs (keeping >= 2 stages per CTA) to reach that count.  More than 8
// activation rows (two MMA column tiles) use at most 32-row CTAs.
void gemv_tma_policy(int64_t M, int64_t K, int64_t N, int* row_tiles, int* ksplit) {
  constexpr int64_t kTarget = 192;
  const int64_t nst = K / kStageK;
  auto ctas = [&](int r) { return (N + 16 * r - 1) / (16 * r); };
  auto split_for = [&](int r) {
    int ks = 1;
    while (ks < 4 && ctas(r) * ks < kTarget && nst / (ks * 2) >= 2) ks *= 2;
    return ks;
  };
  int r1 = 1, ks = 1;
  if (ctas(4) >= kTarget) {
    r1 = 4;
  } else {
    for (int r : {2, 1}) {
      ks = split_for(r);
      if (ctas(r) * ks >= kTarget || r == 1) {
        r1 = r;
        break;
      }
    }
  }
  *ksplit = ks;
  *row_tiles = M > 8 && r1 > 2 ? 2 : r1;
}

// Workspace the call needs: none when the one-row kernel converts x itself.
size_t gemv_tma_workspace(int64_t M, int64_t K, int64_t N) {
  int rt = 1, ks = 1;
  gemv_tma_policy(M, K, N, &rt, &ks);
  return one_row_in_kernel(M, K, ks) ? 0 : xprep_layout(M, K).bytes;
}

// The launch shape a call takes: the measured policy, unless RW4_GEMV_ROW_TILES (row_tiles) or
// RW4_GEMV_KSPLIT force one (measurements only: a forced K split changes the order in which a
// row's sums are added).
static void launch_shape(int64_t M, int64_t K, int64_t N, int row_tiles, int* rt, int* ks) {
  static const int forced_ks = [] {
    const char* e = getenv("RW4_GEMV_KSPLIT");
    return e ? atoi(e) : 0;
  }();
  int policy_rt = 1;
  gemv_tma_policy(M, K, N, &policy_rt, ks);
  if (row_tiles != 1 && row_tiles != 2 && row_tiles != 4) row_tiles = policy_rt;
  if (forced_ks == 1 || forced_ks == 2 || forced_ks == 4) *ks = forced_ks;
  if (row_tiles == 4 && (M > 8 || *ks > 1)) row_tiles = 2;
  *rt = row_tiles;
}

// Everything before the GEMV launch itself: the x-prep pass (with the norm) unless the one-row
// kernel converts x itself; *kn is the norm that kernel applies.
static int prepare_x(const void* x, int64_t M, int64_t K, int ks, void* ws, size_t ws_bytes,
                     cudaStream_t s, const XNorm* norm, const XNorm** kn) {
  if ((M + 15) / 16 > 65535) return fail(RW4_EINVAL, "rw4_linear: M=%lld too large", (long long)M);
  const bool xq = one_row_in_kernel(M, K, ks);
  *kn = xq ? norm : nullptr;
  if (xq) return RW4_OK;
  const XPrepLayout l = xprep_layout(M, K);
  if (!ws || ws_bytes < l.bytes)
    return fail(RW4_EINVAL, "rw4_linear: the GEMV needs a %zu-byte workspace (got %zu)", l.bytes,
                ws_bytes);
  if (!aligned(ws, 256)) return fail(RW4_EINVAL, "rw4_linear: workspace must be 256-byte aligned");
  return launch_xprep(x, (int)M, (int)K, l, static_cast<uint8_t*>(ws), s, norm);
}

int gemv_tma_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                    const void* zr, int64_t N, void* y, cudaStream_t s, int row_tiles, void* ws,
                    size_t ws_bytes, const void* res, const XNorm* norm) {
  const int Mi = (int)M, Ki = (int)K, Ni = (int)N;
  int ks = 1;
  launch_shape(M, K, N, row_tiles, &row_tiles, &ks);
  // the norm runs in the activation conversion: the GEMV's own for one row, else the x-prep pass
  const XNorm* kn = nullptr;
  const int pst = prepare_x(x, M, K, ks, ws, ws_bytes, s, norm, &kn);
  if (pst != RW4_OK) return pst;
  const XPrepLayout l = xprep_layout(M, K);
  uint8_t* w = static_cast<uint8_t*>(ws);
  if (M <= 8) {
    if (row_tiles == 4) return launch_tma<1, 4, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
    if (row_tiles == 2) {
      if (ks == 4) return launch_tma<1, 2, 6, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
      if (ks == 2) return launch_tma<1, 2, 6, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
      return launch_tma<1, 2, 6>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
    }
    if (ks == 4) return launch_tma<1, 1, 8, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
    if (ks == 2) return launch_tma<1, 1, 8, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
    return launch_tma<1, 1, 8>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
  }
  // 9..16 activation rows per slice: 16 KB of x per stage, so shallower rings keep two CTAs per SM
  if (row_tiles >= 2) {
    if (ks == 4) return launch_tma<2, 2, 4, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
    if (ks == 2) return launch_tma<2, 2, 4, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
    return launch_tma<2, 2, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
  }
  if (ks == 4) return launch_tma<2, 1, 4, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
  if (ks == 2) return launch_tma<2, 1, 4, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
  return launch_tma<2, 1, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, res, kn);
}

// SwiGLU form: y[M, N / 2] = act_fn(x W_gate^T) * (x W_up^T) for W = [gate; up] (N rows, gate
// first), in one launch.  It takes the plain call's launch shape for the N-row weight, so gate
// and up get the plain GEMV's bits, and the epilogue rounds as rw4_silu_mul does; supported where
// that shape has no K split (the 64-row shape becomes 32 gate + 32 up rows, the 16-row one 8 + 8
// would not pair, so 16-row shapes run as 32-row ones: a row's sums do not depend on the CTA's
// height).
bool gemv_tma_swiglu_supported(int64_t M, int64_t K, int64_t N) {
  if (M < 1 || M > 64 || N < 2 || N % 2 || !gemv_tma_supported(K)) return false;
  int rt = 1, ks = 1;
  launch_shape(M, K, N, 0, &rt, &ks);
  return ks == 1;
}

int gemv_tma_swiglu_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq,
                           const void* sc, const void* zr, int64_t N, void* y, cudaStream_t s,
                           void* ws, size_t ws_bytes, const XNorm* norm) {
  if (!gemv_tma_swiglu_supported(M, K, N))
    return fail(RW4_EUNSUPPORTED, "gemv_tma: no one-launch SwiGLU for M=%lld K=%lld N=%lld",
                (long long)M, (long long)K, (long long)N);
  const int Mi = (int)M, Ki = (int)K, Ni = (int)N;
  int rt = 1, ks = 1;
  launch_shape(M, K, N, 0, &rt, &ks);
  const XNorm* kn = nullptr;
  const int pst = prepare_x(x, M, K, ks, ws, ws_bytes, s, norm, &kn);
  if (pst != RW4_OK) return pst;
  const XPrepLayout l = xprep_layout(M, K);
  uint8_t* w = static_cast<uint8_t*>(ws);
  if (M <= 8) {
    if (rt == 4)
      return launch_tma<1, 4, 4, 1, true>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, nullptr, kn);
    return launch_tma<1, 2, 6, 1, true>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, nullptr, kn);
  }
  return launch_tma<2, 2, 4, 1, true>(x, Mi, Ki, wq, sc, zr, Ni, y, l, w, s, nullptr, kn);
}

}  // namespace rw4
