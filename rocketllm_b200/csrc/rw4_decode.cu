// Decode-step kernels around the RW4 GEMVs: the ops a Llama-family decoder layer runs between its
// projections, each one launch, each reproducing the rounding sequence of the bf16 transformers
// module it replaces (transformers models/llama/modeling_llama.py), so that a fused decode step
// stays within rounding of the module-by-module one:
//
//   rw4_rmsnorm        LlamaRMSNorm: fp32 mean of squares, x * rsqrt(mean + eps) rounded to bf16,
//                      times the bf16 weight (rounded again)                 [:48-68]
//   rw4_rope_kv        apply_rotary_pos_emb on q and k with bf16 cos / sin (each product and the
//                      sum rounded to bf16), k and v written into a static [B, KVH, T, D] cache at
//                      the device-side position                            [:78-112, StaticCache]
//   rw4_silu_mul       act_fn(gate) * up for a concatenated [gate | up] row: silu in fp32 rounded
//                      to bf16, the product rounded to bf16                  [:171-184]
//   rw4_linear_rmsnorm_ws    linear(rmsnorm(x)): a projection after the layer's norm, the norm
//                      folded into the activation conversion (the one-row GEMV's prologue or the
//                      x-prep pass)
//   rw4_linear_rmsnorm_swiglu_ws   act_fn(gate) * up of linear(rmsnorm(x)) over a [gate; up]
//                      weight: the MLP's first half in the GEMV's epilogue
//   rw4_linear_residual_ws   residual + linear(x): the GEMV with the residual added in its epilogue
//                      (the product rounded to bf16 first, then the sum), as a decoder layer's
//                      `hidden_states = residual + self_attn(...)` / `+ mlp(...)`.
//   rw4_argmax_rows    the greedy choice over the vocabulary, torch.argmax(scores, dim=-1)
//                      (transformers generation/utils.py, the greedy branch of _sample)
// All are memory-bound and tiny at decode batch sizes; their point is the launch count (about 1,600
// small kernels per Llama-8B token through the modules, 5 per layer here besides attention).  They
// are launched with programmatic dependent launch: each waits for the kernel before it
// (griddepcontrol.wait) before it touches memory, then lets the next one launch, so the following
// GEMV streams its first weight stages while they run.
#include <cooperative_groups.h>

#include <climits>

#include "rw4_common.cuh"
#include "rw4_xprep.cuh"

namespace rw4 {
int check_linear_args(const char* who, const void* x, int64_t M, int64_t K, const uint8_t* wq,
                      const void* sc, const void* zr, int64_t N, int32_t group, const void* y);
int gemv_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                const void* zr, int64_t N, void* y, cudaStream_t s, void* ws, size_t ws_bytes);
bool gemv_tma_supported(int64_t K);
int gemv_tma_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                    const void* zr, int64_t N, void* y, cudaStream_t s, int row_tiles, void* ws,
                    size_t ws_bytes, const void* res, const XNorm* norm = nullptr);
size_t gemv_workspace(int64_t M, int64_t K, int64_t N);
bool gemv_tma_swiglu_supported(int64_t M, int64_t K, int64_t N);
int gemv_tma_swiglu_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq,
                           const void* sc, const void* zr, int64_t N, void* y, cudaStream_t s,
                           void* ws, size_t ws_bytes, const XNorm* norm);
bool gemm_skinny_supported(int64_t M, int64_t K, int64_t N);
int gemm_skinny_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                       const void* zr, int64_t N, void* y, cudaStream_t s, void* ws,
                       size_t ws_bytes, const void* res, const XNorm* norm = nullptr);
}  // namespace rw4

namespace {

using rw4::fail;

__device__ __forceinline__ float bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Start of every kernel here: wait for the previous grid's writes, then release the next grid.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

bool pdl_on() {
  static const bool off = getenv("RW4_NO_PDL") != nullptr;
  return !off;
}

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, const char* what,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_on() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (err != cudaSuccess) return rw4::cuda_status(err, what);
  return rw4::launch_status(what);
}

constexpr int kNormThreads = 256;

// One CTA per row.
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                   int H, float eps, __nv_bfloat16* __restrict__ y) {
  pdl_enter();
  const __nv_bfloat16* xr = x + (int64_t)blockIdx.x * H;
  __nv_bfloat16* yr = y + (int64_t)blockIdx.x * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += kNormThreads) {
    const float v = __bfloat162float(xr[i]);
    ss = fmaf(v, v, ss);
  }
  ss += __shfl_xor_sync(0xFFFFFFFFu, ss, 16);
  ss += __shfl_xor_sync(0xFFFFFFFFu, ss, 8);
  ss += __shfl_xor_sync(0xFFFFFFFFu, ss, 4);
  ss += __shfl_xor_sync(0xFFFFFFFFu, ss, 2);
  ss += __shfl_xor_sync(0xFFFFFFFFu, ss, 1);
  __shared__ float part[kNormThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += part[i];
  const float r = rsqrtf(tot / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += kNormThreads)
    yr[i] = __float2bfloat16_rn(__bfloat162float(w[i]) * bf(__bfloat162float(xr[i]) * r));
}

// One thread per (row, head, pair d < D/2) of q heads then k heads; v is copied by the k threads.
// q/k/v rows have element strides ld (a concatenated q|k|v projection output); cos / sin [rows, D]
// bf16; the cache is [B, KVH, T, D] with row b's token written at position *pos.
__global__ void rope_kv_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                               const __nv_bfloat16* __restrict__ v, int64_t ld, int rows, int Hq,
                               int Hk, int D, const __nv_bfloat16* __restrict__ cosv,
                               const __nv_bfloat16* __restrict__ sinv, const int64_t* __restrict__ pos,
                               int64_t T, __nv_bfloat16* __restrict__ q_out,
                               __nv_bfloat16* __restrict__ k_cache,
                               __nv_bfloat16* __restrict__ v_cache) {
  pdl_enter();
  const int half = D / 2;
  const int64_t total = (int64_t)rows * (Hq + Hk) * half;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % half);
  const int h = (int)((i / half) % (Hq + Hk));
  const int b = (int)(i / ((int64_t)half * (Hq + Hk)));
  const __nv_bfloat16* cs = cosv + (int64_t)b * D;
  const __nv_bfloat16* sn = sinv + (int64_t)b * D;
  const float c0 = __bfloat162float(cs[d]), c1 = __bfloat162float(cs[d + half]);
  const float s0 = __bfloat162float(sn[d]), s1 = __bfloat162float(sn[d + half]);
  const bool is_q = h < Hq;
  const int hh = is_q ? h : h - Hq;
  const __nv_bfloat16* src = (is_q ? q : k) + (int64_t)b * ld + (int64_t)hh * D;
  const float a = __bfloat162float(src[d]), bb = __bfloat162float(src[d + half]);
  // x * cos + rotate_half(x) * sin, rotate_half(x) = cat(-x[half:], x[:half]); each op in bf16
  const float o0 = bf(bf(a * c0) + bf(-bb * s0));
  const float o1 = bf(bf(bb * c1) + bf(a * s1));
  if (is_q) {
    __nv_bfloat16* dst = q_out + ((int64_t)b * Hq + hh) * D;
    dst[d] = __float2bfloat16_rn(o0);
    dst[d + half] = __float2bfloat16_rn(o1);
  } else {
    const int64_t p = pos[0];
    if (p < 0 || p >= T) return;  // the caller checks the position on the host
    const int64_t off = (((int64_t)b * Hk + hh) * T + p) * D;
    k_cache[off + d] = __float2bfloat16_rn(o0);
    k_cache[off + d + half] = __float2bfloat16_rn(o1);
    const __nv_bfloat16* vs = v + (int64_t)b * ld + (int64_t)hh * D;
    v_cache[off + d] = vs[d];
    v_cache[off + d + half] = vs[d + half];
  }
}

// out[r, i] = bf16(bf16(silu(g)) * u) with g = gu[r, i], u = gu[r, I + i].
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int rows, int I,
                                __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)rows * I) return;
  const int64_t r = i / I, c = i % I;
  const float g = __bfloat162float(gu[r * 2 * I + c]);
  const float u = __bfloat162float(gu[r * 2 * I + I + c]);
  out[i] = __float2bfloat16_rn(bf(g / (1.f + expf(-g))) * u);
}

// y = bf16(y + r) elementwise (the residual add after a GEMV that had no epilogue for it).
__global__ void add_kernel(__nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ r,
                           int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2bfloat16_rn(__bfloat162float(y[i]) + __bfloat162float(r[i]));
}

// ---- greedy token choice -----------------------------------------------------------------------
// out[r] = the index of row r's largest bf16 score: the first index among equal maxima, and a NaN
// counts as larger than every number (torch.argmax's rule on CUDA).  One thread-block cluster of
// kArgmaxCluster CTAs per row, each CTA a contiguous share of the row; the CTAs' winners meet in
// CTA 0 through distributed shared memory, so one launch reads the row once with no global
// scratch.  (At 128,256 scores torch's reduction runs one CTA per row.)
constexpr int kArgmaxCluster = 8;
constexpr int kArgmaxThreads = 256;

// (a, ia) wins over (b, ib)
__device__ __forceinline__ bool argmax_better(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na != nb) return na;
  if (!na && a != b) return a > b;
  return ia < ib;
}

__global__ void __launch_bounds__(kArgmaxThreads)
    argmax_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld, int V, bool vec,
                  int64_t* __restrict__ out) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float wv[kArgmaxThreads / 32];
  __shared__ int wi[kArgmaxThreads / 32];
  __shared__ float cta_v;
  __shared__ int cta_i;
  pdl_enter();
  const int c = (int)cluster.block_rank();
  const __nv_bfloat16* xr = x + (int64_t)blockIdx.y * ld;
  // this CTA's share, a multiple of 8 scores
  const int per = ((V + kArgmaxCluster - 1) / kArgmaxCluster + 7) & ~7;
  const int beg = min(V, c * per), end = min(V, beg + per);
  float bv = -INFINITY;
  int bi = INT_MAX;
  if (vec) {
    // each thread walks its 8-score vectors in increasing order, so a strict win keeps the first
    for (int i = beg + 8 * (int)threadIdx.x; i < end; i += 8 * kArgmaxThreads) {
      const uint4 raw = *reinterpret_cast<const uint4*>(xr + i);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = __bfloat162float(e[j]);
        if (argmax_better(v, i + j, bv, bi)) {
          bv = v;
          bi = i + j;
        }
      }
    }
  } else {
    for (int i = beg + (int)threadIdx.x; i < end; i += kArgmaxThreads) {
      const float v = __bfloat162float(xr[i]);
      if (argmax_better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
    if (argmax_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    wv[warp] = bv;
    wi[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgmaxThreads / 32; ++w)
      if (argmax_better(wv[w], wi[w], bv, bi)) {
        bv = wv[w];
        bi = wi[w];
      }
    cta_v = bv;
    cta_i = bi;
  }
  cluster.sync();   // every CTA's winner is in its shared memory
  if (c == 0 && threadIdx.x == 0) {
    for (int q = 1; q < kArgmaxCluster; ++q) {
      const float qv = *cluster.map_shared_rank(&cta_v, q);
      const int qi = *cluster.map_shared_rank(&cta_i, q);
      if (argmax_better(qv, qi, bv, bi)) {
        bv = qv;
        bi = qi;
      }
    }
    out[blockIdx.y] = bi;
  }
  cluster.sync();   // no CTA leaves while CTA 0 still reads its shared memory
}

unsigned blocks(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace

extern "C" int rw4_argmax_rows(const void* scores_bf16, int64_t rows, int64_t V, int64_t ld,
                               int64_t* out, void* stream) {
  if (rows < 0 || V <= 0 || V > INT_MAX - 8 * kArgmaxThreads || ld < V)   // int indices
    return fail(RW4_EINVAL, "rw4_argmax_rows: bad shape (rows %lld, V %lld, ld %lld)",
                (long long)rows, (long long)V, (long long)ld);
  if (rows == 0) return RW4_OK;
  if (!scores_bf16 || !out) return fail(RW4_EINVAL, "rw4_argmax_rows: null pointer");
  if (rows > 65535) return fail(RW4_EINVAL, "rw4_argmax_rows: more than 65535 rows");
  // 16-byte loads when every row starts aligned and holds whole vectors (no load past V)
  const bool vec = rw4::aligned(scores_bf16, 16) && ld % 8 == 0 && V % 8 == 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kArgmaxCluster, (unsigned)rows);
  cfg.blockDim = dim3(kArgmaxThreads);
  cfg.stream = rw4::as_stream(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kArgmaxCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_on() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err =
      cudaLaunchKernelEx(&cfg, argmax_kernel, static_cast<const __nv_bfloat16*>(scores_bf16), ld,
                         (int)V, vec, out);
  if (err != cudaSuccess) return rw4::cuda_status(err, "rw4_argmax_rows launch");
  return rw4::launch_status("rw4_argmax_rows launch");
}

extern "C" int rw4_rmsnorm(const void* x, const void* weight, int64_t rows, int64_t H, float eps,
                           void* y, void* stream) {
  if (rows < 0 || H <= 0 || H > (1 << 24)) return fail(RW4_EINVAL, "rw4_rmsnorm: bad shape");
  if (rows == 0) return RW4_OK;
  if (!x || !weight || !y) return fail(RW4_EINVAL, "rw4_rmsnorm: null pointer");
  if (rows > 65535) return fail(RW4_EINVAL, "rw4_rmsnorm: more than 65535 rows");
  return launch_pdl(rmsnorm_kernel, dim3((unsigned)rows), dim3(kNormThreads),
                    rw4::as_stream(stream), "rw4_rmsnorm launch",
                    static_cast<const __nv_bfloat16*>(x),
                    static_cast<const __nv_bfloat16*>(weight), (int)H, eps,
                    static_cast<__nv_bfloat16*>(y));
}

extern "C" int rw4_rope_kv(const void* q, const void* k, const void* v, int64_t ld, int32_t rows,
                           int32_t heads, int32_t kv_heads, int32_t head_dim, const void* cos_bf16,
                           const void* sin_bf16, const int64_t* pos, int64_t cache_len,
                           void* q_out, void* k_cache, void* v_cache, void* stream) {
  if (rows < 0 || heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 2 || cache_len <= 0)
    return fail(RW4_EINVAL, "rw4_rope_kv: bad shape");
  if (rows == 0) return RW4_OK;
  if (!q || !k || !v || !cos_bf16 || !sin_bf16 || !pos || !q_out || !k_cache || !v_cache)
    return fail(RW4_EINVAL, "rw4_rope_kv: null pointer");
  const int64_t n = (int64_t)rows * (heads + kv_heads) * (head_dim / 2);
  return launch_pdl(rope_kv_kernel, dim3(blocks(n, 256)), dim3(256), rw4::as_stream(stream),
                    "rw4_rope_kv launch", static_cast<const __nv_bfloat16*>(q),
                    static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v),
                    ld, (int)rows, (int)heads, (int)kv_heads, (int)head_dim,
                    static_cast<const __nv_bfloat16*>(cos_bf16),
                    static_cast<const __nv_bfloat16*>(sin_bf16), pos, cache_len,
                    static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cache),
                    static_cast<__nv_bfloat16*>(v_cache));
}

extern "C" int rw4_silu_mul(const void* gate_up, int64_t rows, int64_t I, void* out, void* stream) {
  if (rows < 0 || I <= 0) return fail(RW4_EINVAL, "rw4_silu_mul: bad shape");
  if (rows == 0) return RW4_OK;
  if (!gate_up || !out) return fail(RW4_EINVAL, "rw4_silu_mul: null pointer");
  return launch_pdl(silu_mul_kernel, dim3(blocks(rows * I, 256)), dim3(256),
                    rw4::as_stream(stream), "rw4_silu_mul launch",
                    static_cast<const __nv_bfloat16*>(gate_up), (int)rows, (int)I,
                    static_cast<__nv_bfloat16*>(out));
}

namespace {
// On the TMA path the rows are normalised inside the activation conversion (the one-row GEMV's
// own prologue, the x-prep pass, or the decode GEMM's x-prep pass); otherwise rw4_rmsnorm writes
// the normalised rows into the workspace first.
bool norm_folded(int64_t K) {
  static const bool no_tma = getenv("RW4_GEMV_NO_TMA") != nullptr;
  return !no_tma && rw4::gemv_tma_supported(K);
}
}  // namespace

// Workspace of rw4_linear_rmsnorm_ws: the linear's own, plus room for the normalised rows when the
// norm is not folded into the conversion.
extern "C" int rw4_linear_rmsnorm_workspace_size(int64_t M, int64_t K, int64_t N, size_t* bytes) {
  if (!bytes) return fail(RW4_EINVAL, "rw4_linear_rmsnorm_workspace_size: null output");
  if (M < 0 || K <= 0 || N < 0 || K % 64)
    return fail(RW4_EINVAL, "rw4_linear_rmsnorm_workspace_size: bad shape");
  const size_t lin = (M > 0 && N > 0) ? rw4::gemv_workspace(M, K, N) : 0;
  *bytes = norm_folded(K) ? lin : ((lin + 255) & ~size_t(255)) + (size_t)M * K * 2;
  return RW4_OK;
}

extern "C" int rw4_linear_rmsnorm_ws(const void* x_bf16, int64_t M, int64_t K,
                                     const void* norm_weight, float eps, const uint8_t* packed,
                                     const void* scale_f16, const void* zero_f16, int64_t N,
                                     int32_t group, void* y_bf16, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  using namespace rw4;
  int st = check_linear_args("rw4_linear_rmsnorm_ws", x_bf16, M, K, packed, scale_f16, zero_f16,
                             N, group, y_bf16);
  if (st != RW4_OK || M == 0 || N == 0) return st;
  if (!norm_weight || !aligned(norm_weight, 16))
    return fail(RW4_EINVAL, "rw4_linear_rmsnorm_ws: norm weight null or not 16-byte aligned");
  if (M > 64)
    return fail(RW4_EINVAL, "rw4_linear_rmsnorm_ws: M=%lld; at most 64 rows", (long long)M);
  size_t need = 0;
  st = rw4_linear_rmsnorm_workspace_size(M, K, N, &need);
  if (st != RW4_OK) return st;
  if (need && (!workspace || workspace_bytes < need || !aligned(workspace, 256)))
    return fail(RW4_EINVAL, "rw4_linear_rmsnorm_ws: needs a 256-byte aligned %zu-byte workspace",
                need);
  cudaStream_t s = as_stream(stream);
  const XNorm norm{norm_weight, eps};
  if (norm_folded(K)) {
    // the norm runs inside the activation conversion that the multi-row kernels start with
    if (M >= 49 && gemm_skinny_supported(M, K, N))
      return gemm_skinny_launch(x_bf16, M, K, packed, scale_f16, zero_f16, N, y_bf16, s,
                                workspace, workspace_bytes, nullptr, &norm);
    return gemv_tma_launch(x_bf16, M, K, packed, scale_f16, zero_f16, N, y_bf16, s, 0,
                           workspace, workspace_bytes, nullptr, &norm);
  }
  // no TMA path (K % 512 != 0): normalise, then the linear
  const size_t lin = (gemv_workspace(M, K, N) + 255) & ~size_t(255);
  uint8_t* xn = static_cast<uint8_t*>(workspace) + lin;
  st = rw4_rmsnorm(x_bf16, norm_weight, M, K, eps, xn, stream);
  if (st != RW4_OK) return st;
  return rw4_linear_ws(xn, M, K, packed, scale_f16, zero_f16, N, group, y_bf16, 0, workspace,
                       lin, stream);
}

// rw4_linear_rmsnorm_swiglu_ws in one launch: the TMA GEMV path (as rw4_linear_rmsnorm_ws would
// take it) with a launch shape the SwiGLU epilogue pairs; otherwise two calls through the
// workspace.
namespace {
bool swiglu_one_launch(int64_t M, int64_t K, int64_t N) {
  using namespace rw4;
  return norm_folded(K) && !(M >= 49 && gemm_skinny_supported(M, K, N)) &&
         gemv_tma_swiglu_supported(M, K, N);
}
}  // namespace

extern "C" int rw4_linear_rmsnorm_swiglu_workspace_size(int64_t M, int64_t K, int64_t N,
                                                        size_t* bytes) {
  if (!bytes) return fail(RW4_EINVAL, "rw4_linear_rmsnorm_swiglu_workspace_size: null output");
  if (N % 2) return fail(RW4_EINVAL, "rw4_linear_rmsnorm_swiglu_workspace_size: odd N");
  size_t lin = 0;
  const int st = rw4_linear_rmsnorm_workspace_size(M, K, N, &lin);
  if (st != RW4_OK) return st;
  *bytes = (M == 0 || N == 0 || swiglu_one_launch(M, K, N))
               ? lin
               : ((lin + 255) & ~size_t(255)) + (size_t)M * N * 2;
  return RW4_OK;
}

extern "C" int rw4_linear_rmsnorm_swiglu_ws(const void* x_bf16, int64_t M, int64_t K,
                                            const void* norm_weight, float eps,
                                            const uint8_t* packed, const void* scale_f16,
                                            const void* zero_f16, int64_t N, int32_t group,
                                            void* y_bf16, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  using namespace rw4;
  int st = check_linear_args("rw4_linear_rmsnorm_swiglu_ws", x_bf16, M, K, packed, scale_f16,
                             zero_f16, N, group, y_bf16);
  if (st != RW4_OK || M == 0 || N == 0) return st;
  if (N % 2) return fail(RW4_EINVAL, "rw4_linear_rmsnorm_swiglu_ws: N=%lld is not [gate; up]",
                         (long long)N);
  if (!norm_weight || !aligned(norm_weight, 16))
    return fail(RW4_EINVAL, "rw4_linear_rmsnorm_swiglu_ws: norm weight null or not 16-byte aligned");
  if (M > 64)
    return fail(RW4_EINVAL, "rw4_linear_rmsnorm_swiglu_ws: M=%lld; at most 64 rows", (long long)M);
  size_t need = 0;
  st = rw4_linear_rmsnorm_swiglu_workspace_size(M, K, N, &need);
  if (st != RW4_OK) return st;
  if (need && (!workspace || workspace_bytes < need || !aligned(workspace, 256)))
    return fail(RW4_EINVAL,
                "rw4_linear_rmsnorm_swiglu_ws: needs a 256-byte aligned %zu-byte workspace", need);
  cudaStream_t s = as_stream(stream);
  if (swiglu_one_launch(M, K, N)) {
    const XNorm norm{norm_weight, eps};
    return gemv_tma_swiglu_launch(x_bf16, M, K, packed, scale_f16, zero_f16, N, y_bf16, s,
                                  workspace, workspace_bytes, &norm);
  }
  // two calls: [gate | up] into the workspace, then act_fn(gate) * up
  size_t lin = 0;
  st = rw4_linear_rmsnorm_workspace_size(M, K, N, &lin);
  if (st != RW4_OK) return st;
  lin = (lin + 255) & ~size_t(255);
  uint8_t* gu = static_cast<uint8_t*>(workspace) + lin;
  st = rw4_linear_rmsnorm_ws(x_bf16, M, K, norm_weight, eps, packed, scale_f16, zero_f16, N, group,
                             gu, workspace, lin, stream);
  if (st != RW4_OK) return st;
  return rw4_silu_mul(gu, M, N / 2, y_bf16, stream);
}

extern "C" int rw4_linear_residual_ws(const void* x_bf16, int64_t M, int64_t K,
                                      const uint8_t* packed, const void* scale_f16,
                                      const void* zero_f16, int64_t N, int32_t group,
                                      const void* residual, void* y_bf16, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  using namespace rw4;
  int st = check_linear_args("rw4_linear_residual_ws", x_bf16, M, K, packed, scale_f16, zero_f16,
                             N, group, y_bf16);
  if (st != RW4_OK || M == 0 || N == 0) return st;
  if (!residual) return fail(RW4_EINVAL, "rw4_linear_residual_ws: null residual");
  if (M > 64)
    return fail(RW4_EINVAL, "rw4_linear_residual_ws: M=%lld; the GEMV takes at most 64 rows",
                (long long)M);
  cudaStream_t s = as_stream(stream);
  if (M >= 49 && gemm_skinny_supported(M, K, N))   // the path rw4_linear takes for these shapes
    return gemm_skinny_launch(x_bf16, M, K, packed, scale_f16, zero_f16, N, y_bf16, s, workspace,
                              workspace_bytes, residual);
  static const bool no_tma = getenv("RW4_GEMV_NO_TMA") != nullptr;
  if (!no_tma && gemv_tma_supported(K))
    return gemv_tma_launch(x_bf16, M, K, packed, scale_f16, zero_f16, N, y_bf16, s, 0, workspace,
                           workspace_bytes, residual);
  if (residual == y_bf16)
    return fail(RW4_EINVAL, "rw4_linear_residual_ws: K=%lld takes the register-staged GEMV, "
                "which cannot add in place", (long long)K);
  st = gemv_launch(x_bf16, M, K, packed, scale_f16, zero_f16, N, y_bf16, s, workspace,
                   workspace_bytes);
  if (st != RW4_OK) return st;
  add_kernel<<<blocks(M * N, 256), 256, 0, s>>>(static_cast<__nv_bfloat16*>(y_bf16),
                                                static_cast<const __nv_bfloat16*>(residual),
                                                M * N);
  return launch_status("rw4_linear_residual_ws add");
}
