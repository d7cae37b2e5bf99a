// RW4 codec kernels: dequantize (packed -> fp32/bf16/fp16) and quantize (fp32/bf16/fp16 ->
// packed).
//
// Both are bit-exact restatements of RocketLLM's int4 codec (rocketllm/quant/kv_cache.py):
//   dequantize  (:249-257)  v = fp32(code) * fp32(scale) + fp32(zero), narrowed, then cast RNE.
//               The product of a 4-bit code and an fp16 scale is exact in fp32, so one fused
//               multiply-add rounds exactly where the reference's multiply-then-add does.
//   quantize    (:190-221)  per group: lo = min, hi = max, scale = (hi - lo) / 15 computed in the
//               INPUT dtype (bf16 / fp16 arithmetic rounds after each op; an fp32 op rounded once
//               to the narrow type is that type's correctly rounded op, since fp32 carries more
//               than twice its significand bits plus two), scale = 1 where it is not
//               positive, code = clamp(rint((x - lo) / scale), 0, 15) in fp32 (rint = round half to
//               even, as torch.round), scale and lo stored as fp16; a ragged last group repeats the
//               row's last value (:160-187).
// Both are HBM-bound elementwise passes: 0.5625 B/value read + 2 B/value written (dequant to bf16).
#include "rw4_common.cuh"

namespace {

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}

// Fast path: K == padded K, K % 16 == 0, group % 16 == 0.  One thread expands 8 packed bytes
// (16 values, all inside one group) and writes them with vector stores.
template <typename OutT>
__global__ void __launch_bounds__(256)
    dequant_vec_kernel(const uint8_t* __restrict__ packed, const __half* __restrict__ scale,
                       const __half* __restrict__ zero, int64_t N, int64_t K, int group,
                       OutT* __restrict__ out) {
  const int64_t per_row = K / 16;
  const int64_t total = N * per_row;
  const int64_t groups = K / group;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = idx / per_row;
    const int64_t k0 = (idx - n * per_row) * 16;
    const uint2 w = ldg_stream_u2(packed + n * (K / 2) + k0 / 2);
    const int64_t gi = n * groups + k0 / group;
    const float s = __half2float(scale[gi]);
    const float z = __half2float(zero[gi]);
    OutT vals[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t word = (i < 4) ? w.x : w.y;
      const uint32_t byte = (word >> (8 * (i & 3))) & 0xFFu;
      vals[2 * i] = from_f32<OutT>(fmaf((float)(byte & 0xFu), s, z));
      vals[2 * i + 1] = from_f32<OutT>(fmaf((float)(byte >> 4), s, z));
    }
    OutT* dst = out + n * K + k0;
    constexpr int kVecs = (16 * sizeof(OutT)) / 16;
#pragma unroll
    for (int v = 0; v < kVecs; ++v) {
      reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(vals)[v];
    }
  }
}

// General path: any K (ragged tail narrowed away), any group dividing the padded K.
template <typename OutT>
__global__ void __launch_bounds__(256)
    dequant_any_kernel(const uint8_t* __restrict__ packed, const __half* __restrict__ scale,
                       const __half* __restrict__ zero, int64_t N, int64_t K, int64_t Kp,
                       int group, OutT* __restrict__ out) {
  const int64_t total = N * K;
  const int64_t groups = Kp / group;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = idx / K;
    const int64_t k = idx - n * K;
    const uint8_t byte = packed[n * (Kp / 2) + k / 2];
    const uint32_t code = (k & 1) ? (byte >> 4) : (byte & 0xF);
    const int64_t gi = n * groups + k / group;
    out[idx] = from_f32<OutT>(fmaf((float)code, __half2float(scale[gi]), __half2float(zero[gi])));
  }
}

template <typename InT>
__device__ __forceinline__ float load_f32(const InT* p);
template <>
__device__ __forceinline__ float load_f32<float>(const float* p) {
  return *p;
}
template <>
__device__ __forceinline__ float load_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <>
__device__ __forceinline__ float load_f32<__half>(const __half* p) {
  return __half2float(*p);
}

// One arithmetic result of the input dtype: fp32 as it is, bf16 / fp16 rounded to that type.
template <typename InT>
__device__ __forceinline__ float round_in(float v);
template <>
__device__ __forceinline__ float round_in<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float round_in<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
template <>
__device__ __forceinline__ float round_in<__half>(float v) {
  return __half2float(__float2half_rn(v));
}

// One warp per (row, group).  Each lane owns the code pairs (2l, 2l+1), (2l+64, 2l+65), ...
template <typename InT>
__global__ void __launch_bounds__(256)
    quantize_kernel(const InT* __restrict__ w, int64_t N, int64_t K, int group, int64_t groups,
                    uint8_t* __restrict__ packed, __half* __restrict__ scale,
                    __half* __restrict__ zero) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t total = N * groups;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t item = warp; item < total; item += nwarps) {
    const int64_t n = item / groups;
    const int64_t g = item - n * groups;
    const InT* row = w + n * K;
    const int64_t base = g * group;
    // min / max over the group (padding repeats the last value, so it never changes them).
    float lo = INFINITY, hi = -INFINITY;
    for (int i = lane; i < group; i += 32) {
      const int64_t k = base + i < K ? base + i : K - 1;
      const float v = load_f32<InT>(row + k);
      lo = fminf(lo, v);
      hi = fmaxf(hi, v);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, off));
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, off));
    }
    // tensor arithmetic in the input dtype: each op computed in fp32, rounded back to that type
    float s = round_in<InT>(__fdiv_rn(round_in<InT>(hi - lo), 15.0f));
    if (!(s > 0.0f)) s = 1.0f;
    for (int i = 2 * lane; i < group; i += 64) {
      uint32_t pair = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t k = base + i + h < K ? base + i + h : K - 1;
        const float v = load_f32<InT>(row + k);
        float c = rintf(__fdiv_rn(v - lo, s));
        c = fminf(fmaxf(c, 0.0f), 15.0f);
        pair |= ((uint32_t)c) << (4 * h);
      }
      packed[n * (groups * group / 2) + (base + i) / 2] = (uint8_t)pair;
    }
    if (lane == 0) {
      scale[item] = __float2half_rn(s);
      zero[item] = __float2half_rn(lo);
    }
  }
}

int grid_for(int64_t work_items, int threads) {
  int64_t blocks = (work_items + threads - 1) / threads;
  const int64_t cap = (int64_t)rw4::sm_count() * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

}  // namespace

extern "C" int rw4_dequant(const uint8_t* packed, const void* scale_f16, const void* zero_f16,
                           int64_t N, int64_t K, int32_t group, void* out, int32_t out_dtype,
                           void* stream) {
  using namespace rw4;
  if (N < 0 || K < 0) return fail(RW4_EINVAL, "rw4_dequant: negative shape N=%lld K=%lld",
                                  (long long)N, (long long)K);
  if (group < 2 || (group & 1)) return fail(RW4_EINVAL, "rw4_dequant: group %d must be even and >= 2", group);
  if (N == 0 || K == 0) return RW4_OK;
  if (!packed || !scale_f16 || !zero_f16 || !out) return fail(RW4_EINVAL, "rw4_dequant: null pointer");
  const int g = (int)(K < group ? K : group);
  if (g & 1) return fail(RW4_EINVAL, "rw4_dequant: effective group %d must be even", g);
  const int64_t Kp = (K + g - 1) / g * g;
  const size_t osz = out_dtype == RW4_F32 ? 4 : 2;
  if (out_dtype != RW4_F32 && out_dtype != RW4_BF16 && out_dtype != RW4_F16)
    return fail(RW4_EINVAL, "rw4_dequant: out_dtype %d", out_dtype);
  cudaStream_t s = as_stream(stream);
  const __half* sc = static_cast<const __half*>(scale_f16);
  const __half* zr = static_cast<const __half*>(zero_f16);
  const bool vec = (Kp == K) && (K % 16 == 0) && (g % 16 == 0) && aligned(packed, 8) &&
                   aligned(out, 16) && ((K * osz) % 16 == 0);
  if (vec) {
    const int blocks = grid_for(N * (K / 16), 256);
    switch (out_dtype) {
      case RW4_F32: dequant_vec_kernel<float><<<blocks, 256, 0, s>>>(packed, sc, zr, N, K, g, (float*)out); break;
      case RW4_BF16: dequant_vec_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(packed, sc, zr, N, K, g, (__nv_bfloat16*)out); break;
      default: dequant_vec_kernel<__half><<<blocks, 256, 0, s>>>(packed, sc, zr, N, K, g, (__half*)out); break;
    }
  } else {
    const int blocks = grid_for(N * K, 256);
    switch (out_dtype) {
      case RW4_F32: dequant_any_kernel<float><<<blocks, 256, 0, s>>>(packed, sc, zr, N, K, Kp, g, (float*)out); break;
      case RW4_BF16: dequant_any_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(packed, sc, zr, N, K, Kp, g, (__nv_bfloat16*)out); break;
      default: dequant_any_kernel<__half><<<blocks, 256, 0, s>>>(packed, sc, zr, N, K, Kp, g, (__half*)out); break;
    }
  }
  return launch_status("rw4_dequant launch");
}

extern "C" int rw4_quantize(const void* w, int32_t w_dtype, int64_t N, int64_t K, int32_t group,
                            uint8_t* packed, void* scale_f16, void* zero_f16, void* stream) {
  using namespace rw4;
  if (N < 0 || K < 0) return fail(RW4_EINVAL, "rw4_quantize: negative shape");
  if (group < 2 || (group & 1)) return fail(RW4_EINVAL, "rw4_quantize: group %d must be even and >= 2", group);
  if (N == 0 || K == 0) return RW4_OK;
  if (!w || !packed || !scale_f16 || !zero_f16) return fail(RW4_EINVAL, "rw4_quantize: null pointer");
  const int g = (int)(K < group ? K : group);
  if (g & 1) return fail(RW4_EINVAL, "rw4_quantize: effective group %d must be even", g);
  const int64_t groups = (K + g - 1) / g;
  const int blocks = grid_for(N * groups * 32, 256);
  cudaStream_t s = as_stream(stream);
  if (w_dtype == RW4_F32) {
    quantize_kernel<float><<<blocks, 256, 0, s>>>((const float*)w, N, K, g, groups, packed,
                                                  (__half*)scale_f16, (__half*)zero_f16);
  } else if (w_dtype == RW4_BF16) {
    quantize_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)w, N, K, g, groups,
                                                          packed, (__half*)scale_f16,
                                                          (__half*)zero_f16);
  } else if (w_dtype == RW4_F16) {
    quantize_kernel<__half><<<blocks, 256, 0, s>>>((const __half*)w, N, K, g, groups, packed,
                                                   (__half*)scale_f16, (__half*)zero_f16);
  } else {
    return fail(RW4_EINVAL, "rw4_quantize: w_dtype %d (want RW4_F32, RW4_BF16 or RW4_F16)",
                w_dtype);
  }
  return launch_status("rw4_quantize launch");
}
