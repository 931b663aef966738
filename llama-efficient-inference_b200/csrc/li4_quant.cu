// li4_quant.cu -- INT4 format producer (quantize) and exact unpack (dequantize), sm_100a.
//
// Both kernels restate the reference's fp32 arithmetic operation by operation
// with IEEE round-to-nearest intrinsics, so their outputs are bit-identical
// to llama/quantize.py:44-75 (quantize_tensor) and :78-104
// (dequantize_packed).  They are bandwidth-bound; neither is on the decode
// hot loop (quantize runs once per weight, dequantize feeds the M > 16
// prefill GEMM).
#include "li4_common.cuh"
#include "li4_internal.h"

namespace li4 {

// torch.clamp(v, 0, 15): NaN and -0.0 pass through unchanged.
__device__ __forceinline__ float clamp_0_15(float v) {
  if (v < 0.f) v = 0.f;
  if (v > 15.f) v = 15.f;
  return v;
}

// Reference dequantization of one value: fp32 (q - zero) * scale -> fp16
// (llama/quantize.py:101-104).
__device__ __forceinline__ __half dequant_one(uint32_t q, float z, float s) {
  return __float2half_rn(__fmul_rn(__fsub_rn((float)q, z), s));
}

// One thread per 16 packed bytes (32 k values) of a row.
__global__ void dequant_vec_kernel(const uint8_t* __restrict__ packed, const __half* __restrict__ scale,
                                   const __half* __restrict__ zero, __half* __restrict__ w16, int N, int K,
                                   int group, long long spn, long long ssn, long long swn) {
  const int chunks = K / 32;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)N * chunks) return;
  const int n = (int)(idx / chunks);
  const int c = (int)(idx - (long long)n * chunks);
  const uint4 v = *reinterpret_cast<const uint4*>(packed + n * spn + c * 16);
  const uint32_t words[4] = {v.x, v.y, v.z, v.w};
  const int k0 = c * 32;
  __half* out = w16 + n * swn + k0;
  const __half* srow = scale + n * ssn;
  const __half* zrow = zero + n * ssn;
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {  // byte e of the word -> k = k0 + 8*wi + 2e, +1
      const uint32_t byte = (words[wi] >> (8 * e)) & 0xFFu;
      const int k = k0 + 8 * wi + 2 * e;
      const int g = k / group;  // group is even, so k and k+1 share it
      const float z = __half2float(zrow[g]);
      const float s = __half2float(srow[g]);
      const __half lo = dequant_one(byte & 0xFu, z, s);
      const __half hi = dequant_one(byte >> 4, z, s);
      o[e] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
    }
    *reinterpret_cast<uint4*>(out + 8 * wi) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Any shape / alignment: one thread per output value.
__global__ void dequant_scalar_kernel(const uint8_t* __restrict__ packed, const __half* __restrict__ scale,
                                      const __half* __restrict__ zero, __half* __restrict__ w16, int N, int K,
                                      int group, long long spn, long long ssn, long long swn) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)N * K) return;
  const int n = (int)(idx / K);
  const int k = (int)(idx - (long long)n * K);
  const uint32_t byte = packed[n * spn + k / 2];
  const uint32_t q = (k & 1) ? (byte >> 4) : (byte & 0xFu);
  const int g = k / group;
  w16[n * swn + k] = dequant_one(q, __half2float(zero[n * ssn + g]), __half2float(scale[n * ssn + g]));
}

template <typename T>
__device__ __forceinline__ float load_as_float(const T* p);
template <>
__device__ __forceinline__ float load_as_float<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float load_as_float<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float load_as_float<float>(const float* p) { return *p; }

// min/max that propagate NaN like torch.amin / torch.amax.
__device__ __forceinline__ float nan_min(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  return b < a ? b : a;
}
__device__ __forceinline__ float nan_max(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  return b > a ? b : a;
}

// One warp per (row, group): llama/quantize.py:62-75 operation by operation.
template <typename T>
__global__ void quantize_kernel(const T* __restrict__ w, uint8_t* __restrict__ packed, __half* __restrict__ scale,
                                __half* __restrict__ zero, int N, int K, int group, long long swn) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int n_groups = K / group;
  if (warp_id >= (long long)N * n_groups) return;
  const int n = (int)(warp_id / n_groups);
  const int g = (int)(warp_id - (long long)n * n_groups);
  const T* src = w + n * swn + (long long)g * group;

  float mn = INFINITY, mx = -INFINITY;
  for (int e = lane; e < group; e += 32) {
    const float v = load_as_float<T>(src + e);
    mn = nan_min(mn, v);
    mx = nan_max(mx, v);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float omn = __shfl_xor_sync(0xffffffffu, mn, off);
    const float omx = __shfl_xor_sync(0xffffffffu, mx, off);
    mn = nan_min(mn, omn);
    mx = nan_max(mx, omx);
  }
  // scale = (max - min) / 15 ; scale == 0 -> 1   (llama/quantize.py:67-68)
  float s = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
  if (s == 0.f) s = 1.0f;
  // zero_point = round(-min / scale).clamp(0, 15)   (llama/quantize.py:69)
  const float zp = clamp_0_15(rintf(__fdiv_rn(-mn, s)));
  // q = round(w / scale + zero_point).clamp(0, 15) ; pack even | odd << 4   (:71-73)
  uint8_t* dst = packed + (long long)n * (K / 2) + (long long)g * (group / 2);
  for (int j = lane; j < group / 2; j += 32) {
    const float v0 = load_as_float<T>(src + 2 * j);
    const float v1 = load_as_float<T>(src + 2 * j + 1);
    const float q0 = clamp_0_15(rintf(__fadd_rn(__fdiv_rn(v0, s), zp)));
    const float q1 = clamp_0_15(rintf(__fadd_rn(__fdiv_rn(v1, s), zp)));
    dst[j] = (uint8_t)((uint32_t)q0 | ((uint32_t)q1 << 4));
  }
  if (lane == 0) {  // scale.half(), zero_point.half()   (:75)
    scale[(long long)n * n_groups + g] = __float2half_rn(s);
    zero[(long long)n * n_groups + g] = __float2half_rn(zp);
  }
}

}  // namespace li4

extern "C" int li4_dequantize(const void* packed, const void* scale, const void* zero, void* w16, int64_t N,
                              int64_t K, int64_t group_size, int64_t stride_pn, int64_t stride_sn, int64_t stride_wn,
                              void* stream) {
  using namespace li4;
  if (N < 0 || K < 0 || group_size < 2 || group_size % 2 != 0 || (K > 0 && K % group_size != 0))
    return set_error(LI4_ERR_INVALID_ARG, "dequantize: N=%lld K=%lld group_size=%lld (need K %% group == 0, even group)",
                     (long long)N, (long long)K, (long long)group_size);
  if (N == 0 || K == 0) { clear_error(); return LI4_OK; }
  if (!packed || !scale || !zero || !w16) return set_error(LI4_ERR_INVALID_ARG, "dequantize: null tensor pointer");
  if (stride_pn < K / 2 || stride_sn < K / group_size || stride_wn < K)
    return set_error(LI4_ERR_INVALID_ARG, "dequantize: row strides smaller than the rows");
  if ((int64_t)N * K > (int64_t(1) << 40)) return set_error(LI4_ERR_INVALID_ARG, "dequantize: tensor too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = (K % 32 == 0) && aligned16(packed) && stride_pn % 16 == 0 && aligned16(w16) && stride_wn % 8 == 0;
  const int threads = 256;
  if (vec) {
    const long long items = N * (K / 32);
    dequant_vec_kernel<<<(unsigned)((items + threads - 1) / threads), threads, 0, s>>>(
        static_cast<const uint8_t*>(packed), static_cast<const __half*>(scale), static_cast<const __half*>(zero),
        static_cast<__half*>(w16), (int)N, (int)K, (int)group_size, stride_pn, stride_sn, stride_wn);
  } else {
    const long long items = N * K;
    dequant_scalar_kernel<<<(unsigned)((items + threads - 1) / threads), threads, 0, s>>>(
        static_cast<const uint8_t*>(packed), static_cast<const __half*>(scale), static_cast<const __half*>(zero),
        static_cast<__half*>(w16), (int)N, (int)K, (int)group_size, stride_pn, stride_sn, stride_wn);
  }
  const int rc = check_cuda(cudaGetLastError(), "dequantize: kernel launch");
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_quantize(const void* w, int w_dtype, void* packed, void* scale, void* zero, int64_t N, int64_t K,
                            int64_t group_size, int64_t stride_wn, void* stream) {
  using namespace li4;
  if (N < 0 || K < 0 || group_size < 2 || group_size % 2 != 0 || (K > 0 && K % group_size != 0))
    return set_error(LI4_ERR_INVALID_ARG, "quantize: N=%lld K=%lld group_size=%lld (need K %% group == 0, even group)",
                     (long long)N, (long long)K, (long long)group_size);
  if (N == 0 || K == 0) { clear_error(); return LI4_OK; }
  if (!w || !packed || !scale || !zero) return set_error(LI4_ERR_INVALID_ARG, "quantize: null tensor pointer");
  if (stride_wn < K) return set_error(LI4_ERR_INVALID_ARG, "quantize: row stride smaller than the row");
  if ((int64_t)N * K > (int64_t(1) << 40)) return set_error(LI4_ERR_INVALID_ARG, "quantize: tensor too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long warps = N * (K / group_size);
  const int threads = 256;
  const unsigned blocks = (unsigned)((warps * 32 + threads - 1) / threads);
  uint8_t* pk = static_cast<uint8_t*>(packed);
  __half* sc = static_cast<__half*>(scale);
  __half* zp = static_cast<__half*>(zero);
  switch (w_dtype) {
    case LI4_F16:
      quantize_kernel<__half><<<blocks, threads, 0, s>>>(static_cast<const __half*>(w), pk, sc, zp, (int)N, (int)K,
                                                          (int)group_size, stride_wn);
      break;
    case LI4_BF16:
      quantize_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(static_cast<const __nv_bfloat16*>(w), pk, sc, zp,
                                                                 (int)N, (int)K, (int)group_size, stride_wn);
      break;
    case LI4_F32:
      quantize_kernel<float><<<blocks, threads, 0, s>>>(static_cast<const float*>(w), pk, sc, zp, (int)N, (int)K,
                                                         (int)group_size, stride_wn);
      break;
    default:
      return set_error(LI4_ERR_INVALID_ARG, "quantize: unknown dtype %d", w_dtype);
  }
  const int rc = check_cuda(cudaGetLastError(), "quantize: kernel launch");
  if (rc == LI4_OK) clear_error();
  return rc;
}
