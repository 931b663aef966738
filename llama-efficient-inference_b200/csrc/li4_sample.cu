// li4_sample.cu -- greedy next-token selection on the GPU, sm_100a.
//
// One CTA per row of logits: the index of the row's maximum, the first one on
// ties, a NaN counting as the maximum -- torch.argmax's answer (the
// reference's greedy step, bench.py:154-161 / llama/generation.py:59-60).
// Reading fp16 logits is exact: the reference's fp32 logits are the same
// values widened (llama/model.py:455).
#include "li4_common.cuh"
#include "li4_internal.h"

namespace li4 {

constexpr int kArgmaxThreads = 1024;

struct Best {
  float v;
  long long i;
};

// a before b in torch.argmax order: larger value, NaN above all, then smaller index.
__device__ __forceinline__ bool better(const Best& a, const Best& b) {
  const bool an = a.v != a.v, bn = b.v != b.v;
  if (an != bn) return an;
  if (!an && a.v != b.v) return a.v > b.v;
  return a.i < b.i;
}

__device__ __forceinline__ void take(Best& best, float v, long long i) {
  const Best c{v, i};
  if (better(c, best)) best = c;
}

template <bool F16>
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const void* logits, long long cols,
                                                                     long long stride, long long* out,
                                                                     long long out_stride) {
  __shared__ Best s_best[kArgmaxThreads / 32];
  const long long row = blockIdx.x;
  pdl_launch_dependents();
  pdl_wait_primary();  // the logits come from the preceding kernel
  Best best{-INFINITY, (long long)cols};  // loses to every real entry
  if constexpr (F16) {
    const __half* x = static_cast<const __half*>(logits) + row * stride;
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
    const long long nvec = vec ? cols / 8 : 0;
    for (long long c = threadIdx.x; c < nvec; c += kArgmaxThreads) {
      const uint4 u = reinterpret_cast<const uint4*>(x)[c];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
        take(best, f.x, 8 * c + 2 * e);
        take(best, f.y, 8 * c + 2 * e + 1);
      }
    }
    for (long long c = 8 * nvec + threadIdx.x; c < cols; c += kArgmaxThreads) take(best, __half2float(x[c]), c);
  } else {
    const float* x = static_cast<const float*>(logits) + row * stride;
    for (long long c = threadIdx.x; c < cols; c += kArgmaxThreads) take(best, x[c], c);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
    if (better(other, best)) best = other;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) s_best[warp] = best;
  __syncthreads();
  if (warp == 0) {
    best = s_best[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Best other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
      if (better(other, best)) best = other;
    }
    if (lane == 0) out[row * out_stride] = best.i;
  }
}

}  // namespace li4

extern "C" int li4_argmax_rows(const void* logits, int dtype, int64_t rows, int64_t cols, int64_t stride,
                               int64_t* out, int64_t out_stride, void* stream) {
  using namespace li4;
  if (dtype != LI4_F16 && dtype != LI4_F32)
    return set_error(LI4_ERR_UNSUPPORTED, "argmax_rows: dtype %d (LI4_F16 or LI4_F32)", dtype);
  if (rows < 0 || cols < 1 || stride < cols || !logits || !out || out_stride < 1)
    return set_error(LI4_ERR_INVALID_ARG, "argmax_rows: rows=%lld cols=%lld stride=%lld out_stride=%lld",
                     (long long)rows, (long long)cols, (long long)stride, (long long)out_stride);
  if ((reinterpret_cast<uintptr_t>(out) & 7u) || (reinterpret_cast<uintptr_t>(logits) & (dtype == LI4_F16 ? 1u : 3u)))
    return set_error(LI4_ERR_ALIGNMENT, "argmax_rows: misaligned logits or output");
  if (rows == 0) return LI4_OK;
  if (rows > 65535) return set_error(LI4_ERR_UNSUPPORTED, "argmax_rows: rows=%lld above 65535", (long long)rows);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)rows, 1, 1);
  cfg.blockDim = dim3(kArgmaxThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  long long* o = reinterpret_cast<long long*>(out);
  const int rc = dtype == LI4_F16
                     ? check_cuda(cudaLaunchKernelEx(&cfg, argmax_rows_kernel<true>, logits, (long long)cols,
                                                     (long long)stride, o, (long long)out_stride),
                                  "argmax_rows: kernel launch")
                     : check_cuda(cudaLaunchKernelEx(&cfg, argmax_rows_kernel<false>, logits, (long long)cols,
                                                     (long long)stride, o, (long long)out_stride),
                                  "argmax_rows: kernel launch");
  if (rc == LI4_OK) clear_error();
  return rc;
}
