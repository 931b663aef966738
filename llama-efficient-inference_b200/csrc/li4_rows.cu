// li4_rows.cu -- the register-rows GEMV kernel (sm_100a), for M = 1 and K <= 2048.
//
// A warp owns two output rows (r, r + 8 of a 16-row tile) and all of K: lane l holds bytes
// [l*K/64, (l+1)*K/64) of both packed rows, so a warp's loads cover each row contiguously.
// Before the dependency wait the warp loads its rows, their group scale and zero (a lane's
// K/32 k values lie in one group of 128), and unpacks them into exact fp16 (q - zero) pairs
// held in registers (64 registers at K = 2048): all of the weight work overlaps the preceding
// kernel.  After the wait each lane reads its K/32 values of x straight from global memory,
// forms sum (q - z) * x with fp16 x fp16 -> fp32 FMAs (exact products), scales by the group
// scale in fp32, and the 32 lanes reduce by shuffles in a fixed order.  There is no shared
// memory, no mbarrier and no cross-warp reduction on the launch chain, which after the wait is
// one L2 round trip for x, the FMAs, five shuffle steps and the stores.
//
// A CTA (8 warps) is one 16-row tile, so the fused epilogues that pair rows j and j + 8 of a
// tile (SwiGLU, QKV + RoPE) find both rows in one warp, and the per-tile sum of squares for the
// next RMSNorm (li4_fusion.sumsq_out) is a fixed-order sum over the CTA's 16 rows.
#include "li4_common.cuh"
#include "li4_gemv_device.cuh"
#include "li4_internal.h"

#include <mutex>
#include <vector>

namespace li4 {

constexpr int kRowsWarps = 8;
constexpr int kRowsThreads = kRowsWarps * 32;

// acc += w.lo * x.lo + w.hi * x.hi for fp16 pairs, fp32 accumulation (products exact).
__device__ __forceinline__ float dot2_acc(uint32_t w, uint32_t x, float acc) {
  asm("{\n\t.reg .f16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %1;\n\t"
      "mov.b32 {xl, xh}, %2;\n\t"
      "fma.rn.f32.f16 %0, wl, xl, %0;\n\t"
      "fma.rn.f32.f16 %0, wh, xh, %0;\n\t}"
      : "+f"(acc)
      : "r"(w), "r"(x));
  return acc;
}

// x pairs in the unpack's (k, k + 4) order from 8 consecutive fp16 values (4 words).
__device__ __forceinline__ void x_pairs(const uint4& v, uint32_t p[4]) {
  p[0] = __byte_perm(v.x, v.z, 0x5410);  // (x0, x4)
  p[1] = __byte_perm(v.x, v.z, 0x7632);  // (x1, x5)
  p[2] = __byte_perm(v.y, v.w, 0x5410);  // (x2, x6)
  p[3] = __byte_perm(v.y, v.w, 0x7632);  // (x3, x7)
}

// One output of row `row` through the epilogue, the residual value already loaded; returns the
// value written (as emit_one, li4_gemv_device.cuh).
__device__ __forceinline__ float rows_emit(const GemvArgs& a, int row, float v, float rv) {
  __half h = __float2half_rn(v);
  if (a.epi == LI4_EPI_STORE_F32) {  // fp16 Linear output widened (llama/model.py:455)
    reinterpret_cast<float*>(a.y)[row] = __half2float(h);
    return __half2float(h);
  }
  if (a.epi == LI4_EPI_RESIDUAL) h = __float2half_rn(__half2float(h) + rv);  // x + wo(...) (llama/model.py:358-362)
  a.y[row] = h;
  return __half2float(h);
}

// KW: packed bytes of one row per lane (K / 64): 16 (K = 1024) or 32 (K = 2048).
template <int KW, bool FUSED>
__global__ void __launch_bounds__(kRowsThreads, 2) gemv_rows_kernel(const __grid_constant__ GemvArgs a) {
  constexpr int WORDS = KW / 4;  // packed 32-bit words per row per lane (8 k each)
  constexpr int KL = KW * 2;     // k values per lane
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int r_lo = tile * 16 + warp, r_hi = r_lo + 8;
  const int rl = min(r_lo, a.N - 1), rh = min(r_hi, a.N - 1);  // rows past N repeat row N-1 (not written)
  __shared__ float s_sq[16];

  pdl_launch_dependents();
  // ---- weights (never written by the preceding kernel): load and unpack before the wait
  uint32_t wq[2][WORDS];
  {
    const uint4* plo = reinterpret_cast<const uint4*>(a.packed + (long long)rl * a.spn + lane * KW);
    const uint4* phi = reinterpret_cast<const uint4*>(a.packed + (long long)rh * a.spn + lane * KW);
#pragma unroll
    for (int j = 0; j < KW / 16; ++j) {
      const uint4 l = ldg_stream_v4(plo + j), h = ldg_stream_v4(phi + j);
      wq[0][4 * j + 0] = l.x; wq[0][4 * j + 1] = l.y; wq[0][4 * j + 2] = l.z; wq[0][4 * j + 3] = l.w;
      wq[1][4 * j + 0] = h.x; wq[1][4 * j + 1] = h.y; wq[1][4 * j + 2] = h.z; wq[1][4 * j + 3] = h.w;
    }
  }
  const int g = (lane * KL) >> 7;  // the lane's group (K/32 k values, inside one group of 128)
  const unsigned short* sc = reinterpret_cast<const unsigned short*>(a.scale);
  const unsigned short* ze = reinterpret_cast<const unsigned short*>(a.zero);
  const float s_lo0 = __half2float(__ushort_as_half(__ldg(sc + (long long)rl * a.ssn + g)));
  const float s_hi0 = __half2float(__ushort_as_half(__ldg(sc + (long long)rh * a.ssn + g)));
  const ZeroConsts z_lo = make_zero_consts(__ushort_as_half(__ldg(ze + (long long)rl * a.ssn + g)));
  const ZeroConsts z_hi = make_zero_consts(__ushort_as_half(__ldg(ze + (long long)rh * a.ssn + g)));
  uint32_t w16[2][WORDS * 4];  // (q_i - z, q_{i+4} - z) pairs, word j -> entries 4j .. 4j+3
#pragma unroll
  for (int j = 0; j < WORDS; ++j) {
    __half2 p[4];
    unpack8_qz(wq[0][j], z_lo, p);
#pragma unroll
    for (int i = 0; i < 4; ++i) w16[0][4 * j + i] = h2_as_u32(p[i]);
    unpack8_qz(wq[1][j], z_hi, p);
#pragma unroll
    for (int i = 0; i < 4; ++i) w16[1][4 * j + i] = h2_as_u32(p[i]);
  }

  // Keep the unpack above the dependency wait: the compiler would otherwise sink it below the
  // wait (fewer live registers), back onto the launch chain.  A branch on every unpacked word,
  // taken only when N < 1 (never: the host checks N >= 1), must be evaluated before the wait.
  uint32_t fold = __float_as_uint(s_lo0) ^ __float_as_uint(s_hi0);
#pragma unroll
  for (int i = 0; i < WORDS * 4; ++i) fold ^= w16[0][i] ^ w16[1][i];
  if (a.N < 1 && fold == 0u) atomicOr(&g_li4_device_error, 0u);
  const float s_lo = s_lo0, s_hi = s_hi0;

  pdl_wait_primary();  // x (and the residual) come from the preceding kernel
  // ---- x: the lane's KL values, loaded together (one L2 round trip)
  uint4 xv[WORDS];  // one 16-byte piece of x (8 k) per packed word
  const uint4* xp = reinterpret_cast<const uint4*>(a.x + lane * KL);
#pragma unroll
  for (int j = 0; j < WORDS; ++j) xv[j] = xp[j];
  float res_lo = 0.f, res_hi = 0.f;
  if (FUSED && a.epi == LI4_EPI_RESIDUAL && lane == 0) {
    if (r_lo < a.N) res_lo = __half2float(a.res[r_lo]);
    if (r_hi < a.N) res_hi = __half2float(a.res[r_hi]);
  }
  float acc_lo = 0.f, acc_hi = 0.f;
#pragma unroll
  for (int j = 0; j < WORDS; ++j) {
    uint32_t xp4[4];
    x_pairs(xv[j], xp4);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc_lo = dot2_acc(w16[0][4 * j + i], xp4[i], acc_lo);
      acc_hi = dot2_acc(w16[1][4 * j + i], xp4[i], acc_hi);
    }
  }
  acc_lo *= s_lo;
  acc_hi *= s_hi;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc_lo += __shfl_xor_sync(0xffffffffu, acc_lo, o);
    acc_hi += __shfl_xor_sync(0xffffffffu, acc_hi, o);
  }

  // ---- epilogue (lane 0 of each warp: rows r_lo, r_hi)
  float sq = 0.f;  // squares of the written values (sumsq_out)
  if (lane == 0) {
    if (FUSED && epi_paired(a)) {  // N % 16 == 0: both rows exist
      emit_pair(a, 0, tile * 8 + warp, acc_lo, acc_hi);
    } else if (FUSED) {
      if (r_lo < a.N) {
        const float h = rows_emit(a, r_lo, acc_lo, res_lo);
        sq += h * h;
      }
      if (r_hi < a.N) {
        const float h = rows_emit(a, r_hi, acc_hi, res_hi);
        sq += h * h;
      }
    } else {
      if (r_lo < a.N) a.y[r_lo] = __float2half_rn(acc_lo);
      if (r_hi < a.N) a.y[r_hi] = __float2half_rn(acc_hi);
    }
  }
  if (FUSED && a.ssq_out != nullptr) {  // the tile's sum of squares, rows in warp order
    if (lane == 0) s_sq[warp] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kRowsWarps; ++w) t += s_sq[w];
      a.ssq_out[tile] = t;
    }
  }
}

int launch_rows(const GemvArgs& a, bool fused, cudaStream_t stream) {
  const int kw = a.K / 64;
  auto kernel = kw == 32 ? (fused ? gemv_rows_kernel<32, true> : gemv_rows_kernel<32, false>)
                         : (fused ? gemv_rows_kernel<16, true> : gemv_rows_kernel<16, false>);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.N + 15) / 16), 1, 1);
  cfg.blockDim = dim3(kRowsThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, a), "int4_linear: register-rows kernel launch");
}

int rows_device_errors(unsigned* flags, bool reset) { return tu_device_errors(flags, reset); }

}  // namespace li4
