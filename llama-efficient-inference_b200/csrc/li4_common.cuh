// li4_common.cuh -- device helpers shared by the INT4 kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace li4 {

// ---------------------------------------------------------------------------
// Nibble unpack.
//
// One 32-bit word of a packed row holds 8 consecutive k values q0..q7
// (byte j = q[2j] | q[2j+1] << 4, so nibble i sits at bits 4i..4i+3; the
// layout of llama/quantize.py:73).  The unpack uses the fp16 "magic number"
// construction published for INT4 GEMMs (Kim et al. 2022, "Who Says Elephants
// Can't Run"; Frantar et al. 2024, "MARLIN"): OR-ing a nibble into the
// mantissa of 1024.0 (0x6400) gives the exact fp16 value 1024 + q (or
// 1024 + 16 q when the nibble lands on mantissa bits 4..7).  Subtracting
// 1024 + zero (resp. FMA with 1/16 and -(64 + zero)) then yields q - zero
// exactly: every intermediate is a small integer representable in fp16.
//
// Result: four half2 registers holding (q_i - z, q_{i+4} - z), i = 0..3.
// Callers must pair them with x values in the same (i, i+4) order.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t magic) {
  uint32_t r;
  // (a & mask) | magic ; LUT = (0xF0 & 0xCC) | 0xAA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(magic));
  return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Per-row constants for the exact (q - z) unpack.
struct ZeroConsts {
  __half2 lo;   // (1024 + z, 1024 + z)
  __half2 hi;   // (-(64 + z), -(64 + z))
};

__device__ __forceinline__ ZeroConsts make_zero_consts(__half z) {
  ZeroConsts c;
  const __half zl = __hadd(z, __ushort_as_half(0x6400));      // 1024 + z (exact for z in 0..15)
  const __half zh = __hneg(__hadd(z, __ushort_as_half(0x5400)));  // -(64 + z)
  c.lo = __halves2half2(zl, zl);
  c.hi = __halves2half2(zh, zh);
  return c;
}

// q - z for the 8 nibbles of w, exact in fp16.
//   p[0] = (q0 - z, q4 - z), p[1] = (q1 - z, q5 - z),
//   p[2] = (q2 - z, q6 - z), p[3] = (q3 - z, q7 - z)
__device__ __forceinline__ void unpack8_qz(uint32_t w, const ZeroConsts& zc, __half2 p[4]) {
  constexpr uint32_t MAGIC = 0x64006400u;  // half2(1024, 1024)
  const __half2 inv16 = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));  // 1/16
  const uint32_t w8 = w >> 8;
  const uint32_t lo0 = lop3_and_or(w, 0x000F000Fu, MAGIC);   // 1024 + q0 | 1024 + q4
  const uint32_t hi0 = lop3_and_or(w, 0x00F000F0u, MAGIC);   // 1024 + 16 q1 | 1024 + 16 q5
  const uint32_t lo1 = lop3_and_or(w8, 0x000F000Fu, MAGIC);  // 1024 + q2 | 1024 + q6
  const uint32_t hi1 = lop3_and_or(w8, 0x00F000F0u, MAGIC);  // 1024 + 16 q3 | 1024 + 16 q7
  p[0] = __hsub2(u32_as_h2(lo0), zc.lo);
  p[1] = __hfma2(u32_as_h2(hi0), inv16, zc.hi);
  p[2] = __hsub2(u32_as_h2(lo1), zc.lo);
  p[3] = __hfma2(u32_as_h2(hi1), inv16, zc.hi);
}

// Position (0..7) inside the word of element e (0..7) of the p[] output:
// p[i].x -> nibble i, p[i].y -> nibble i + 4.
__host__ __device__ __forceinline__ int unpack_pos(int i, int hi) { return i + 4 * hi; }

// ---------------------------------------------------------------------------
// Tensor-core tile: D[16x8] += A[16x16] * B[16x8], fp16 inputs, fp32 accum.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// acc += a.x * b.x + a.y * b.y with fp16 operands and an fp32 accumulator
// (sm_100 mixed-precision FMA: the product is formed exactly, one rounding).
__device__ __forceinline__ float fma2_f16_f32(uint32_t a, uint32_t b, float acc) {
  asm("{\n\t.reg .f16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %1;\n\t"
      "mov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
      "fma.rn.f32.f16 %0, ah, bh, %0;\n\t}"
      : "+f"(acc) : "r"(a), "r"(b));
  return acc;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait_primary() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Global loads.
// ---------------------------------------------------------------------------
// Streaming 16-byte load of weight bytes: read once per launch, so do not
// allocate in L1.
// L2 policy for weight bytes: every weight byte is read once per decode step, so it goes first
// when L2 needs room -- the KV cache and the activations that the step's latency-bound loads
// read stay resident instead of being pushed out by the weight stream.
__device__ __forceinline__ uint64_t weight_l2_policy() {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// (The register-ring kernels load weights without the policy: with it their 113-GEMV step
// measured no gain -- 1495 against 1549 GB/s in one run.)  The L2::256B hint has each 16-byte load
// fetch its aligned 256-byte block into L2, i.e. the next three ksteps of the same weight row
// that the ring requests next: lm_head at M = 1 33.3 against 34.8 us (L2::128B: no change).
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ __half ldg_half(const __half* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return __ushort_as_half(r);
}

}  // namespace li4
