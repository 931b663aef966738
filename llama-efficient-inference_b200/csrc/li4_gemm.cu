// li4_gemm.cu -- INT4 (group 128) x fp16 GEMM on the 5th-generation tensor cores (tcgen05), sm_100a.
//
// y[M, N] = x[M, K] @ W[N, K]^T for M > 16 (prefill), W in the packed INT4 format of
// llama/quantize.py:44-75.  This replaces the reference's prefill path, dequantize_packed (v1/v2/v3,
// llama/quantize.py:78-126, 143-146) + F.linear: the fp16 weights are rebuilt tile by tile in
// shared memory, bit-identical to the reference's fp16((q - zero) * scale), and never reach HBM.
//
// One CTA computes a tile of 128 output features x BT tokens (BT = 128 for prefill, 16 / 32 / 64
// for short batches), looping over K in steps of 64:
//   * A operand = the W tile [128 features x 64 k] fp16, K-major, 128-byte swizzle, written by 8
//     dequant warps: every thread loads 16 packed bytes (32 k of one feature row) four steps ahead
//     into registers, and in its step unpacks them (the fp16 magic-number construction: exact
//     q - zero), multiplies by the group scale in fp16 (the exact product rounded once: the
//     reference's rounding), puts the k values back in order, stores four 16-byte chunks at their
//     swizzled positions and arrives on the stage's "W full" mbarrier.
//   * B operand = the x tile [BT tokens x 64 k] fp16, K-major, 128-byte swizzle, copied by 2 warps
//     with cp.async three steps ahead (rows past M are zero-filled); "x full" mbarrier.
//   * One thread of the MMA warp waits for both, issues the step's four tcgen05.mma (M = 128,
//     N = BT, K = 16, fp32 accumulation in tensor memory) and commits them to the stage's "empty"
//     mbarrier, which the producers wait for before refilling the stage.  No CTA-wide barrier
//     inside the K loop.
//   * Epilogue: tcgen05.ld of the accumulator (TMEM lane = feature, column = token), fp16
//     rounding, stores of consecutive features per token.
// Every mbarrier wait is bounded: one that runs out sets bit 4 of li4_device_errors, waits
// (bounded) for the CTA's own MMAs, frees the tensor memory and returns.
#include "li4_common.cuh"
#include "li4_gemv_device.cuh"
#include "li4_internal.h"

#include <mutex>
#include <vector>

namespace li4 {

constexpr int kGemmBK = 64;       // k per step: one 128-byte swizzle row of fp16
constexpr int kGemmStages = 4;    // shared-memory stages
constexpr int kGemmAhead = 3;     // x tiles in flight ahead of the one being consumed
constexpr unsigned kGemmWaitLimit = 1u << 24;  // mbarrier polls before giving up

__device__ unsigned g_gemm_device_error;  // bit 4 of li4_device_errors

int gemm_device_errors(unsigned* flags, bool reset) {
  int rc = check_cuda(cudaMemcpyFromSymbol(flags, g_gemm_device_error, sizeof(unsigned)), "device_errors: gemm");
  if (rc == LI4_OK && reset) {
    const unsigned zero = 0;
    rc = check_cuda(cudaMemcpyToSymbol(g_gemm_device_error, &zero, sizeof(unsigned)), "device_errors: clearing");
  }
  return rc;
}

struct GemmArgs {
  const __half* x;
  const uint8_t* packed;
  const __half* scale;
  const __half* zero;
  __half* y;
  int M, N, K;
  long long sxm, spn, ssn, sym;
};

// ---- tcgen05 / shared-memory descriptors (sm_100 UMMA formats)
// Shared-memory matrix descriptor, K-major operand, 128-byte swizzle: start address >> 4 (bits 0-13),
// leading byte offset 16 B (ignored for swizzled K-major; encoded 1, bits 16-29), stride byte
// offset 1024 B between 8-row groups (bits 32-45), version 1 (bits 46-47), swizzle mode 2 =
// 128-byte (bits 61-63).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_byte_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_byte_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and B fp16 (bits 7-9, 10-12
// = 0), both K-major (bits 15, 16 = 0), N >> 3 (bits 17-22), M >> 4 (bits 24-28).
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      :
      : "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ bool gemm_wait(uint64_t* bar, unsigned parity) {
  for (unsigned i = 0; i < kGemmWaitLimit; ++i)
    if (mbar_test_wait(bar, parity)) return true;
  atomicOr(&g_gemm_device_error, 16u);
  return false;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 32 consecutive k of one feature row (16 packed bytes) -> fp16((q - z) * s) in k order, 4 x 16 B.
__device__ __forceinline__ void dequant32(const uint4& w, __half z, __half s, uint4 out[4]) {
  const ZeroConsts zc = make_zero_consts(z);
  const __half2 s2 = __halves2half2(s, s);
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __half2 p[4];
    unpack8_qz(ws[j], zc, p);  // p[i] = (q_i - z, q_{i+4} - z), exact
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __hmul2(p[i], s2);  // one rounding of the exact product
    const uint32_t a = h2_as_u32(p[0]), b = h2_as_u32(p[1]), c = h2_as_u32(p[2]), d = h2_as_u32(p[3]);
    out[j] = make_uint4(__byte_perm(a, b, 0x5410),   // (k0, k1)
                        __byte_perm(c, d, 0x5410),   // (k2, k3)
                        __byte_perm(a, b, 0x7632),   // (k4, k5)
                        __byte_perm(c, d, 0x7632));  // (k6, k7)
  }
}

// Warp roles of int4_gemm_kernel: 8 W warps (half a feature row's 64 k per thread), 2 x warps
// (cp.async), 1 MMA warp (one thread issues the tensor-core work).
constexpr int kGemmWWarps = 8, kGemmXWarps = 2;
constexpr int kGemmWAhead = 4;  // steps of packed W in flight per thread (registers)
constexpr int kGemmMmaWarp = kGemmWWarps + kGemmXWarps;
constexpr int kGemmWSThreads = (kGemmMmaWarp + 1) * 32;

template <int BT>
__global__ void __launch_bounds__(kGemmWSThreads, 1) int4_gemm_kernel(const __grid_constant__ GemmArgs a) {
  constexpr int A_BYTES = 128 * 128;                 // W tile: 128 features x 64 k fp16
  constexpr int B_BYTES = BT * 128;                  // x tile: BT tokens x 64 k fp16
  constexpr int STAGE = A_BYTES + B_BYTES;           // multiple of 1024 (BT % 8 == 0)
  constexpr int TMEM_COLS = BT < 32 ? 32 : BT;       // power of two >= 32
  constexpr int S = kGemmStages;
  constexpr int XA = kGemmAhead;                     // steps the x warps run ahead of their arrivals
  static_assert(XA < S, "the x warps may run at most S - 1 steps ahead of the MMAs");
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzle atoms are 1024 bytes: the stages start on a 1024-byte boundary
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_w = reinterpret_cast<uint64_t*>(smem + S * STAGE);  // W tile of the stage written (128 arrivals)
  uint64_t* full_x = full_w + S;                                     // x tile landed (64 arrivals)
  uint64_t* empty = full_x + S;                                      // the stage's MMAs have read it (commit)
  uint64_t* done = empty + S;                                        // every MMA of the CTA has finished (commit)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * 128, m0 = blockIdx.y * BT;
  const int nk = a.K / kGemmBK;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_holder)),
                 "n"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_w[s], kGemmWWarps * 32);
      mbar_init(&full_x[s], kGemmXWarps * 32);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;
  bool ok = true;

  if (warp < kGemmWWarps) {
    // ---- W: threads 2r, 2r + 1 dequantize k halves 0 / 1 (32 k, 16 packed bytes) of feature row r
    const int r = tid >> 1, h = tid & 1;
    const int row = min(n0 + r, a.N - 1);  // rows past N repeat row N-1 (their outputs are not stored)
    const uint8_t* wsrc = a.packed + (long long)row * a.spn + h * 16;
    const unsigned short* ssrc = reinterpret_cast<const unsigned short*>(a.scale) + (long long)row * a.ssn;
    const unsigned short* zsrc = reinterpret_cast<const unsigned short*>(a.zero) + (long long)row * a.ssn;
    static_assert(kGemmWAhead == 4, "the W register ring below holds this step and the next four");
    uint4 w0 = {}, w1 = {}, w2 = {}, w3 = {}, w4 = {};  // packed bytes of steps t .. t + 4
    if (nk > 0) w0 = ldg_stream_v4(wsrc);
    if (nk > 1) w1 = ldg_stream_v4(wsrc + 32);
    if (nk > 2) w2 = ldg_stream_v4(wsrc + 64);
    if (nk > 3) w3 = ldg_stream_v4(wsrc + 96);
    for (int step = 0; step < nk; ++step) {
      const int s = step % S;
      if (step + kGemmWAhead < nk) w4 = ldg_stream_v4(wsrc + (long long)(step + kGemmWAhead) * 32);
      const int g = (step * kGemmBK) >> 7;
      const __half sc = __ushort_as_half(__ldg(ssrc + g)), ze = __ushort_as_half(__ldg(zsrc + g));
      if (step >= S && ok) ok = gemm_wait(&empty[s], ((step / S) - 1) & 1);
      uint4 q[4];
      dequant32(w0, ze, sc, q);
      w0 = w1;
      w1 = w2;
      w2 = w3;
      w3 = w4;
      uint8_t* at = smem + s * STAGE + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(at + (((h * 4 + c) ^ (r & 7)) << 4)) = q[c];
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy stores -> the tensor core
      mbar_arrive(&full_w[s]);
    }
  } else if (warp < kGemmMmaWarp) {
    // ---- x: the BT x 64 tile of each step by cp.async, XA steps in flight
    const int xt = tid - kGemmWWarps * 32;  // 0 .. kGemmXWarps * 32 - 1
    for (int step = 0; step < nk + XA; ++step) {
      if (step < nk) {
        const int s = step % S;
        if (step >= S && ok) ok = gemm_wait(&empty[s], ((step / S) - 1) & 1);
        uint8_t* bt = smem + s * STAGE + A_BYTES;
        const int k0 = step * kGemmBK;
        for (int c = xt; c < BT * 8; c += kGemmXWarps * 32) {
          const int t = c >> 3, ch = c & 7;
          const int m = m0 + t;
          const __half* src = a.x + (long long)min(m, a.M - 1) * a.sxm + k0 + ch * 8;
          cp_async16(smem_addr(bt + t * 128 + ((ch ^ (t & 7)) << 4)), src, m < a.M ? 16 : 0);
        }
      }
      cp_async_commit();  // (empty groups past the end keep the wait count uniform)
      const int landed = step - XA;  // the oldest step still in flight has landed after this wait
      cp_async_wait<XA>();
      if (landed >= 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&full_x[landed % S]);
      }
    }
  } else if (lane == 0) {
    // ---- MMA: one thread; a step's four MMAs read its stage, the commit frees it
    const uint32_t idesc = umma_idesc_f16(128, BT);
    for (int step = 0; step < nk && ok; ++step) {
      const int s = step % S;
      const unsigned ph = (step / S) & 1;
      ok = gemm_wait(&full_w[s], ph) && gemm_wait(&full_x[s], ph);
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t abase = smem_addr(smem + s * STAGE), bbase = abase + A_BYTES;
#pragma unroll
      for (int kk = 0; kk < kGemmBK / 16; ++kk)  // K = 16 per MMA: 32 bytes further along the swizzled rows
        umma_f16(tmem, umma_desc_sw128(abase + kk * 32), umma_desc_sw128(bbase + kk * 32), idesc,
                 (step > 0 || kk > 0) ? 1u : 0u);
      umma_commit(&empty[s]);
    }
    umma_commit(done);  // completes once every MMA issued above has
  }

  // ---- epilogue (warps 0-7: warp w reads TMEM lane quarter w % 4, the token half w / 4): fp16 outputs,
  // consecutive features per token
  bool fin = ok;
  if (warp < kGemmWWarps) fin = gemm_wait(done, 0) && ok;
  const bool all_ok = __syncthreads_and(fin ? 1 : 0) != 0;  // uniform: tcgen05.ld is warp-collective
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (all_ok && nk > 0 && warp < kGemmWWarps) {
    const int quarter = warp & 3;
    const int feat = n0 + quarter * 32 + lane;
    constexpr int CHUNK = 16;
    constexpr int HALF = BT / 2;  // BT >= 32: two halves of whole 16-column chunks; BT = 16: warps 0-3 only
    const int c_begin = BT >= 32 ? (warp >> 2) * HALF : 0, c_end = BT >= 32 ? c_begin + HALF : (warp < 4 ? BT : 0);
#pragma unroll 1
    for (int c0 = c_begin; c0 < c_end; c0 += CHUNK) {
      uint32_t v[CHUNK];
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (feat < a.N) {
#pragma unroll
        for (int j = 0; j < CHUNK; ++j) {
          const int m = m0 + c0 + j;
          if (m < a.M) a.y[(long long)m * a.sym + feat] = __float2half_rn(__uint_as_float(v[j]));
        }
      }
    }
  }
  if (!all_ok && warp == kGemmMmaWarp && lane == 0) gemm_wait(done, 0);  // MMAs finished before the memory goes
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(TMEM_COLS) : "memory");
  }
}

template <int BT>
static size_t gemm_smem_bytes() {
  return 1024 + (size_t)kGemmStages * (128 * 128 + BT * 128) + (3 * kGemmStages + 1) * 8 + 16;
}

template <int BT>
static int launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  const size_t smem = gemm_smem_bytes<BT>();
  static std::mutex mu;
  static std::vector<int> done_dev;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    bool seen = false;
    for (int d : done_dev) seen |= (d == dev);
    if (!seen) {
      const int rc = check_cuda(cudaFuncSetAttribute(int4_gemm_kernel<BT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)smem),
                                "int4_gemm: shared memory limit");
      if (rc != LI4_OK) return rc;
      done_dev.push_back(dev);
    }
  }
  dim3 grid((unsigned)((a.N + 127) / 128), (unsigned)((a.M + BT - 1) / BT), 1);
  int4_gemm_kernel<BT><<<grid, kGemmWSThreads, smem, stream>>>(a);
  return check_cuda(cudaGetLastError(), "int4_gemm: kernel launch");
}

}  // namespace li4

extern "C" int li4_int4_gemm(const void* x, const void* packed, const void* scale, const void* zero, void* y,
                             int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t stride_xm,
                             int64_t stride_pn, int64_t stride_sn, int64_t stride_ym, void* stream) {
  using namespace li4;
  if (M < 1 || N < 1 || K < 128 || K % 128 != 0)
    return set_error(LI4_ERR_INVALID_ARG, "int4_gemm: M=%lld N=%lld K=%lld (M, N >= 1; K a positive multiple of 128)",
                     (long long)M, (long long)N, (long long)K);
  if (group_size != 128)
    return set_error(LI4_ERR_UNSUPPORTED, "int4_gemm: group_size %lld (the tensor-core GEMM takes 128)",
                     (long long)group_size);
  if (M > (int64_t(1) << 30) || N > (int64_t(1) << 30) || K > (int64_t(1) << 24))
    return set_error(LI4_ERR_INVALID_ARG, "int4_gemm: M=%lld N=%lld K=%lld too large", (long long)M, (long long)N,
                     (long long)K);
  if (!x || !packed || !scale || !zero || !y) return set_error(LI4_ERR_INVALID_ARG, "int4_gemm: null pointer");
  if (stride_xm < K || stride_pn < K / 2 || stride_sn < K / 128 || stride_ym < N)
    return set_error(LI4_ERR_INVALID_ARG, "int4_gemm: row strides smaller than the rows");
  if (!aligned16(x) || stride_xm % 8 != 0 || !aligned16(packed) || stride_pn % 16 != 0)
    return set_error(LI4_ERR_ALIGNMENT, "int4_gemm: x and packed rows must start on 16-byte boundaries");
  if ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(zero)) & 1u)
    return set_error(LI4_ERR_ALIGNMENT, "int4_gemm: fp16 tensors must be 2-byte aligned");
  GemmArgs a;
  a.x = static_cast<const __half*>(x);
  a.packed = static_cast<const uint8_t*>(packed);
  a.scale = static_cast<const __half*>(scale);
  a.zero = static_cast<const __half*>(zero);
  a.y = static_cast<__half*>(y);
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.sxm = stride_xm;
  a.spn = stride_pn;
  a.ssn = stride_sn;
  a.sym = stride_ym;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  if (M <= 16) rc = launch_gemm<16>(a, s);
  else if (M <= 32) rc = launch_gemm<32>(a, s);
  else if (M <= 64) rc = launch_gemm<64>(a, s);
  else if (M <= 2048) rc = launch_gemm<128>(a, s);  // more CTAs on the SMs
  else rc = launch_gemm<256>(a, s);
  if (rc == LI4_OK) clear_error();
  return rc;
}
