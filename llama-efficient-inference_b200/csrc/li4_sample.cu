// li4_sample.cu -- greedy next-token selection on the GPU, sm_100a.
//
// One cluster of CTAs per row of logits: the index of the row's maximum, the first one on
// ties, a NaN counting as the maximum -- torch.argmax's answer (the
// reference's greedy step, bench.py:154-161 / llama/generation.py:59-60).
// Reading fp16 logits is exact: the reference's fp32 logits are the same
// values widened (llama/model.py:455).
#include "li4_common.cuh"
#include "li4_internal.h"

#include <algorithm>
#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace li4 {

constexpr int kArgmaxThreads = 512;
constexpr int kArgmaxCluster = 8;

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

// A cluster of kArgmaxCluster CTAs per row: CTA c scans columns [c*chunk, (c+1)*chunk) with
// 16-byte loads unrolled so they are in flight together, and the cluster's first CTA picks
// the winner among the CTAs' candidates through distributed shared memory.
// The winner of a row as one signed 64-bit key whose order is torch.argmax's: the value's
// order-preserving bits (NaN above every number, -0 as +0) above the complement of the global
// index (the smaller index wins a tie), with the top bit flipped so that signed comparison (a
// MAX reduction over int64) orders the keys as unsigned comparison would.
__device__ __forceinline__ long long argmax_signed_key(float v, long long global_index) {
  unsigned u = __float_as_uint(v), ord;
  if (v != v) {
    ord = 0xFFFFFFFFu;
  } else {
    if (v == 0.f) u = 0u;
    ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  const unsigned long long key =
      ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)global_index);
  return (long long)(key ^ 0x8000000000000000ull);
}

// Exchange of the shards' winners between tensor-parallel ranks (li4_argmax_rows_allreduce): the
// row's key goes to every rank as two 8-byte words {key half, epoch} stored straight into each
// rank's receive buffer over NVLink (one 8-byte store is seen whole); the rank then polls its own
// buffer (bounded) for every rank's two words of the row, and the largest key names the token.
// The epoch is the row's call count on this rank (every rank makes the same calls), and its
// parity picks one of two buffer halves, so call k + 1 never overwrites words of call k that a
// slower rank may still be reading.
struct KeyExchange {
  unsigned long long* recv[8];  // every rank's receive buffer [2][world][rows][2] words
  unsigned* epochs;             // this rank's call count per row
  long long rows;
  int world, rank;
};

__device__ unsigned g_sample_device_error;  // bit 6 of li4_device_errors
constexpr unsigned kKeyWaitLimit = 1u << 20;
__device__ unsigned g_key_wait_limit = kKeyWaitLimit;

int sample_device_errors(unsigned* flags, bool reset) {
  int rc = check_cuda(cudaMemcpyFromSymbol(flags, g_sample_device_error, sizeof(unsigned)), "device_errors: argmax");
  if (rc == LI4_OK && reset) {
    const unsigned zero = 0;
    rc = check_cuda(cudaMemcpyToSymbol(g_sample_device_error, &zero, sizeof(unsigned)), "device_errors: clearing");
  }
  return rc;
}

int sample_set_wait_limit(unsigned polls) {
  const unsigned v = polls ? polls : kKeyWaitLimit;
  return check_cuda(cudaMemcpyToSymbol(g_key_wait_limit, &v, sizeof(v)), "debug_set_wait_limits: argmax exchange");
}

__device__ __forceinline__ long long exchange_key(const KeyExchange& x, long long row, long long key) {
  const unsigned epoch = atomicAdd(&x.epochs[row], 1u) + 1u;
  const long long half = (long long)(epoch & 1u) * x.world * x.rows * 2;
  const unsigned long long hi = ((unsigned long long)epoch << 32) | (unsigned)((unsigned long long)key >> 32);
  const unsigned long long lo = ((unsigned long long)epoch << 32) | (unsigned)((unsigned long long)key);
  for (int r = 0; r < x.world; ++r) {
    if (r == x.rank) continue;
    unsigned long long* dst = x.recv[r] + half + ((long long)x.rank * x.rows + row) * 2;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(hi) : "memory");
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst + 1), "l"(lo) : "memory");
  }
  long long best = key;
  bool failed = false;
  for (int r = 0; r < x.world; ++r) {
    if (r == x.rank) continue;
    const unsigned long long* src = x.recv[x.rank] + half + ((long long)r * x.rows + row) * 2;
    unsigned long long w0 = 0, w1 = 0;
    const unsigned limit = failed ? 1u : g_key_wait_limit;
    for (unsigned it = 0;; ++it) {
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w0) : "l"(src) : "memory");
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w1) : "l"(src + 1) : "memory");
      if ((unsigned)(w0 >> 32) == epoch && (unsigned)(w1 >> 32) == epoch) break;
      if (it + 1 >= limit) {
        if (!failed) atomicOr(&g_sample_device_error, 64u);
        failed = true;
        break;
      }
    }
    const long long k = (long long)(((w0 & 0xFFFFFFFFull) << 32) | (w1 & 0xFFFFFFFFull));
    if (k > best) best = k;
  }
  return best;
}

// key_offset < 0: out[row] = the row's argmax index; otherwise out[row] = argmax_signed_key of the
// row's winner at global index key_offset + index, or, with an exchange (x.world > 0), the global
// index of the winner over every rank's shard.
template <bool F16>
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const void* logits, long long cols,
                                                                     long long stride, long long* out,
                                                                     long long out_stride, long long chunk,
                                                                     long long key_offset,
                                                                     const __grid_constant__ KeyExchange x) {
  __shared__ Best s_best[kArgmaxThreads / 32];
  __shared__ Best s_cta;
  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks(), c = (int)cluster.block_rank();
  const long long row = blockIdx.y;
  pdl_launch_dependents();
  pdl_wait_primary();  // the logits come from the preceding kernel
  const long long c0 = (long long)c * chunk, c1 = min(cols, c0 + chunk);
  Best best{-INFINITY, (long long)cols};  // loses to every real entry
  if constexpr (F16) {
    const __half* x = static_cast<const __half*>(logits) + row * stride;
    // chunk is a multiple of 8: each CTA's first vector starts on a 16-byte boundary when the row does
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
    const long long v0 = vec ? c0 / 8 : 0, v1 = vec ? c1 / 8 : 0;
#pragma unroll 4
    for (long long v = v0 + threadIdx.x; v < v1; v += kArgmaxThreads) {
      const uint4 u = reinterpret_cast<const uint4*>(x)[v];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
        take(best, f.x, 8 * v + 2 * e);
        take(best, f.y, 8 * v + 2 * e + 1);
      }
    }
    for (long long i = (vec ? max(c0, 8 * v1) : c0) + threadIdx.x; i < c1; i += kArgmaxThreads)
      take(best, __half2float(x[i]), i);
  } else {
    const float* x = static_cast<const float*>(logits) + row * stride;
    // chunk is a multiple of 8: each CTA's first 16-byte vector is aligned when the row is; the
    // loop is unrolled so a thread's loads are in flight together
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
    const long long v0 = vec ? c0 / 4 : 0, v1 = vec ? c1 / 4 : 0;
#pragma unroll 8
    for (long long v = v0 + threadIdx.x; v < v1; v += kArgmaxThreads) {
      const float4 f = reinterpret_cast<const float4*>(x)[v];
      take(best, f.x, 4 * v);
      take(best, f.y, 4 * v + 1);
      take(best, f.z, 4 * v + 2);
      take(best, f.w, 4 * v + 3);
    }
    for (long long i = (vec ? max(c0, 4 * v1) : c0) + threadIdx.x; i < c1; i += kArgmaxThreads) take(best, x[i], i);
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
    best = lane < kArgmaxThreads / 32 ? s_best[lane] : Best{-INFINITY, (long long)cols};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Best other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
      if (better(other, best)) best = other;
    }
    if (lane == 0) s_cta = best;
  }
  cluster.sync();
  if (c == 0 && threadIdx.x == 0) {
    Best win = s_cta;
    for (int rk = 1; rk < S; ++rk) {
      const Best other = *cluster.map_shared_rank(&s_cta, rk);
      if (better(other, win)) win = other;
    }
    if (key_offset < 0) {
      out[row * out_stride] = win.i;
    } else if (x.world == 0) {
      out[row * out_stride] = argmax_signed_key(win.v, key_offset + win.i);
    } else {
      const long long best = exchange_key(x, row, argmax_signed_key(win.v, key_offset + win.i));
      out[row * out_stride] = 0xFFFFFFFFLL - (best & 0xFFFFFFFFLL);
    }
  }
  cluster.sync();  // every CTA's candidate stays in place until the first CTA has read it
}

}  // namespace li4

static int argmax_launch(const void* logits, int dtype, int64_t rows, int64_t cols, int64_t stride, int64_t* out,
                         int64_t out_stride, int64_t key_offset, void* stream,
                         const li4::KeyExchange& x = li4::KeyExchange{}) {
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
  // columns per CTA of the row's cluster: a multiple of 8 (16-byte vectors), at least 8
  const int S = kArgmaxCluster;
  const long long chunk = std::max<long long>(8, ((cols + S - 1) / S + 7) / 8 * 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)S, (unsigned)rows, 1);
  cfg.blockDim = dim3(kArgmaxThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)S;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  long long* o = reinterpret_cast<long long*>(out);
  const long long ko = (long long)key_offset;
  const int rc = dtype == LI4_F16
                     ? check_cuda(cudaLaunchKernelEx(&cfg, argmax_rows_kernel<true>, logits, (long long)cols,
                                                     (long long)stride, o, (long long)out_stride, chunk, ko, x),
                                  "argmax_rows: kernel launch")
                     : check_cuda(cudaLaunchKernelEx(&cfg, argmax_rows_kernel<false>, logits, (long long)cols,
                                                     (long long)stride, o, (long long)out_stride, chunk, ko, x),
                                  "argmax_rows: kernel launch");
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_argmax_rows(const void* logits, int dtype, int64_t rows, int64_t cols, int64_t stride,
                               int64_t* out, int64_t out_stride, void* stream) {
  return argmax_launch(logits, dtype, rows, cols, stride, out, out_stride, -1, stream);
}

extern "C" int li4_argmax_rows_keys(const void* logits, int dtype, int64_t rows, int64_t cols, int64_t stride,
                                    int64_t index_offset, int64_t* keys, int64_t keys_stride, void* stream) {
  if (index_offset < 0 || index_offset + cols > (int64_t(1) << 32) - 1)
    return li4::set_error(LI4_ERR_INVALID_ARG, "argmax_rows_keys: index_offset=%lld cols=%lld (global indices "
                          "below 2^32 - 1)", (long long)index_offset, (long long)cols);
  return argmax_launch(logits, dtype, rows, cols, stride, keys, keys_stride, index_offset, stream);
}

extern "C" int li4_argmax_rows_allreduce(const void* logits, int dtype, int64_t rows, int64_t cols, int64_t stride,
                                         int64_t index_offset, void* const* recv, size_t recv_bytes,
                                         unsigned* epochs, int world, int rank, int64_t* out, int64_t out_stride,
                                         void* stream) {
  using namespace li4;
  if (index_offset < 0 || index_offset + cols > (int64_t(1) << 32) - 1)
    return set_error(LI4_ERR_INVALID_ARG, "argmax_rows_allreduce: index_offset=%lld cols=%lld (global indices "
                     "below 2^32 - 1)", (long long)index_offset, (long long)cols);
  if (world < 1 || world > 8 || rank < 0 || rank >= world || !recv || !epochs ||
      (reinterpret_cast<uintptr_t>(epochs) & 3u))
    return set_error(LI4_ERR_INVALID_ARG, "argmax_rows_allreduce: world=%d rank=%d (1..8 ranks), receive buffers "
                     "and a 4-byte aligned epoch array", world, rank);
  const size_t need = (size_t)2 * world * (size_t)(rows > 0 ? rows : 0) * 2 * sizeof(unsigned long long);
  if (recv_bytes < need)
    return set_error(LI4_ERR_INVALID_ARG, "argmax_rows_allreduce: receive buffers of %zu bytes, %zu needed "
                     "(2 x world x rows x 2 words of 8 bytes)", recv_bytes, need);
  KeyExchange x = {};
  for (int r = 0; r < world; ++r) {
    if (!recv[r] || (reinterpret_cast<uintptr_t>(recv[r]) & 7u))
      return set_error(LI4_ERR_ALIGNMENT, "argmax_rows_allreduce: receive buffer %d is null or not 8-byte aligned", r);
    x.recv[r] = static_cast<unsigned long long*>(recv[r]);
  }
  x.epochs = epochs;
  x.rows = rows;
  x.world = world;
  x.rank = rank;
  return argmax_launch(logits, dtype, rows, cols, stride, out, out_stride, index_offset, stream, x);
}
