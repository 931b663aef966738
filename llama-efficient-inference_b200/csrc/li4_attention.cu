// li4_attention.cu -- decode attention (one new token per sequence), sm_100a.
//
// A cluster of 1..8 CTAs per (KV head, sequence) splits the cached keys and
// values between its CTAs, and reads them once for all `REP` query heads that
// share them (grouped-query attention without the reference's repeat_kv
// copies, llama/model.py:155-164, 265-266).  The CTAs push their softmax max
// and sum, and then their partial P.V, into each other's shared memory (two
// cluster barriers), so the probabilities are normalised by the global sum
// before their fp16 rounding, as in the reference.
// The arithmetic follows the reference's fp16 decode step
// (llama/model.py:266-275):
//   s = fp16(q . k)             fp16 matmul, fp32 accumulation
//   s = fp16(s / sqrt(d))
//   p = fp16(softmax_fp32(s))   softmax(scores.float()).type_as(q)
//   o = fp16(sum_j p_j v_j)     fp16 matmul, fp32 accumulation
// The position lives in device memory, so one captured CUDA graph serves every
// position: keys 0 .. *pos are attended (the reference's cache slice
// [:start_pos + 1]).
#include "li4_common.cuh"
#include "li4_internal.h"

#include <cooperative_groups.h>

#include <mutex>
#include <vector>

namespace cg = cooperative_groups;

namespace li4 {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;

// DPL = HD / 32 consecutive fp16 values of one cached row as floats.
template <int DPL>
__device__ __forceinline__ void load_lane_dims(const __half* p, float (&v)[DPL]) {
  if constexpr (DPL == 1) {
    v[0] = __half2float(*p);
  } else if constexpr (DPL == 2) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(p));
    v[0] = f.x;
    v[1] = f.y;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    v[0] = a.x;
    v[1] = a.y;
    v[2] = b.x;
    v[3] = b.y;
  }
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gsrc)
               : "memory");
}

struct AttnArgs {
  const __half* q;
  long long sqb;
  const __half* cache_k;
  const __half* cache_v;
  long long csb, css;
  __half* out;
  long long sob;
  int n_kv_heads;
  const long long* pos;
  int max_seq;
  int chunk_max;  // keys per CTA at most: ceil(max_seq / cluster size)
  int red_in_k;   // STAGE: the warps' P.V partials reuse the key staging (free once the scores are in)
};

// STAGE: the CTA's keys and values are first copied into shared memory with cp.async (all of
// them in flight at once), the key rows with their 16-byte chunks XOR-swizzled by row so the
// per-key reads of a warp spread over the banks.
template <int REP, int HD, bool STAGE>
__global__ void __launch_bounds__(kAttnThreads) decode_attention_kernel(const __grid_constant__ AttnArgs a) {
  constexpr int DPL = HD / 32;  // dims per lane in P.V
  constexpr int CPR = HD / 8;   // 16-byte chunks per cached row
  constexpr int SWZ = (CPR < 8 ? CPR : 8) - 1;
  extern __shared__ __align__(16) float smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks();   // CTAs sharing this (KV head, sequence)
  const int c = (int)cluster.block_rank();
  float* q_s = smem;                         // [REP][HD]
  float* part = q_s + REP * HD;              // [S][REP][HD] partial P.V (collected in the first CTA)
  float* scores = part + S * REP * HD;       // [REP][chunk_max]
  // STAGE: [chunk_max][HD] keys (swizzled), then values, from the next 16-byte boundary (cp.async targets)
  __half* k_s = reinterpret_cast<__half*>((reinterpret_cast<uintptr_t>(scores + REP * a.chunk_max) + 15) & ~uintptr_t(15));
  __half* v_s = k_s + (size_t)a.chunk_max * HD;                         // STAGE: [chunk_max][HD]
  // [warps][REP][HD]: in the key staging when it is large enough, else after the staging / scores
  float* red = a.red_in_k ? reinterpret_cast<float*>(k_s)
                          : reinterpret_cast<float*>(STAGE ? reinterpret_cast<uintptr_t>(v_s + (size_t)a.chunk_max * HD)
                                                           : reinterpret_cast<uintptr_t>(k_s));
  __shared__ float s_wmax[kAttnWarps][REP], s_wsum[kAttnWarps][REP];
  __shared__ float s_lmax[REP], s_gmax[REP], s_gsum[REP];
  __shared__ float s_cm[8][REP], s_cl[8][REP];  // (max, sum) of every CTA of the cluster, pushed by each

  const int kvh = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __half* kbase = a.cache_k + (long long)b * a.csb + (long long)kvh * HD;
  const __half* vbase = a.cache_v + (long long)b * a.csb + (long long)kvh * HD;
  // cache rows [r0, r1) into their staging slots (slot 0 = row j0): keys (swizzled), then values
  auto stage_k = [&](int r0, int r1, int j0) {
    for (int idx = tid; idx < (r1 - r0) * CPR; idx += kAttnThreads) {
      const int jj = r0 - j0 + idx / CPR, cc = idx % CPR;
      cp_async16(k_s + jj * HD + ((cc ^ (jj & SWZ)) << 3), kbase + (long long)(j0 + jj) * a.css + cc * 8);
    }
  };
  auto stage_v = [&](int r0, int r1, int j0) {
    for (int idx = tid; idx < (r1 - r0) * CPR; idx += kAttnThreads) {
      const int jj = r0 - j0 + idx / CPR, cc = idx % CPR;
      cp_async16(v_s + jj * HD + cc * 8, vbase + (long long)(j0 + jj) * a.css + cc * 8);
    }
  };
  // Every CTA of the cluster must have started before a peer writes into its shared memory:
  // arrive now, wait just before the first remote store (by then the barrier is long complete).
  __shared__ long long s_pe;
  cluster.barrier_arrive();
  pdl_launch_dependents();
  // The preceding kernel writes q and cache row *pos only; the rows before it were written by
  // earlier steps.  Start copying them while that kernel finishes (keys and values as two
  // groups, so the scores can start before the values land), with the position as it reads now
  // (one value for the whole CTA, so every thread takes the same branch below); after the wait,
  // copy row *pos -- or everything again if the position has moved.
  if (tid == 0) s_pe = *a.pos;
  __syncthreads();
  long long pe = s_pe;
  pe = pe < 0 ? 0 : (pe >= a.max_seq ? a.max_seq - 1 : pe);
  const int chunk_e = ((int)pe + 1 + S - 1) / S;
  const int j0e = c * chunk_e, j1e = min((int)pe + 1, j0e + chunk_e);
  if (STAGE) {
    stage_k(j0e, min(j1e, (int)pe), j0e);
    asm volatile("cp.async.commit_group;" ::: "memory");
    stage_v(j0e, min(j1e, (int)pe), j0e);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  pdl_wait_primary();  // q and the cache row of this step come from the preceding kernel

  long long p = *a.pos;
  p = p < 0 ? 0 : (p >= a.max_seq ? a.max_seq - 1 : p);
  const int L = (int)p + 1;
  const int chunk = (L + S - 1) / S;
  const int j0 = c * chunk, j1 = min(L, j0 + chunk);
  const bool moved = p != pe;

  if (STAGE) {
    if (!moved) {
      if (j0 <= (int)p && (int)p < j1 && tid < 2 * CPR) {  // row *pos: one 16-byte chunk per thread
        const int jj = (int)p - j0, cc = tid % CPR;
        if (tid < CPR)
          *reinterpret_cast<uint4*>(k_s + jj * HD + ((cc ^ (jj & SWZ)) << 3)) =
              __ldcg(reinterpret_cast<const uint4*>(kbase + p * a.css + cc * 8));
        else
          *reinterpret_cast<uint4*>(v_s + jj * HD + cc * 8) =
              __ldcg(reinterpret_cast<const uint4*>(vbase + p * a.css + cc * 8));
      }
    } else {  // the position moved: every copy in flight lands first, then the whole range again
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncthreads();
      stage_k(j0, j1, j0);
      stage_v(j0, j1, j0);
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
  }
  for (int t = tid; t < REP * HD; t += kAttnThreads)
    q_s[t] = __half2float(a.q[(long long)b * a.sqb + (long long)kvh * REP * HD + t]);
  if (STAGE) {  // the keys (the values may still be in flight)
    if (!moved) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
  }
  __syncthreads();

  // scores of this CTA's keys: one key per thread, REP dot products over HD dims
  const float inv_scale = 1.0f / sqrtf((float)HD);
  float mx[REP];
#pragma unroll
  for (int r = 0; r < REP; ++r) mx[r] = -INFINITY;
  for (int j = j0 + tid; j < j1; j += kAttnThreads) {
    const uint4* kr = reinterpret_cast<const uint4*>(STAGE ? k_s + (j - j0) * HD : kbase + (long long)j * a.css);
    float dot[REP];
#pragma unroll
    for (int r = 0; r < REP; ++r) dot[r] = 0.f;
#pragma unroll
    for (int cc = 0; cc < HD / 8; ++cc) {
      const uint4 kv = kr[STAGE ? (cc ^ ((j - j0) & SWZ)) : cc];
      const uint32_t w[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
#pragma unroll
        for (int r = 0; r < REP; ++r) {
          dot[r] = fmaf(q_s[r * HD + cc * 8 + 2 * e], kf.x, dot[r]);
          dot[r] = fmaf(q_s[r * HD + cc * 8 + 2 * e + 1], kf.y, dot[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float s16 = __half2float(__float2half_rn(dot[r]));
      const float sc = __half2float(__float2half_rn(s16 * inv_scale));  // torch divides by a scalar as a product with its reciprocal
      scores[r * a.chunk_max + (j - j0)] = sc;
      mx[r] = fmaxf(mx[r], sc);
    }
  }
  // softmax over all L keys of the cluster, fp32.  Each CTA reduces its keys to (max m_c, sum of
  // exp(s - m_c)) and pushes both into every CTA's shared memory; after one cluster barrier every
  // CTA has the global max M and sum L = sum_c l_c exp(m_c - M), and rounds p = exp(s - M) / L.
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float v = mx[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) s_wmax[warp][r] = v;
  }
  __syncthreads();
  if (tid < REP) {
    float v = s_wmax[0][tid];
#pragma unroll
    for (int w = 1; w < kAttnWarps; ++w) v = fmaxf(v, s_wmax[w][tid]);
    s_lmax[tid] = v;
  }
  __syncthreads();
  float sum[REP];
#pragma unroll
  for (int r = 0; r < REP; ++r) sum[r] = 0.f;
  for (int j = tid; j < j1 - j0; j += kAttnThreads) {
#pragma unroll
    for (int r = 0; r < REP; ++r) sum[r] += expf(scores[r * a.chunk_max + j] - s_lmax[r]);
  }
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float v = sum[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) s_wsum[warp][r] = v;
  }
  __syncthreads();
  cluster.barrier_wait();
  if (tid < REP) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) v += s_wsum[w][tid];
    const float m = s_lmax[tid];
    for (int rk = 0; rk < S; ++rk) {  // push (m_c, l_c) into every CTA of the cluster
      *cluster.map_shared_rank(&s_cm[c][tid], rk) = m;
      *cluster.map_shared_rank(&s_cl[c][tid], rk) = v;
    }
  }
  cluster.sync();
  if (tid < REP) {
    float M = -INFINITY;
    for (int rk = 0; rk < S; ++rk) M = fmaxf(M, s_cm[rk][tid]);
    float Lsum = 0.f;
    for (int rk = 0; rk < S; ++rk)
      if (s_cm[rk][tid] != -INFINITY) Lsum += s_cl[rk][tid] * expf(s_cm[rk][tid] - M);
    s_gmax[tid] = M;
    s_gsum[tid] = Lsum;
  }
  __syncthreads();
  for (int j = tid; j < j1 - j0; j += kAttnThreads) {
#pragma unroll
    for (int r = 0; r < REP; ++r)
      scores[r * a.chunk_max + j] =
          __half2float(__float2half_rn(expf(scores[r * a.chunk_max + j] - s_gmax[r]) / s_gsum[r]));
  }
  if (STAGE) asm volatile("cp.async.wait_group 0;" ::: "memory");  // the values
  __syncthreads();

  // P.V over this CTA's keys: warp w takes keys j0 + w, j0 + w + 8, ...; lane holds DPL dims
  float acc[REP][DPL];
#pragma unroll
  for (int r = 0; r < REP; ++r)
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[r][e] = 0.f;
  const int nloc = j1 - j0;
  int j = warp;
  for (; j + 3 * kAttnWarps < nloc; j += 4 * kAttnWarps) {
    float v4[4][DPL];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      load_lane_dims<DPL>(STAGE ? v_s + (j + u * kAttnWarps) * HD + DPL * lane
                                : vbase + (long long)(j0 + j + u * kAttnWarps) * a.css + DPL * lane,
                          v4[u]);
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        const float pj = scores[r * a.chunk_max + j + u * kAttnWarps];
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[r][e] = fmaf(pj, v4[u][e], acc[r][e]);
      }
  }
  for (; j < nloc; j += kAttnWarps) {
    float vv[DPL];
    load_lane_dims<DPL>(STAGE ? v_s + j * HD + DPL * lane : vbase + (long long)(j0 + j) * a.css + DPL * lane, vv);
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float pj = scores[r * a.chunk_max + j];
#pragma unroll
      for (int e = 0; e < DPL; ++e) acc[r][e] = fmaf(pj, vv[e], acc[r][e]);
    }
  }
#pragma unroll
  for (int r = 0; r < REP; ++r)
#pragma unroll
    for (int e = 0; e < DPL; ++e) red[(warp * REP + r) * HD + DPL * lane + e] = acc[r][e];
  __syncthreads();
  float* part0 = cluster.map_shared_rank(part, 0);  // the first CTA collects [S][REP * HD] partials
  for (int t = tid; t < REP * HD; t += kAttnThreads) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) v += red[w * REP * HD + t];
    part0[c * REP * HD + t] = v;
  }
  cluster.sync();  // the last cluster barrier: after it only the first CTA reads shared memory, its own
  if (c == 0) {
    for (int t = tid; t < REP * HD; t += kAttnThreads) {
      float v = 0.f;
      for (int rk = 0; rk < S; ++rk) v += part[rk * REP * HD + t];
      a.out[(long long)b * a.sob + (long long)kvh * REP * HD + t] = __float2half_rn(v);
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core form, for CTAs whose keys and values fit in shared memory (every
// decode shape of the Llama models at their context lengths).  Same cluster split,
// same rounding points; the two products run as mma.m16n8k16 tiles:
//   S = Q K^T   A = q (REP head rows of 16, the rest zero) from registers, B = 8 keys
//               x 16 dims from the staged keys (ldmatrix), fp32 accumulation
//   O = P V     A = the fp16 probabilities of 16 keys, taken straight from the score
//               accumulators, B = 16 keys x 8 dims of the staged values (ldmatrix.trans)
// Warp w owns the 16-key blocks w, w + 8, ...; its scores stay in registers from the
// score tile to the P.V tile.  Each warp reduces its (max, sum of exp) per head, the
// CTA combines its warps, the cluster its CTAs (one push round through distributed
// shared memory), and every lane derives the global (max, sum) itself.  Both K and V
// rows are XOR-swizzled in 16-byte chunks so the 8 rows of an ldmatrix hit 8 banks.
// ---------------------------------------------------------------------------
constexpr size_t kAttnStageLimit = 96 * 1024;  // K + V of a CTA's keys staged when they fit in this

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

__device__ __forceinline__ uint32_t h2_bits(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int REP, int HD>
__global__ void __launch_bounds__(kAttnThreads) decode_attention_mma_kernel(const __grid_constant__ AttnArgs a) {
  constexpr int CPR = HD / 8;  // 16-byte chunks per cached row
  constexpr int SWZ = (CPR < 8 ? CPR : 8) - 1;
  constexpr int KS = HD / 16;  // k-steps of the score tile
  constexpr int DT = HD / 8;   // 8-dim tiles of the output
  constexpr int MAXB = (int)((kAttnStageLimit / (4 * HD) + 16 * kAttnWarps - 1) / (16 * kAttnWarps));
  static_assert(REP <= 8, "head rows of the score tile");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks();
  const int c = (int)cluster.block_rank();
  const int rows16 = a.chunk_max;  // staging rows per CTA, a multiple of 16 here
  __half* k_s = reinterpret_cast<__half*>(smem_raw);
  __half* v_s = k_s + (size_t)rows16 * HD;
  float* part = reinterpret_cast<float*>(v_s + (size_t)rows16 * HD);  // [S][REP * HD] (first CTA)
  float* red = part + (size_t)S * REP * HD;                            // [warps][REP * HD]
  __shared__ float s_wm[kAttnWarps][8], s_wl[kAttnWarps][8];
  __shared__ float s_cm[8][8], s_cl[8][8];  // (max, sum) of every CTA of the cluster, pushed by each

  const int kvh = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = lane >> 2, quad = lane & 3;
  const __half* kbase = a.cache_k + (long long)b * a.csb + (long long)kvh * HD;
  const __half* vbase = a.cache_v + (long long)b * a.csb + (long long)kvh * HD;
  auto swz = [](int row, int chunk) { return row * HD + ((chunk ^ (row & SWZ)) << 3); };
  auto stage = [&](__half* dst, const __half* base, int r0, int r1, int j0) {
    for (int idx = tid; idx < (r1 - r0) * CPR; idx += kAttnThreads) {
      const int jj = r0 - j0 + idx / CPR, cc = idx % CPR;
      cp_async16(dst + swz(jj, cc), base + (long long)(j0 + jj) * a.css + cc * 8);
    }
  };
  __shared__ long long s_pe;
  cluster.barrier_arrive();  // every CTA has started before a peer writes into its shared memory
  pdl_launch_dependents();
  // the position as it reads before the wait, one value for the whole CTA (so the choice below
  // between "as staged" and "moved" is the same in every thread)
  if (tid == 0) s_pe = *a.pos;
  __syncthreads();
  long long pe = s_pe;
  pe = pe < 0 ? 0 : (pe >= a.max_seq ? a.max_seq - 1 : pe);
  {
    const int chunk_e = ((int)pe + 1 + S - 1) / S;
    const int j0e = c * chunk_e, j1e = min((int)pe + 1, j0e + chunk_e);
    stage(k_s, kbase, j0e, min(j1e, (int)pe), j0e);
    asm volatile("cp.async.commit_group;" ::: "memory");
    stage(v_s, vbase, j0e, min(j1e, (int)pe), j0e);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  pdl_wait_primary();  // q and the cache row of this step come from the preceding kernel

  // q rows of the score tile's A operand (head grp of this KV head; zero rows above REP), the
  // cache row at the position read before the wait, and the position again, all in flight together
  uint32_t qa[KS][2];
  {
    const __half* qrow = a.q + (long long)b * a.sqb + (long long)(kvh * REP + (grp < REP ? grp : 0)) * HD;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qa[ks][0] = grp < REP ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * quad) : 0u;
      qa[ks][1] = grp < REP ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * quad) : 0u;
    }
  }
  uint4 rowpe = make_uint4(0u, 0u, 0u, 0u);
  if (tid < 2 * CPR)
    rowpe = __ldcg(reinterpret_cast<const uint4*>((tid < CPR ? kbase : vbase) + pe * a.css + (tid % CPR) * 8));
  long long p = *a.pos;
  p = p < 0 ? 0 : (p >= a.max_seq ? a.max_seq - 1 : p);
  const int L = (int)p + 1;
  const int chunk = (L + S - 1) / S;
  const int j0 = c * chunk, j1 = min(L, j0 + chunk);
  const int nloc = j1 > j0 ? j1 - j0 : 0;
  const int nblk = (nloc + 15) / 16;
  if (p == pe) {
    if (j0 <= (int)p && (int)p < j1 && tid < 2 * CPR)  // row *pos: one 16-byte chunk per thread
      *reinterpret_cast<uint4*>((tid < CPR ? k_s : v_s) + swz((int)p - j0, tid % CPR)) = rowpe;
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // the keys (the values may still be in flight)
  } else {  // the position moved: the copies in flight land first, then the whole range again
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    stage(k_s, kbase, j0, j1, j0);
    stage(v_s, vbase, j0, j1, j0);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 0;" ::: "memory");
  }
  // value rows past the keys of the last block meet zero probabilities: make them finite zeros
  for (int idx = tid; idx < (nblk * 16 - nloc) * CPR; idx += kAttnThreads) {
    const int jj = nloc + idx / CPR;
    *reinterpret_cast<uint4*>(v_s + swz(jj, idx % CPR)) = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();

  // scores of this warp's blocks: sc[bi][t][e] = key 16 (warp + 8 bi) + 8 t + 2 quad + e, head grp
  const float inv_scale = 1.0f / sqrtf((float)HD);
  float sc[MAXB][2][2];
  float mw = -INFINITY;
#pragma unroll
  for (int bi = 0; bi < MAXB; ++bi) {
    const int blk = warp + bi * kAttnWarps;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      sc[bi][t][0] = sc[bi][t][1] = -INFINITY;
      if (blk >= nblk) continue;  // (uniform over the warp)
      const int key0 = blk * 16 + t * 8;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kp = 0; kp < KS / 2; ++kp) {
        uint32_t bq[4];
        ldsm_x4(bq, k_s + swz(key0 + (lane & 7), kp * 4 + (lane >> 3)));
        mma_16816(acc, qa[2 * kp][0], 0u, qa[2 * kp][1], 0u, bq[0], bq[1]);
        mma_16816(acc, qa[2 * kp + 1][0], 0u, qa[2 * kp + 1][1], 0u, bq[2], bq[3]);
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = key0 + 2 * quad + e;
        const float s16 = __half2float(__float2half_rn(acc[e]));
        const float v = __half2float(__float2half_rn(s16 * inv_scale));  // torch divides as a product with 1/sqrt(d)
        sc[bi][t][e] = key < nloc ? v : -INFINITY;
        mw = fmaxf(mw, sc[bi][t][e]);
      }
    }
  }
  // (max, sum of exp) of head grp over this warp's keys, then over the CTA's warps
  mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, 1));
  mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, 2));
  float lw = 0.f;
  if (mw != -INFINITY) {
#pragma unroll
    for (int bi = 0; bi < MAXB; ++bi)
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 2; ++e) lw += expf(sc[bi][t][e] - mw);
  }
  lw += __shfl_xor_sync(0xffffffffu, lw, 1);
  lw += __shfl_xor_sync(0xffffffffu, lw, 2);
  if (quad == 0 && grp < REP) {
    s_wm[warp][grp] = mw;
    s_wl[warp][grp] = lw;
  }
  __syncthreads();
  cluster.barrier_wait();
  if (tid < REP) {
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) m = fmaxf(m, s_wm[w][tid]);
    float l = 0.f;
    if (m != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w)
        if (s_wm[w][tid] != -INFINITY) l += s_wl[w][tid] * expf(s_wm[w][tid] - m);
    }
    for (int rk = 0; rk < S; ++rk) {  // push (m_c, l_c) into every CTA of the cluster
      *cluster.map_shared_rank(&s_cm[c][tid], rk) = m;
      *cluster.map_shared_rank(&s_cl[c][tid], rk) = l;
    }
  }
  cluster.sync();
  // the global (max, sum) of head grp, derived by every lane in the same order
  const int hg = grp < REP ? grp : 0;
  float gM = -INFINITY;
  for (int rk = 0; rk < S; ++rk) gM = fmaxf(gM, s_cm[rk][hg]);
  float gL = 0.f;
  for (int rk = 0; rk < S; ++rk)
    if (s_cm[rk][hg] != -INFINITY) gL += s_cl[rk][hg] * expf(s_cm[rk][hg] - gM);
  asm volatile("cp.async.wait_group 0;" ::: "memory");  // the values
  __syncthreads();

  // O = P V over this warp's blocks: P = fp16(exp(s - M) / L) (softmax(scores.float()).type_as(q))
  float o[DT][4];
#pragma unroll
  for (int dt = 0; dt < DT; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
#pragma unroll
  for (int bi = 0; bi < MAXB; ++bi) {
    const int blk = warp + bi * kAttnWarps;
    if (blk >= nblk) continue;  // (uniform over the warp)
    uint32_t pa[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float p0 = grp < REP ? expf(sc[bi][t][0] - gM) / gL : 0.f;
      const float p1 = grp < REP ? expf(sc[bi][t][1] - gM) / gL : 0.f;
      pa[t] = h2_bits(p0, p1);
    }
#pragma unroll
    for (int dp = 0; dp < DT / 2; ++dp) {
      uint32_t bv[4];
      const int i = lane >> 3;
      ldsm_x4_trans(bv, v_s + swz(blk * 16 + (i & 1) * 8 + (lane & 7), 2 * dp + (i >> 1)));
      mma_16816(o[2 * dp], pa[0], 0u, pa[1], 0u, bv[0], bv[1]);
      mma_16816(o[2 * dp + 1], pa[0], 0u, pa[1], 0u, bv[2], bv[3]);
    }
  }
  if (grp < REP) {
#pragma unroll
    for (int dt = 0; dt < DT; ++dt) {
      red[(warp * REP + grp) * HD + dt * 8 + 2 * quad] = o[dt][0];
      red[(warp * REP + grp) * HD + dt * 8 + 2 * quad + 1] = o[dt][1];
    }
  }
  __syncthreads();
  float* part0 = cluster.map_shared_rank(part, 0);  // the first CTA collects [S][REP * HD] partials
  for (int t = tid; t < REP * HD; t += kAttnThreads) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) v += red[w * REP * HD + t];
    part0[c * REP * HD + t] = v;
  }
  cluster.sync();  // the last cluster barrier: after it only the first CTA reads shared memory, its own
  if (c == 0) {
    for (int t = tid; t < REP * HD; t += kAttnThreads) {
      float v = 0.f;
      for (int rk = 0; rk < S; ++rk) v += part[rk * REP * HD + t];
      a.out[(long long)b * a.sob + (long long)kvh * REP * HD + t] = __float2half_rn(v);
    }
  }
}

// Shared memory of the tensor-core form: K and V staging of rows16 rows, the cluster's partials,
// the warps' partials.
static size_t attn_mma_smem_bytes(int rep, int head_dim, int rows16, int cluster) {
  return (size_t)2 * rows16 * head_dim * sizeof(__half) + sizeof(float) * (size_t)rep * head_dim * (cluster + kAttnWarps);
}

// The warps' P.V partials reuse the key staging when it holds them.
static bool attn_red_in_k(int rep, int head_dim, int chunk_max, bool stage) {
  return stage && (size_t)chunk_max * head_dim * sizeof(__half) >= (size_t)kAttnWarps * rep * head_dim * sizeof(float);
}

// q, the cluster's partials, the scores, the K / V staging and the warps' partials (see the kernel).
static size_t attn_smem_bytes(int rep, int head_dim, int chunk_max, bool stage, int cluster) {
  size_t bytes = sizeof(float) * ((size_t)rep * head_dim * (1 + cluster) + (size_t)rep * chunk_max) + 16;
  if (stage) bytes += (size_t)2 * chunk_max * head_dim * sizeof(__half);
  if (!attn_red_in_k(rep, head_dim, chunk_max, stage)) bytes += sizeof(float) * (size_t)kAttnWarps * rep * head_dim;
  return bytes;
}

// CTAs per (KV head, sequence): a cluster of up to 8 when the (KV head, sequence)
// pairs alone leave SMs idle, as long as the doubled launch stays within 2 CTAs per SM
// and >= 32 keys per CTA at max_seq.
static int attn_cluster_size(int64_t pairs, int64_t max_seq, int sm) {
  int S = 1;
  while (S < 8 && pairs * S * 2 <= 2LL * sm && max_seq / (2 * S) >= 32) S *= 2;
  return S;
}

template <typename KernelT>
static int launch_attn(KernelT kernel, const AttnArgs& a, int batch, int cluster, size_t smem, cudaStream_t stream) {
  if (smem + 4096 > 48 * 1024) {  // dynamic + the static softmax partials past the 48 KiB default
    static std::mutex mu;
    static std::vector<std::pair<int, size_t>> raised;  // (device, bytes) of this instantiation
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    bool ok = false;
    for (auto& e : raised)
      if (e.first == dev && e.second >= smem) ok = true;
    if (!ok) {
      const int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                                "decode_attention: cudaFuncSetAttribute");
      if (rc != LI4_OK) return rc;
      raised.emplace_back(dev, smem);
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.n_kv_heads, (unsigned)batch, (unsigned)cluster);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = (unsigned)cluster;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, a), "decode_attention: kernel launch");
}

template <int REP, int HD>
static int launch_attention(const AttnArgs& a, int batch, int cluster, size_t smem, bool stage, bool mma,
                            cudaStream_t stream) {
  if (mma) return launch_attn(decode_attention_mma_kernel<REP, HD>, a, batch, cluster, smem, stream);
  if (stage) return launch_attn(decode_attention_kernel<REP, HD, true>, a, batch, cluster, smem, stream);
  return launch_attn(decode_attention_kernel<REP, HD, false>, a, batch, cluster, smem, stream);
}

}  // namespace li4

extern "C" int li4_decode_attention(const void* q, int64_t stride_qb, const void* cache_k, const void* cache_v,
                                    int64_t cache_stride_b, int64_t cache_stride_s, void* out, int64_t stride_ob,
                                    int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                                    const int64_t* pos, int64_t max_seq, void* stream) {
  using namespace li4;
  if (head_dim != 32 && head_dim != 64 && head_dim != 128)
    return set_error(LI4_ERR_UNSUPPORTED, "decode_attention: head_dim=%lld (32, 64 or 128)", (long long)head_dim);
  if (batch < 0 || n_kv_heads < 1 || n_heads < n_kv_heads || n_heads % n_kv_heads != 0 || max_seq < 1)
    return set_error(LI4_ERR_INVALID_ARG, "decode_attention: batch=%lld n_heads=%lld n_kv_heads=%lld max_seq=%lld",
                     (long long)batch, (long long)n_heads, (long long)n_kv_heads, (long long)max_seq);
  const int64_t rep = n_heads / n_kv_heads;
  if (rep != 1 && rep != 2 && rep != 4 && rep != 8)
    return set_error(LI4_ERR_UNSUPPORTED, "decode_attention: n_heads / n_kv_heads = %lld (1, 2, 4 or 8)",
                     (long long)rep);
  if (!q || !cache_k || !cache_v || !out || !pos)
    return set_error(LI4_ERR_INVALID_ARG, "decode_attention: null pointer");
  if (stride_qb < n_heads * head_dim || stride_ob < n_heads * head_dim || cache_stride_s < n_kv_heads * head_dim ||
      cache_stride_b < cache_stride_s * max_seq)
    return set_error(LI4_ERR_INVALID_ARG, "decode_attention: strides smaller than the rows");
  if (!aligned16(cache_k) || !aligned16(cache_v) || cache_stride_s % 8 != 0 || cache_stride_b % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(q) & 1u) || (reinterpret_cast<uintptr_t>(out) & 1u))
    return set_error(LI4_ERR_ALIGNMENT, "decode_attention: cache rows must be 16-byte aligned");
  if (max_seq > (1 << 20))
    return set_error(LI4_ERR_UNSUPPORTED, "decode_attention: max_seq=%lld above 2^20", (long long)max_seq);
  int cluster = attn_cluster_size(batch * n_kv_heads, max_seq, current_sm_count());
  while (cluster < 8 &&
         attn_smem_bytes((int)rep, (int)head_dim, (int)((max_seq + cluster - 1) / cluster), false, cluster) >
             200 * 1024)
    cluster *= 2;
  const int chunk_max = (int)((max_seq + cluster - 1) / cluster);
  const bool stage = (size_t)2 * chunk_max * head_dim * sizeof(__half) <= kAttnStageLimit;
  // the tensor-core form: keys and values of 16-key blocks staged, q rows read as 4-byte pairs
  const int rows16 = (chunk_max + 15) / 16 * 16;
  const bool mma = (size_t)2 * rows16 * head_dim * sizeof(__half) <= kAttnStageLimit &&
                   (reinterpret_cast<uintptr_t>(q) & 3u) == 0 && stride_qb % 2 == 0;
  const size_t smem = mma ? attn_mma_smem_bytes((int)rep, (int)head_dim, rows16, cluster)
                          : attn_smem_bytes((int)rep, (int)head_dim, chunk_max, stage, cluster);
  if (smem > 200 * 1024)
    return set_error(LI4_ERR_UNSUPPORTED, "decode_attention: max_seq=%lld needs %zu bytes of shared memory per CTA",
                     (long long)max_seq, smem);
  if (batch == 0) return LI4_OK;
  AttnArgs a;
  a.q = static_cast<const __half*>(q);
  a.sqb = stride_qb;
  a.cache_k = static_cast<const __half*>(cache_k);
  a.cache_v = static_cast<const __half*>(cache_v);
  a.csb = cache_stride_b;
  a.css = cache_stride_s;
  a.out = static_cast<__half*>(out);
  a.sob = stride_ob;
  a.n_kv_heads = (int)n_kv_heads;
  a.pos = reinterpret_cast<const long long*>(pos);
  a.max_seq = (int)max_seq;
  a.chunk_max = mma ? rows16 : chunk_max;  // the tensor-core form stages whole 16-key blocks
  a.red_in_k = attn_red_in_k((int)rep, (int)head_dim, chunk_max, stage) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  const int sel = (int)rep * 1000 + (int)head_dim;
  switch (sel) {
#define LI4_ATTN_CASE(R, H)                                                                  \
  case R * 1000 + H:                                                                           \
    rc = launch_attention<R, H>(a, (int)batch, cluster, smem, stage, mma, s);                  \
    break;
    LI4_ATTN_CASE(1, 32) LI4_ATTN_CASE(2, 32) LI4_ATTN_CASE(4, 32) LI4_ATTN_CASE(8, 32)
    LI4_ATTN_CASE(1, 64) LI4_ATTN_CASE(2, 64) LI4_ATTN_CASE(4, 64) LI4_ATTN_CASE(8, 64)
    LI4_ATTN_CASE(1, 128) LI4_ATTN_CASE(2, 128) LI4_ATTN_CASE(4, 128) LI4_ATTN_CASE(8, 128)
#undef LI4_ATTN_CASE
    default: rc = set_error(LI4_ERR_UNSUPPORTED, "decode_attention: rep=%lld head_dim=%lld", (long long)rep,
                            (long long)head_dim);
  }
  if (rc == LI4_OK) clear_error();
  return rc;
}
