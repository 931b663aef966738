// li4_gemv.cu -- fused INT4 dequant + GEMV / small-M GEMM for decode (M <= 16), sm_100a.
//
// y[M, N] = x[M, K] @ W[N, K]^T with W in the packed INT4 format of
// llama/quantize.py:44-75 (see include/llama_int4_b200.h).
//
// Work decomposition (both kernel families):
//   * a CTA (4 warps) owns a tile of ROWS = 16*RT consecutive output rows n
//     and one K range of `ks_per_split` ksteps (a kstep = 128 k = 64 packed
//     bytes per row); grid.y indexes the K range (split-K), grid.x walks the
//     row tiles persistently;
//   * the 4 warps interleave the ksteps of the K range; inside a warp, lane
//     (grp = lane/4, quad = lane%4) reads rows grp and grp+8 of each 16-row
//     slab, bytes [16*quad, 16*quad + 16) of each kstep: one 128-bit load
//     covers 32 k values of one row, 4 lanes cover a 64-byte kstep, so every
//     warp-wide load touches 8 rows x 64 contiguous bytes;
//   * x for the CTA's K range is staged once in shared memory, permuted into
//     the (k, k+4) pairs that the nibble unpack produces;
//   * partial sums of the 4 warps are reduced in shared memory; with split-K
//     the K ranges write fp32 partials to a workspace and the last CTA to
//     arrive on a tile (arrival counter) sums them in fixed order, writes
//     fp16 y and resets the counter -- one launch, no zero-fill, no cast
//     kernel (replaces llama/int4_gemv.py:80-89, 126-139).
//
// Math:
//   * MMA family: W slab (16 rows x 16 k, exact q - zero in fp16) is the A
//     operand of mma.m16n8k16 and x^T the B operand (M in the n dimension,
//     padded to 8 or 16); fp32 accumulation per 128-k kstep, then scaled by
//     the group scale in fp32 (groups >= 128), or scale applied to A in fp16
//     (groups 32/64: the fp16 weight equals the reference's bit for bit).
//   * CUDA-core family (M <= 8): each lane forms sum_k (q - zero) * x over its
//     32 k with sm_100 mixed-precision fp16 x fp16 + fp32 FMAs, scales by the
//     group scale in fp32, and the 4 lanes of a row are reduced by warp
//     shuffles.
#include "li4_common.cuh"
#include "li4_gemv_device.cuh"
#include "li4_internal.h"

#include <algorithm>
#include <mutex>
#include <vector>

namespace li4 {

// Start pulling the first row tile's weight bytes into L2 (TMA bulk prefetch)
// before waiting on the preceding kernel.
template <int ROWS>
__device__ __forceinline__ void prefetch_first_tile(const GemvArgs& a, int ks0, int nks) {
  const int tile = blockIdx.x;
  if (tile >= a.n_tiles || nks == 0) return;
  const int r = tile * ROWS + threadIdx.x;
  if (threadIdx.x < ROWS && r < a.N) {
    const uint8_t* p = a.packed + (long long)r * a.spn + (long long)ks0 * 64;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(nks * 64) : "memory");
  }
}

// Sum the per-warp partials of one row tile and write y (split == 1) or the
// split-K partials + last-arriver reduction (split > 1).
template <int ROWS, int COLS>
__device__ __forceinline__ void finish_tile(const GemvArgs& a, int tile, const float* red, int* s_flag) {
  const int row0 = tile * ROWS;
  const int M = a.M;
  if (a.split == 1) {
    for (int idx = threadIdx.x; idx < ROWS * M; idx += kThreads) {
      const int row = idx / M, m = idx - (idx / M) * M;
      const int n = row0 + row;
      if (n < a.N) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[(w * ROWS + row) * COLS + m];
        a.y[(long long)m * a.sym + n] = __float2half_rn(v);
      }
    }
    return;
  }
  for (int idx = threadIdx.x; idx < ROWS * M; idx += kThreads) {
    const int row = idx / M, m = idx - (idx / M) * M;
    const int n = row0 + row;
    if (n < a.N) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) v += red[(w * ROWS + row) * COLS + m];
      a.partial[((long long)blockIdx.y * M + m) * a.N + n] = v;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&a.counters[tile], 1u);
    *s_flag = (prev == (unsigned)(a.split - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (*s_flag) {
    __threadfence();
    for (int idx = threadIdx.x; idx < ROWS * M; idx += kThreads) {
      const int row = idx / M, m = idx - (idx / M) * M;
      const int n = row0 + row;
      if (n < a.N) {
        float v = 0.f;
        for (int s = 0; s < a.split; ++s) v += __ldcg(&a.partial[((long long)s * M + m) * a.N + n]);
        a.y[(long long)m * a.sym + n] = __float2half_rn(v);
      }
    }
    if (threadIdx.x == 0) a.counters[tile] = 0u;  // ready for the next launch
  }
}

// ---------------------------------------------------------------------------
// Tensor-core family.
// ---------------------------------------------------------------------------
template <int RT, int NT, bool SCALE_IN_A>
__global__ void __launch_bounds__(kThreads) gemv_mma_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_flag;
  constexpr int ROWS = 16 * RT;
  constexpr int COLS = 8 * NT;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int grp = lane >> 2, quad = lane & 3;
  const int nks = a.ks_per_split;
  const int ks0 = blockIdx.y * nks;
  const int M8 = (NT == 1) ? a.M : 8;
  uint8_t* xs = smem;
  float* red = reinterpret_cast<float*>(smem + ((nks * NT * M8 * 256 + 127) & ~127));

  pdl_launch_dependents();
  prefetch_first_tile<ROWS>(a, ks0, nks);
  pdl_wait_primary();
  stage_x<NT>(a, ks0, nks, M8, xs);
  __syncthreads();

  for (int tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x) {
    const int row0 = tile * ROWS;
    const uint8_t* prow[RT][2];
    const __half* srow[RT][2];
    const __half* zrow[RT][2];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        int r = row0 + rt * 16 + grp + 8 * h;
        r = r < a.N ? r : a.N - 1;
        prow[rt][h] = a.packed + (long long)r * a.spn + (long long)ks0 * 64 + quad * 16;
        srow[rt][h] = a.scale + (long long)r * a.ssn;
        zrow[rt][h] = a.zero + (long long)r * a.ssn;
      }

    float acc[RT][NT][4];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[rt][nt][e] = 0.f;

    for (int kb = warp; kb < nks; kb += kWarps * kBatch) {
      uint4 wv[kBatch][RT][2];
      __half sv[kBatch][RT][2], zv[kBatch][RT][2];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int ks = kb + b * kWarps;
        if (ks < nks) {
          const int g = ((ks0 + ks) * 128 + 32 * quad) >> a.log2_group;
#pragma unroll
          for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              wv[b][rt][h] = ldg_stream_v4(prow[rt][h] + ks * 64);
              sv[b][rt][h] = ldg_half(srow[rt][h] + g);
              zv[b][rt][h] = ldg_half(zrow[rt][h] + g);
            }
        }
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int ks = kb + b * kWarps;
        if (ks < nks) {
          ZeroConsts zc[RT][2];
          __half2 s2[RT][2];
#pragma unroll
          for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              zc[rt][h] = make_zero_consts(zv[b][rt][h]);
              s2[rt][h] = __halves2half2(sv[b][rt][h], sv[b][rt][h]);
            }
          float c[RT][NT][4];
#pragma unroll
          for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) c[rt][nt][e] = 0.f;
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            __half2 p[RT][2][4];
#pragma unroll
            for (int rt = 0; rt < RT; ++rt)
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint4 v = wv[b][rt][h];
                const uint32_t word = (w == 0) ? v.x : (w == 1) ? v.y : (w == 2) ? v.z : v.w;
                unpack8_qz(word, zc[rt][h], p[rt][h]);
                if (SCALE_IN_A) {
#pragma unroll
                  for (int i = 0; i < 4; ++i) p[rt][h][i] = __hmul2(p[rt][h][i], s2[rt][h]);
                }
              }
            uint4 bq[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              if (grp < M8)
                bq[nt] = lds128(xs + xs_chunk_offset(((ks * NT + nt) * M8 + grp) * 4 + quad, w, grp));
              else
                bq[nt] = make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int rt = 0; rt < RT; ++rt)
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                float* cc = SCALE_IN_A ? acc[rt][nt] : c[rt][nt];
                mma_16816(cc, h2_as_u32(p[rt][0][0]), h2_as_u32(p[rt][1][0]), h2_as_u32(p[rt][0][1]),
                          h2_as_u32(p[rt][1][1]), bq[nt].x, bq[nt].y);
                mma_16816(cc, h2_as_u32(p[rt][0][2]), h2_as_u32(p[rt][1][2]), h2_as_u32(p[rt][0][3]),
                          h2_as_u32(p[rt][1][3]), bq[nt].z, bq[nt].w);
              }
          }
          if (!SCALE_IN_A) {
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) {
              const float s_lo = __half2float(sv[b][rt][0]);
              const float s_hi = __half2float(sv[b][rt][1]);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                acc[rt][nt][0] = fmaf(s_lo, c[rt][nt][0], acc[rt][nt][0]);
                acc[rt][nt][1] = fmaf(s_lo, c[rt][nt][1], acc[rt][nt][1]);
                acc[rt][nt][2] = fmaf(s_hi, c[rt][nt][2], acc[rt][nt][2]);
                acc[rt][nt][3] = fmaf(s_hi, c[rt][nt][3], acc[rt][nt][3]);
              }
            }
          }
        }
      }
    }

    __syncthreads();  // previous tile's readers of `red` are done
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = rt * 16 + grp + 8 * (e >> 1);
          const int col = nt * 8 + 2 * quad + (e & 1);
          red[(warp * ROWS + row) * COLS + col] = acc[rt][nt][e];
        }
    __syncthreads();
    finish_tile<ROWS, COLS>(a, tile, red, &s_flag);
  }
}

// ---------------------------------------------------------------------------
// CUDA-core family (M <= 8).
// ---------------------------------------------------------------------------
template <int M, int RT>
__global__ void __launch_bounds__(kThreads) gemv_cc_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_flag;
  constexpr int ROWS = 16 * RT;
  constexpr int COLS = 8;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int grp = lane >> 2, quad = lane & 3;
  const int nks = a.ks_per_split;
  const int ks0 = blockIdx.y * nks;
  uint8_t* xs = smem;
  float* red = reinterpret_cast<float*>(smem + ((nks * M * 256 + 127) & ~127));

  pdl_launch_dependents();
  prefetch_first_tile<ROWS>(a, ks0, nks);
  pdl_wait_primary();
  stage_x<1>(a, ks0, nks, M, xs);
  __syncthreads();

  for (int tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x) {
    const int row0 = tile * ROWS;
    const uint8_t* prow[RT][2];
    const __half* srow[RT][2];
    const __half* zrow[RT][2];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        int r = row0 + rt * 16 + grp + 8 * h;
        r = r < a.N ? r : a.N - 1;
        prow[rt][h] = a.packed + (long long)r * a.spn + (long long)ks0 * 64 + quad * 16;
        srow[rt][h] = a.scale + (long long)r * a.ssn;
        zrow[rt][h] = a.zero + (long long)r * a.ssn;
      }

    float acc[RT][2][M];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[rt][h][m] = 0.f;

    for (int kb = warp; kb < nks; kb += kWarps * kBatch) {
      uint4 wv[kBatch][RT][2];
      __half sv[kBatch][RT][2], zv[kBatch][RT][2];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int ks = kb + b * kWarps;
        if (ks < nks) {
          const int g = ((ks0 + ks) * 128 + 32 * quad) >> a.log2_group;
#pragma unroll
          for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              wv[b][rt][h] = ldg_stream_v4(prow[rt][h] + ks * 64);
              sv[b][rt][h] = ldg_half(srow[rt][h] + g);
              zv[b][rt][h] = ldg_half(zrow[rt][h] + g);
            }
        }
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int ks = kb + b * kWarps;
        if (ks < nks) {
          ZeroConsts zc[RT][2];
#pragma unroll
          for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int h = 0; h < 2; ++h) zc[rt][h] = make_zero_consts(zv[b][rt][h]);
          float part[RT][2][M];
#pragma unroll
          for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int m = 0; m < M; ++m) part[rt][h][m] = 0.f;
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            __half2 p[RT][2][4];
#pragma unroll
            for (int rt = 0; rt < RT; ++rt)
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint4 v = wv[b][rt][h];
                const uint32_t word = (w == 0) ? v.x : (w == 1) ? v.y : (w == 2) ? v.z : v.w;
                unpack8_qz(word, zc[rt][h], p[rt][h]);
              }
#pragma unroll
            for (int m = 0; m < M; ++m) {
              const uint4 xq = lds128(xs + xs_chunk_offset((ks * M + m) * 4 + quad, w, m));
#pragma unroll
              for (int rt = 0; rt < RT; ++rt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  float t = part[rt][h][m];
                  t = fma2_f16_f32(h2_as_u32(p[rt][h][0]), xq.x, t);
                  t = fma2_f16_f32(h2_as_u32(p[rt][h][1]), xq.y, t);
                  t = fma2_f16_f32(h2_as_u32(p[rt][h][2]), xq.z, t);
                  t = fma2_f16_f32(h2_as_u32(p[rt][h][3]), xq.w, t);
                  part[rt][h][m] = t;
                }
            }
          }
#pragma unroll
          for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float s = __half2float(sv[b][rt][h]);
#pragma unroll
              for (int m = 0; m < M; ++m) acc[rt][h][m] = fmaf(s, part[rt][h][m], acc[rt][h][m]);
            }
        }
      }
    }

    // reduce the 4 lanes (quads) that share a row
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int m = 0; m < M; ++m) {
          float v = acc[rt][h][m];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          acc[rt][h][m] = v;
        }

    __syncthreads();
    if (quad == 0) {
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int m = 0; m < M; ++m) red[(warp * ROWS + rt * 16 + grp + 8 * h) * COLS + m] = acc[rt][h][m];
    }
    __syncthreads();
    finish_tile<ROWS, COLS>(a, tile, red, &s_flag);
  }
}

// ---------------------------------------------------------------------------
// Streaming-warp tensor-core kernel (groups >= 128).
//
// Work unit: one kstep (128 k) of one 16-row tile.  Each warp walks its own
// sequence of units through a register ring kStreamDepth units deep: the loads
// of unit u + D are issued right after unit u is consumed, so every warp keeps
// D units (D KiB) in flight at all times, and the first D units are requested
// before griddepcontrol.wait (weights never depend on the preceding kernel).
// Row, scale and zero addresses are rebuilt only when a warp moves to a new
// tile.  Thread (grp, quad) computes rows grp and grp + 8 of the tile with
// m16n8k16 MMAs (exact q - zero in fp16, fp32 accumulation per kstep, scaled
// by the group scale in fp32), exactly as the classic MMA kernel.
//
// Rows mode: a warp owns whole tiles (all ksteps of its K range), so nothing
// is shared between warps.  K-split mode (few tiles): the 8 warps of a CTA share
// every tile, warp w taking ksteps w, w + 8, ...; the partial sums meet in
// shared memory once per tile.
// ---------------------------------------------------------------------------
constexpr int kStreamWarps = 8;
constexpr int kStreamThreads = kStreamWarps * 32;
constexpr int kStreamDepth = 5;

// Per-warp walk over (tile, kstep) units.
struct StreamCursor {
  int tile;   // current tile (>= n_tiles: done)
  int j;      // unit index inside the tile for this warp
};

template <bool KSPLIT>
__device__ __forceinline__ void stream_advance(StreamCursor& c, int units_per_tile, int tile_step) {
  if (++c.j == units_per_tile) {
    c.j = 0;
    c.tile += tile_step;
  }
}


// ---------------------------------------------------------------------------
// All-reduce + residual epilogue (LI4_EPI_ALLREDUCE_RESIDUAL), streaming-warp kernel only.
//
// Under tensor parallelism a row-parallel linear's output is the sum over ranks of
// each rank's fp16 partial.  Here the GEMV that computes a tile also finishes it:
// the tile's outputs go out as 8-byte words {fp16 row j, fp16 row j + 8, epoch},
// stored straight into every peer's receive buffer over NVLink (one 8-byte store
// is seen whole, so the epoch in a word vouches for its data: no flags, no fences),
// and the same threads then poll their own receive buffer until every peer's word
// of the same (tile, m, j) carries this call's epoch, sum the ranks' values in fp32
// in rank order, round, add the residual and store -- exactly the arithmetic of
// li4_allreduce_add after a plain GEMV.  The epoch of a tile is its call count on
// this rank (ar_epochs, one atomic per tile and call); all ranks make the same calls,
// so their counts agree.  A wait that runs out sets bit 5 and uses what it read; the
// thread's later words then get one poll each, so a missing peer costs one poll limit.
// ---------------------------------------------------------------------------
constexpr unsigned kArEpiWaitLimit = 1u << 20;  // polls of one word before giving up
__device__ unsigned g_ar_epi_wait_limit = kArEpiWaitLimit;  // li4_debug_set_wait_limits shortens it for tests

int gemv_set_ar_wait_limit(unsigned polls) {
  const unsigned v = polls ? polls : kArEpiWaitLimit;
  return check_cuda(cudaMemcpyToSymbol(g_ar_epi_wait_limit, &v, sizeof(v)), "debug_set_wait_limits: fused all-reduce");
}

__device__ __forceinline__ unsigned long long ar_pack(float v0, float v1, unsigned epoch) {
  const __half2 h = __floats2half2_rn(v0, v1);
  return ((unsigned long long)epoch << 32) | *reinterpret_cast<const unsigned*>(&h);
}

__device__ __forceinline__ long long ar_index(const GemvArgs& a, int tile, int m, int j) {
  return ((long long)tile * a.M + m) * 8 + j;
}

// This rank's word into every other rank's receive buffer (its own value stays in registers).
__device__ __forceinline__ void ar_push(const GemvArgs& a, long long widx, unsigned long long w) {
  for (int r = 0; r < a.ar_world; ++r) {
    if (r == a.ar_rank) continue;
    unsigned long long* dst = a.ar_recv[r] + (long long)a.ar_rank * a.ar_words + widx;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(w) : "memory");
  }
}

// Up to W words of this thread (live mask) summed over the ranks in rank order, and rows
// row[i], row[i] + 8 of output row m[i] stored.  The residuals are requested first, and each
// rank's W words are polled together, so a thread's words cost one round trip per rank.
template <int W>
__device__ __forceinline__ void ar_finish(const GemvArgs& a, const long long (&widx)[W], const int (&m)[W],
                                          const int (&row)[W], unsigned live, const unsigned long long (&own)[W],
                                          unsigned epoch) {
  float rs0[W], rs1[W], s0[W], s1[W];
#pragma unroll
  for (int i = 0; i < W; ++i) {
    s0[i] = s1[i] = rs0[i] = rs1[i] = 0.f;
    if (live >> i & 1u) {
      const __half* res = a.res + (long long)m[i] * a.srm + row[i];
      rs0[i] = __half2float(res[0]);
      rs1[i] = __half2float(res[8]);
    }
  }
  bool failed = false;
  for (int r = 0; r < a.ar_world; ++r) {
    unsigned long long w[W];
#pragma unroll
    for (int i = 0; i < W; ++i) w[i] = own[i];
    if (r != a.ar_rank) {
      const unsigned long long* base = a.ar_recv[a.ar_rank] + (long long)r * a.ar_words;
      const unsigned limit = failed ? 1u : g_ar_epi_wait_limit;
      unsigned pending = live;
      for (unsigned it = 0; pending != 0u; ++it) {
#pragma unroll
        for (int i = 0; i < W; ++i)
          if (pending >> i & 1u) asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[i]) : "l"(base + widx[i]) : "memory");
#pragma unroll
        for (int i = 0; i < W; ++i)
          if ((pending >> i & 1u) && (unsigned)(w[i] >> 32) == epoch) pending &= ~(1u << i);
        if (pending != 0u && it + 1 >= limit) {
          if (!failed) atomicOr(&g_li4_device_error, 32u);
          failed = true;
          break;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const unsigned lo = (unsigned)w[i];
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&lo));
      s0[i] += f.x;
      s1[i] += f.y;
    }
  }
#pragma unroll
  for (int i = 0; i < W; ++i) {
    if (!(live >> i & 1u)) continue;
    const float2 sum = __half22float2(__floats2half2_rn(s0[i], s1[i]));  // fp16 of the all-reduced partials
    __half* y = a.y + (long long)m[i] * a.sym + row[i];
    y[0] = __float2half_rn(rs0[i] + sum.x);
    y[8] = __float2half_rn(rs1[i] + sum.y);
  }
}

// A 16-row tile from a group of nthr threads that can all read value(r, m), W words per thread
// (W * nthr >= 8 * M): every word is computed, then pushed, then finished.
template <int W, typename F>
__device__ __forceinline__ void emit_tile_ar(const GemvArgs& a, int tile, int tid, int nthr, F value, unsigned epoch) {
  long long widx[W];
  int mm[W], row[W];
  unsigned long long own[W];
  unsigned live = 0;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const int idx = tid + i * nthr, m = idx >> 3, j = idx & 7;
    mm[i] = m;
    row[i] = tile * 16 + j;
    widx[i] = ar_index(a, tile, m, j);
    own[i] = 0ull;
    if (idx < 8 * a.M) {
      live |= 1u << i;
      own[i] = ar_pack(value(j, m), value(j + 8, m), epoch);
    }
  }
#pragma unroll
  for (int i = 0; i < W; ++i)
    if (live >> i & 1u) ar_push(a, widx[i], own[i]);
  ar_finish<W>(a, widx, mm, row, live, own, epoch);
}

// Rows mode, split == 1: a warp's tile from its lanes' accumulators; lane (grp, quad) holds rows
// grp and grp + 8 of columns nt*8 + 2*quad + {0, 1}, i.e. whole words.
template <int NT>
__device__ __forceinline__ void emit_warp_tile_ar(const GemvArgs& a, int tile, const float (&acc)[NT][4], int grp,
                                                  int quad, unsigned epoch) {
  constexpr int W = 2 * NT;
  long long widx[W];
  int mm[W], row[W];
  unsigned long long own[W];
  unsigned live = 0;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int i = 2 * nt + e, m = nt * 8 + 2 * quad + e;
      mm[i] = m;
      row[i] = tile * 16 + grp;
      widx[i] = ar_index(a, tile, m, grp);
      own[i] = ar_pack(acc[nt][e], acc[nt][e + 2], epoch);
      if (m < a.M) live |= 1u << i;
    }
#pragma unroll
  for (int i = 0; i < W; ++i)
    if (live >> i & 1u) ar_push(a, widx[i], own[i]);
  ar_finish<W>(a, widx, mm, row, live, own, epoch);
}

// The call's epoch of a tile, taken by lane 0 of the calling warp and shared with the warp.
__device__ __forceinline__ unsigned ar_warp_epoch(const GemvArgs& a, int tile, int lane) {
  unsigned e = 0;
  if (lane == 0) e = atomicAdd(&a.ar_epochs[tile], 1u) + 1u;
  return __shfl_sync(0xffffffffu, e, 0);
}

template <int NT, bool KSPLIT, bool FUSED, bool AR = false>
__global__ void __launch_bounds__(kStreamThreads, 2) gemv_stream_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int D = kStreamDepth;
  constexpr int COLS = 8 * NT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 2, quad = lane & 3;
  const int nks = a.ks_per_split;
  const int ks0 = blockIdx.y * nks;
  const int M8 = (NT == 1) ? a.M : 8;
  uint8_t* xs = smem;
  float* red = reinterpret_cast<float*>(smem + ((nks * NT * M8 * 256 + 127) & ~127));  // K-split: [2][8][16][COLS]

  // unit walk of this warp
  const int units_per_tile = KSPLIT ? (nks - warp + kStreamWarps - 1) / kStreamWarps : nks;
  const int tile_step = KSPLIT ? gridDim.x : gridDim.x * kStreamWarps;
  StreamCursor lc{KSPLIT ? (int)blockIdx.x : (int)(blockIdx.x * kStreamWarps + warp), 0};
  StreamCursor cc = lc;
  int lrows_tile = -1;
  StreamRows lrows{};

  pdl_launch_dependents();
  StreamUnit buf[D];
#pragma unroll
  for (int d = 0; d < D; ++d) {
    if (lc.tile < a.n_tiles && units_per_tile > 0) {
      if (lc.tile != lrows_tile) { lrows = stream_rows(a, lc.tile, ks0, grp, quad); lrows_tile = lc.tile; }
      stream_load(a, buf[d], lrows, KSPLIT ? warp + kStreamWarps * lc.j : lc.j);
    }
    stream_advance<KSPLIT>(lc, units_per_tile, tile_step);
  }
  pdl_wait_primary();  // x is written by the preceding kernel
  if (KSPLIT) prefetch_residual<FUSED>(a, blockIdx.x, threadIdx.x);
  else prefetch_residual<FUSED>(a, blockIdx.x * kStreamWarps + warp, lane);
  __shared__ float s_rstd[LI4_MAX_M];
  __shared__ unsigned s_ar_epoch[2];  // K-split mode, all-reduce epilogue: the tile's epoch (double-buffered as red)
  if (FUSED && a.norm_w != nullptr) {
    if (a.ssq_in != nullptr) rms_from_ssq<kStreamWarps>(a, s_rstd, threadIdx.x >> 5, threadIdx.x & 31);
    else rms_factors<kStreamWarps>(a, s_rstd, threadIdx.x >> 5, threadIdx.x & 31);
    __syncthreads();
  }
  if (FUSED && a.norm_w != nullptr) stage_x<NT, kStreamThreads, true>(a, ks0, nks, M8, xs, s_rstd);
  else stage_x<NT, kStreamThreads, false>(a, ks0, nks, M8, xs);
  __syncthreads();

  // this thread's B-fragment offsets inside one (kstep, n-tile) group
  const bool bvalid = grp < M8;
  int boff[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) boff[w] = (grp * 4 + quad) * 64 + ((w ^ xs_key(grp, quad)) << 4);
  const int ks_stride = NT * M8 * 256;

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
  int tiles_done = 0;

  bool more = cc.tile < a.n_tiles && units_per_tile > 0;
  while (more) {
#pragma unroll
    for (int d = 0; d < D; ++d) {
      if (!more) break;
      const int ks = KSPLIT ? warp + kStreamWarps * cc.j : cc.j;
      stream_compute<NT>(buf[d], xs + ks * ks_stride, M8 * 256, boff, bvalid, acc);
      const int tile = cc.tile;
      const bool tile_end = (cc.j == units_per_tile - 1);
      // refill this ring slot with the unit D ahead
      if (lc.tile < a.n_tiles) {
        if (lc.tile != lrows_tile) { lrows = stream_rows(a, lc.tile, ks0, grp, quad); lrows_tile = lc.tile; }
        stream_load(a, buf[d], lrows, KSPLIT ? warp + kStreamWarps * lc.j : lc.j);
      }
      stream_advance<KSPLIT>(lc, units_per_tile, tile_step);
      stream_advance<KSPLIT>(cc, units_per_tile, tile_step);
      more = cc.tile < a.n_tiles;
      if (tile_end) {
        const int row0 = tile * 16;
        const int rows = min(16, a.N - row0);
        if (!KSPLIT) {
          if (a.split == 1) {
            if constexpr (AR)
              emit_warp_tile_ar<NT>(a, tile, acc, grp, quad, ar_warp_epoch(a, tile, lane));
            else
              emit_warp_tile<FUSED, NT>(a, tile, acc, grp, quad);
          } else {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int r = grp + 8 * (e >> 1), m = nt * 8 + 2 * quad + (e & 1);
                if (r < rows && m < a.M) a.partial[((long long)blockIdx.y * a.M + m) * a.N + row0 + r] = acc[nt][e];
              }
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
          if (a.split > 1) {  // last K range to arrive sums the partials (fixed order) and resets the counter
            __threadfence();
            __syncwarp();
            unsigned last = 0;
            if (lane == 0) last = (atomicAdd(&a.counters[tile], 1u) == (unsigned)(a.split - 1)) ? 1u : 0u;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
              __threadfence();
              if constexpr (AR)
                emit_tile_ar<4>(a, tile, lane, 32, PartialSum{a.partial + row0, a.M, a.N, a.split},
                                ar_warp_epoch(a, tile, lane));
              else if constexpr (NT == 2) emit_partial_tile<FUSED>(a, tile, lane, PartialSum{a.partial + row0, a.M, a.N, a.split});
              else emit_tile<FUSED>(a, tile, lane, 32, PartialSum{a.partial + row0, a.M, a.N, a.split});
              __syncwarp();
              if (lane == 0) a.counters[tile] = 0u;
            }
          }
        } else {
          float* rb = red + (tiles_done & 1) * (kStreamWarps * 16 * COLS);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              rb[(warp * 16 + grp + 8 * (e >> 1)) * COLS + nt * 8 + 2 * quad + (e & 1)] = acc[nt][e];
              acc[nt][e] = 0.f;
            }
          const bool ar = AR && a.split == 1;
          if (ar && threadIdx.x == 0) s_ar_epoch[tiles_done & 1] = atomicAdd(&a.ar_epochs[tile], 1u) + 1u;
          __syncthreads();
          const WarpTileSum<COLS, kStreamWarps> tile_sum{rb};
          if (a.split == 1) {
            if (ar) emit_tile_ar<1>(a, tile, threadIdx.x, kStreamThreads, tile_sum, s_ar_epoch[tiles_done & 1]);
            else emit_tile<FUSED>(a, tile, threadIdx.x, kStreamThreads, tile_sum);
          } else {
            for (int idx = threadIdx.x; idx < rows * a.M; idx += kStreamThreads) {
              const int r = idx / a.M, m = idx - (idx / a.M) * a.M;
              a.partial[((long long)blockIdx.y * a.M + m) * a.N + row0 + r] = tile_sum(r, m);
            }
          }
          if (a.split > 1) {
            __threadfence();  // every writer publishes its partials before the arrival count
            __syncthreads();
            if constexpr (AR) {
              // the last K range to arrive finishes the tile with the whole CTA (one word per thread)
              if (threadIdx.x == 0) {
                const bool last = atomicAdd(&a.counters[tile], 1u) == (unsigned)(a.split - 1);
                if (last) a.counters[tile] = 0u;
                s_ar_epoch[tiles_done & 1] = last ? atomicAdd(&a.ar_epochs[tile], 1u) + 1u : 0u;
              }
              __syncthreads();
              const unsigned ep = s_ar_epoch[tiles_done & 1];
              if (ep != 0u) {
                __threadfence();
                emit_tile_ar<1>(a, tile, threadIdx.x, kStreamThreads, PartialSum{a.partial + row0, a.M, a.N, a.split},
                                ep);
              }
            } else if (warp == 0) {
              unsigned last = 0;
              if (lane == 0) last = (atomicAdd(&a.counters[tile], 1u) == (unsigned)(a.split - 1)) ? 1u : 0u;
              last = __shfl_sync(0xffffffffu, last, 0);
              if (last) {
                __threadfence();
                if constexpr (NT == 2) emit_partial_tile<FUSED>(a, tile, lane, PartialSum{a.partial + row0, a.M, a.N, a.split});
                else emit_tile<FUSED>(a, tile, lane, 32, PartialSum{a.partial + row0, a.M, a.N, a.split});
                __syncwarp();
                if (lane == 0) a.counters[tile] = 0u;
              }
            }
          }
          ++tiles_done;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Tile-streaming kernel for the common decode configuration: group 128 and a
// K range of exactly 16 ksteps (2048 k) per CTA.  Each warp owns whole tiles
// of 16*RT rows and walks them with the 16 ksteps fully unrolled, so every
// weight / scale / x offset is an immediate and the pointers change once per
// tile.  A register ring of D = 8 / RT units keeps 8 KiB per warp in flight;
// while the last D ksteps of a tile are computed, the first D units of the
// warp's next tile are already being fetched, and the first tile's units are
// requested before griddepcontrol.wait.  Math as in the streaming kernel.
// ---------------------------------------------------------------------------
constexpr int kTileKs = 16;    // ksteps of 128 k per K range
#ifndef LI4_TILE_DEPTH
#define LI4_TILE_DEPTH 4
#endif
constexpr int kTileDepth = LI4_TILE_DEPTH;  // register-ring units (of 16 rows) in flight per warp

template <int RT>
struct TileUnit {
  uint4 w[RT][2];        // rows rt*16 + grp (+8), bytes [16 quad, +16) of one kstep
  uint32_t sz[RT][2];    // scale | zero << 16
};

// Per-lane offsets of one tile's rows: bytes into `packed`, elements into
// `scale` / `zero` (which share a row stride).  32-bit: the planner only picks
// this kernel when every offset fits.
template <int RT>
struct TileRows {
  uint32_t p[RT][2];
  uint32_t s[RT][2];
};

template <int RT>
__device__ __forceinline__ TileRows<RT> tile_rows(const GemvArgs& a, int tile, int ks0, int grp, int quad) {
  TileRows<RT> t;
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int r = tile * 16 * RT + rt * 16 + grp + 8 * h;
      r = r < a.N ? r : a.N - 1;
      t.p[rt][h] = (uint32_t)r * (uint32_t)a.spn + (uint32_t)(ks0 * 64 + quad * 16);
      t.s[rt][h] = (uint32_t)r * (uint32_t)a.ssn + (uint32_t)ks0;
    }
  return t;
}

template <int RT>
__device__ __forceinline__ void tile_load(TileUnit<RT>& u, const GemvArgs& a, const TileRows<RT>& t, int ks) {
  const unsigned short* sc = reinterpret_cast<const unsigned short*>(a.scale);
  const unsigned short* ze = reinterpret_cast<const unsigned short*>(a.zero);
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      u.w[rt][h] = ldg_stream_v4(a.packed + t.p[rt][h] + ks * 64);
      u.sz[rt][h] = ldg_u16(sc + t.s[rt][h] + ks) | (ldg_u16(ze + t.s[rt][h] + ks) << 16);
    }
}

template <int NT, int RT>
__device__ __forceinline__ void tile_compute(const TileUnit<RT>& u, const uint8_t* xs_ks, int nt_stride,
                                             const int boff[4], bool bvalid, float acc[RT][NT][4]) {
  ZeroConsts zc[RT][2];
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int h = 0; h < 2; ++h) zc[rt][h] = make_zero_consts(__ushort_as_half((unsigned short)(u.sz[rt][h] >> 16)));
  float c[RT][NT][4];
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) c[rt][nt][e] = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint4 bq[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      bq[nt] = make_uint4(0u, 0u, 0u, 0u);
      if (bvalid) bq[nt] = lds128_ordered(xs_ks + nt * nt_stride + boff[w]);
    }
#pragma unroll
    for (int rt = 0; rt < RT; ++rt) {
      __half2 pl[4], ph[4];
      const uint4& lo = u.w[rt][0];
      const uint4& hi = u.w[rt][1];
      unpack8_qz((w == 0) ? lo.x : (w == 1) ? lo.y : (w == 2) ? lo.z : lo.w, zc[rt][0], pl);
      unpack8_qz((w == 0) ? hi.x : (w == 1) ? hi.y : (w == 2) ? hi.z : hi.w, zc[rt][1], ph);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma_16816(c[rt][nt], h2_as_u32(pl[0]), h2_as_u32(ph[0]), h2_as_u32(pl[1]), h2_as_u32(ph[1]), bq[nt].x,
                  bq[nt].y);
        mma_16816(c[rt][nt], h2_as_u32(pl[2]), h2_as_u32(ph[2]), h2_as_u32(pl[3]), h2_as_u32(ph[3]), bq[nt].z,
                  bq[nt].w);
      }
    }
  }
#pragma unroll
  for (int rt = 0; rt < RT; ++rt) {
    const float sl = __half2float(__ushort_as_half((unsigned short)(u.sz[rt][0] & 0xFFFFu)));
    const float sh = __half2float(__ushort_as_half((unsigned short)(u.sz[rt][1] & 0xFFFFu)));
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      acc[rt][nt][0] = fmaf(sl, c[rt][nt][0], acc[rt][nt][0]);
      acc[rt][nt][1] = fmaf(sl, c[rt][nt][1], acc[rt][nt][1]);
      acc[rt][nt][2] = fmaf(sh, c[rt][nt][2], acc[rt][nt][2]);
      acc[rt][nt][3] = fmaf(sh, c[rt][nt][3], acc[rt][nt][3]);
    }
  }
}

template <int NT, int RT, bool FUSED>
__global__ void __launch_bounds__(kStreamThreads, (RT == 1 ? 2 : 1)) gemv_tile_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int NKS = kTileKs;
  constexpr int D = kTileDepth / RT;
  constexpr int ROWS = 16 * RT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 2, quad = lane & 3;
  const int ks0 = blockIdx.y * NKS;
  constexpr int M8 = 8;  // x rows padded to 8 per n-tile: every B-fragment offset is an immediate
  uint8_t* xs = smem;
  const int tile_step = gridDim.x * kStreamWarps;
  int tile = blockIdx.x * kStreamWarps + warp;

  pdl_launch_dependents();
  TileUnit<RT> buf[D];
  TileRows<RT> cur = tile_rows<RT>(a, tile < a.n_tiles ? tile : 0, ks0, grp, quad);
  if (tile < a.n_tiles) {
#pragma unroll
    for (int d = 0; d < D; ++d) tile_load<RT>(buf[d], a, cur, d);
  }
  pdl_wait_primary();  // x is written by the preceding kernel
  prefetch_residual<FUSED>(a, tile * RT, lane);
  if (RT == 2) prefetch_residual<FUSED>(a, tile * RT + 1, lane);
  __shared__ float s_rstd[LI4_MAX_M];
  if (FUSED && a.norm_w != nullptr) {
    if (a.ssq_in != nullptr) rms_from_ssq<kStreamWarps>(a, s_rstd, threadIdx.x >> 5, threadIdx.x & 31);
    else rms_factors<kStreamWarps>(a, s_rstd, threadIdx.x >> 5, threadIdx.x & 31);
    __syncthreads();
  }
  if (FUSED && a.norm_w != nullptr) stage_x<NT, kStreamThreads, true>(a, ks0, NKS, M8, xs, s_rstd);
  else stage_x<NT, kStreamThreads, false>(a, ks0, NKS, M8, xs);
  __syncthreads();

  const bool bvalid = grp < ((NT == 1) ? a.M : 8);
  int boff[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) boff[w] = (grp * 4 + quad) * 64 + ((w ^ xs_key(grp, quad)) << 4);
  constexpr int nt_stride = M8 * 256;
  constexpr int ks_stride = NT * nt_stride;

  for (; tile < a.n_tiles; tile += tile_step) {
    const int next = tile + tile_step;
    const bool has_next = next < a.n_tiles;
    TileRows<RT> nxt;
    float acc[RT][NT][4];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[rt][nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < NKS; ++ks) {
      tile_compute<NT, RT>(buf[ks % D], xs + ks * ks_stride, nt_stride, boff, bvalid, acc);
      if (ks + D < NKS) {
        tile_load<RT>(buf[ks % D], a, cur, ks + D);
      } else {
        if (ks + D == NKS) nxt = tile_rows<RT>(a, has_next ? next : tile, ks0, grp, quad);
        if (has_next) tile_load<RT>(buf[ks % D], a, nxt, ks + D - NKS);
      }
    }
    const int row0 = tile * ROWS;
    if (FUSED && a.am_keys != nullptr) {  // greedy argmax of the logits this warp writes (split == 1)
#pragma unroll
      for (int rt = 0; rt < RT; ++rt) {
        if (row0 + rt * 16 >= a.N) continue;  // (uniform over the warp)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          unsigned long long kb[2] = {0ull, 0ull};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int row = row0 + rt * 16 + grp + 8 * (e >> 1), m = nt * 8 + 2 * quad + (e & 1);
            if (row < a.N && m < a.M)  // the value the epilogue writes: fp16-rounded, widened
              kb[e & 1] = max(kb[e & 1], argmax_key(__half2float(__float2half_rn(acc[rt][nt][e])), row));
          }
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            unsigned long long v = kb[j];
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
            const int m = nt * 8 + 2 * quad + j;
            if (grp == 0 && m < a.M && v != 0ull) atomicMax(&a.am_keys[m], v);
          }
        }
      }
    }
#pragma unroll
    for (int rt = 0; rt < RT; ++rt) {
      if (a.split == 1) {
        if (row0 + rt * 16 < a.N) emit_warp_tile<FUSED, NT>(a, tile * RT + rt, acc[rt], grp, quad);
        continue;
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = row0 + rt * 16 + grp + 8 * (e >> 1), m = nt * 8 + 2 * quad + (e & 1);
          if (r < a.N && m < a.M) a.partial[((long long)blockIdx.y * a.M + m) * a.N + r] = acc[rt][nt][e];
        }
    }
    if (a.split > 1) {  // last K range to arrive sums the partials (fixed order) and resets the counter
      __threadfence();
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) last = (atomicAdd(&a.counters[tile], 1u) == (unsigned)(a.split - 1)) ? 1u : 0u;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence();
#pragma unroll
        for (int rt = 0; rt < RT; ++rt) {
          const int sub = tile * RT + rt;
          if (sub * 16 >= a.N) break;
          if constexpr (NT == 2) emit_partial_tile<FUSED>(a, sub, lane, PartialSum{a.partial + sub * 16, a.M, a.N, a.split});
          else emit_tile<FUSED>(a, sub, lane, 32, PartialSum{a.partial + sub * 16, a.M, a.N, a.split});
        }
        __syncwarp();
        if (lane == 0) a.counters[tile] = 0u;
      }
    }
    cur = nxt;
  }
  if (FUSED && a.am_keys != nullptr) argmax_finish(a, [] { __syncthreads(); });
}

// ---------------------------------------------------------------------------
// Bulk-copy pipeline kernel.  A producer warp moves whole 16-row tiles of one K
// range (packed rows, scale and zero rows) from HBM into a ring of shared-memory
// stages with cp.async.bulk (the TMA engine's 1-D bulk copy), completing on
// per-stage mbarriers; consumer warp w owns ring stage w, takes every
// `stages`-th tile whole (all its ksteps, no cross-warp reduction) and runs the
// epilogue from its registers.  The ring holds up to kBulkMaxStages x 18 KiB per SM in
// flight (against 4-5 KiB per warp for the register rings), and the first
// stages are requested before
// griddepcontrol.wait, so the weight stream of a launch overlaps the tail of the
// preceding kernel.  Every mbarrier wait is bounded; a wait that runs out sets
// g_li4_device_error and the kernel drains its own copies and returns.
// ---------------------------------------------------------------------------
// Consumer warps: one per ring stage at most (10 for M <= 8, 8 for M <= 16).  Warp w consumes
// only stage w (tiles w, w + stages, ...), so it waits on each stage's uses in order and never
// polls an mbarrier phase more than one ahead of the barrier (which would read as complete).
__host__ __device__ constexpr int bulk_consumer_warps(int nt) { return nt == 1 ? 10 : 8; }
__host__ __device__ constexpr int bulk_threads(int nt) { return (bulk_consumer_warps(nt) + 1) * 32; }  // + producer
constexpr int kBulkMaxStages = 10;  // = bulk_consumer_warps(1)
template <int NT, bool FUSED>
__global__ void __launch_bounds__(bulk_threads(NT), 1) gemv_bulk_kernel(const __grid_constant__ GemvArgs a, int stages,
                                                                        int contig) {
  constexpr int CW = bulk_consumer_warps(NT);
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int M8 = 8;           // x rows padded to 8 per n-tile (as the tile kernel)
  const int ks_n = a.ks_per_split;
  const BulkLayout L = bulk_layout(ks_n, contig != 0);
  uint8_t* ring = smem;
  uint8_t* xs = ring + (size_t)stages * L.stage;
  uint64_t* full = reinterpret_cast<uint64_t*>(xs + (size_t)ks_n * NT * M8 * 256);
  uint64_t* empty = full + kBulkMaxStages;
  __shared__ float s_rstd[LI4_MAX_M];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks0 = blockIdx.y * ks_n;
  // this CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int my_tiles = (a.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);  // the consumer warp that owns the stage's tile
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == CW) {
    // ---------------- producer warp ----------------
    const unsigned stage_bytes = 16u * (unsigned)(ks_n * 64) + 2u * 16u * (unsigned)(ks_n * 2);
    bool ok = true;
    int issued = 0;
    for (int it = 0; it < my_tiles && ok; ++it) {
      const int s = it % stages;
      if (it >= stages) ok = mbar_wait_bounded(&empty[s], ((it / stages) - 1) & 1);
      if (!ok) break;
      issued = it + 1;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], stage_bytes);
      __syncwarp();
      const int tile = (int)blockIdx.x + it * (int)gridDim.x;
      uint8_t* st = ring + (size_t)s * L.stage;
      if (contig) {  // rows tile*16 .. +15 are one block of packed, scale and zero (the last tile is clamped)
        if (lane == 0) {
          const int r0 = min(tile * 16, a.N - 16);
          bulk_g2s(st, a.packed + (long long)r0 * a.spn, 16 * ks_n * 64, &full[s]);
          bulk_g2s(st + L.sz_off, a.scale + (long long)r0 * a.ssn, 16 * ks_n * 2, &full[s]);
          bulk_g2s(st + L.sz_off + 16 * ks_n * 2, a.zero + (long long)r0 * a.ssn, 16 * ks_n * 2, &full[s]);
        }
      } else if (lane < 16) {
        int r = tile * 16 + lane;
        r = r < a.N ? r : a.N - 1;
        bulk_g2s(st + lane * L.pitch, a.packed + (long long)r * a.spn + (long long)ks0 * 64, ks_n * 64, &full[s]);
        bulk_g2s(st + L.sz_off + lane * ks_n * 2, a.scale + (long long)r * a.ssn + ks0, ks_n * 2, &full[s]);
      } else {
        int r = tile * 16 + (lane - 16);
        r = r < a.N ? r : a.N - 1;
        bulk_g2s(st + L.sz_off + 16 * ks_n * 2 + (lane - 16) * ks_n * 2, a.zero + (long long)r * a.ssn + ks0,
                 ks_n * 2, &full[s]);
      }
    }
    // Drain: the last fill of every stage has landed before the producer leaves (a stage is
    // refilled only after its previous fill was consumed, so these are the only copies that
    // can be in flight; on the normal path they complete as the data arrives).
    for (int it = (issued > stages ? issued - stages : 0); it < issued; ++it)
      mbar_wait_bounded(&full[it % stages], (it / stages) & 1);
    pdl_wait_primary();  // every thread of the grid passes the dependency wait
    return;
  }

  // ---------------- consumer warps: one whole tile per warp ----------------
  const int grp = lane >> 2, quad = lane & 3;
  pdl_wait_primary();  // x (and the residual) come from the preceding kernel
  if (warp < my_tiles) prefetch_residual<FUSED>(a, (int)blockIdx.x + warp * (int)gridDim.x, lane);
  if (FUSED && a.norm_w != nullptr) {  // RMSNorm factors over the consumer warps only (named barrier 1)
    if (a.ssq_in != nullptr) rms_from_ssq<CW>(a, s_rstd, warp, lane);
    else rms_factors<CW>(a, s_rstd, warp, lane);
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");
  }
  if (FUSED && a.norm_w != nullptr) stage_x<NT, CW * 32, true>(a, ks0, ks_n, M8, xs, s_rstd);
  else stage_x<NT, CW * 32, false>(a, ks0, ks_n, M8, xs);
  asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");

  const bool bvalid = grp < ((NT == 1) ? a.M : 8);
  int boff[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) boff[w] = (grp * 4 + quad) * 64 + ((w ^ xs_key(grp, quad)) << 4);
  constexpr int nt_stride = M8 * 256;
  constexpr int ks_stride = NT * nt_stride;

  bool ok = true;
  for (int it = warp; it < my_tiles; it += stages) {  // stage `warp` only; warps >= stages have none
    const int s = warp;
    const int tile = (int)blockIdx.x + it * (int)gridDim.x;
    if (ok) ok = mbar_wait_bounded(&full[s], (it / stages) & 1);
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
    if (ok) {
      const uint8_t* st = ring + (size_t)s * L.stage;
      const unsigned short* sc = reinterpret_cast<const unsigned short*>(st + L.sz_off);
      const unsigned short* ze = sc + 16 * ks_n;
      // stage row of tile row j: a clamped contiguous last tile starts `shift` rows early
      const int shift = contig ? tile * 16 - min(tile * 16, a.N - 16) : 0;
      const int ra = min(grp + shift, 15), rb2 = min(grp + 8 + shift, 15);
      const uint8_t* row_lo = st + ra * L.pitch + quad * 16;
      const uint8_t* row_hi = st + rb2 * L.pitch + quad * 16;
#pragma unroll 4
      for (int ks = 0; ks < ks_n; ++ks) {
        StreamUnit u;
        u.lo = *reinterpret_cast<const uint4*>(row_lo + ks * 64);
        u.hi = *reinterpret_cast<const uint4*>(row_hi + ks * 64);
        u.sz_lo = (uint32_t)sc[ra * ks_n + ks] | ((uint32_t)ze[ra * ks_n + ks] << 16);
        u.sz_hi = (uint32_t)sc[rb2 * ks_n + ks] | ((uint32_t)ze[rb2 * ks_n + ks] << 16);
        stream_compute<NT>(u, xs + ks * ks_stride, nt_stride, boff, bvalid, acc);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // the stage is free for the producer
    const int row0 = tile * 16;
    const int rows = min(16, a.N - row0);
    if (a.split == 1) {
      emit_warp_tile<FUSED, NT>(a, tile, acc, grp, quad);
    } else {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = grp + 8 * (e >> 1), m = nt * 8 + 2 * quad + (e & 1);
          if (r < rows && m < a.M) a.partial[((long long)blockIdx.y * a.M + m) * a.N + row0 + r] = acc[nt][e];
        }
    }
    if (a.split > 1) {  // last K range to arrive sums the partials (fixed order) and resets the counter
      __threadfence();
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) last = (atomicAdd(&a.counters[tile], 1u) == (unsigned)(a.split - 1)) ? 1u : 0u;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence();
        if constexpr (NT == 2) emit_partial_tile<FUSED>(a, tile, lane, PartialSum{a.partial + row0, a.M, a.N, a.split});
        else emit_tile<FUSED>(a, tile, lane, 32, PartialSum{a.partial + row0, a.M, a.N, a.split});
        __syncwarp();
        if (lane == 0) a.counters[tile] = 0u;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host side: planning and launch.
// ---------------------------------------------------------------------------
struct Plan {
  int kernel;      // LI4_KERNEL_CUDA_CORE / LI4_KERNEL_MMA
  int rt;          // 1 or 2 (16 or 32 rows per CTA)
  int nt;          // MMA: 1 (M <= 8) or 2
  bool scale_in_a; // MMA with groups < 128
  int n_ks;
  int split;
  int ks_per_split;
  int n_tiles;
  int grid_x;
  bool auto_grid;  // size grid_x from the kernel's occupancy at launch
  int sm;
  size_t smem;
  size_t ws_counters;  // bytes
  size_t ws_bytes;     // total
  bool stream_ksplit;  // LI4_KERNEL_STREAM: K-split mode
  int stages;          // LI4_KERNEL_BULK: shared-memory ring stages
  bool bulk_contig;    // LI4_KERNEL_BULK: tiles move as three contiguous copies (set at launch from the strides)
  int slots;           // LI4_KERNEL_SLAB: warps sharing one tile's ksteps (stages = tiles per CTA);
                       // LI4_KERNEL_RING: 16-row tiles per stage
  int pitch;           // LI4_KERNEL_SLAB / RING: bytes between packed rows of a stage
};

static inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Shared memory one slab CTA may take: leaves room for the next launch's CTA on the same SM only
// up to about half of the SM's 228 KB, but a larger slab still beats the other kernels.
constexpr size_t kSlabSmemMax = 200 * 1024;

// Launch shape of the slab kernel (li4_slab.cu), or false when the problem does not fit it:
// K ranges of all K unless the staged x would exceed 32 KB (64 KB at M > 8), at most one CTA per
// SM per K range, every CTA's tiles resident in shared memory at once.
static bool slab_shape(int64_t M, int64_t N, int64_t K, int sm, int split_req, int max_ctas, Plan* p) {
  const int n_ks = (int)(K / 128);
  const int nt = (M <= 8) ? 1 : 2;
  const int m8 = (nt == 1) ? (int)M : 8;
  const size_t x_cap = (nt == 1) ? 32768 : 65536;
  int split = 1;
  if (split_req > 0) {
    if (n_ks % split_req != 0) return false;
    split = split_req;
  } else {
    while ((size_t)(n_ks / split) * nt * m8 * 256 > x_cap && n_ks % (2 * split) == 0) split *= 2;
    if ((size_t)(n_ks / split) * nt * m8 * 256 > x_cap) return false;
  }
  const int ks = n_ks / split;
  const int n_tiles = (int)((N + 15) / 16);
  int gx = std::max(1, sm / split);
  if (max_ctas > 0) gx = std::max(1, std::min(gx, max_ctas / split));
  gx = std::min(gx, n_tiles);
  const int tiles_max = (n_tiles + gx - 1) / gx;
  int slots = 1;
  while (slots < 8 && ks % (2 * slots) == 0) slots *= 2;
  const int pitch = ks * 64 + 64;  // rows grp and grp + 1 of a quarter-warp's reads on distinct banks
  const size_t smem = slab_smem_bytes((int)M, nt, ks, tiles_max, slots, pitch);
  if (tiles_max > kSlabMaxTiles || smem > kSlabSmemMax) return false;
  p->kernel = LI4_KERNEL_SLAB;
  p->rt = 1;
  p->nt = nt;
  p->scale_in_a = false;
  p->n_ks = n_ks;
  p->split = split;
  p->ks_per_split = ks;
  p->n_tiles = n_tiles;
  p->grid_x = gx;
  p->auto_grid = false;
  p->sm = sm;
  p->smem = smem;
  p->stream_ksplit = false;
  p->stages = tiles_max;
  p->slots = slots;
  p->pitch = pitch;
  return true;
}

// Launch shape of the ring kernel (li4_ring.cu), or false when the problem does not fit it:
// group 128, M <= 8, K a multiple of 1024 with the staged x (M x K fp16) within 64 KiB, one K
// range; T = rows_req / 16 tiles per stage (1, 2 or 4; 0 takes the first of 4, 2, 1 that gives
// every consumer warp a kstep and two stages room), as many stages as fit next to the staged x
// (2 at least), one CTA per SM (max_ctas caps it) and never more CTAs than stage units.
static bool ring_fits(int64_t M, int ks, int T) {
  if ((T != 1 && T != 2 && T != 4) || (ks * T) % kRingWarps != 0) return false;
  const int stage = ring_stage_bytes(ks, T, ks * 64 + 64);
  return ring_smem_bytes((int)M, ks, 2, stage) <= kRingSmemCap;
}

static bool ring_shape(int64_t M, int64_t N, int64_t K, int sm, int rows_req, int max_ctas, Plan* p) {
  if (M < 1 || M > 8 || K <= 0 || K % 1024 != 0 || M * K * 2 > 65536 || rows_req % 16 != 0) return false;
  const int ks = (int)(K / 128);
  int T = rows_req / 16;
  if (rows_req == 0) {
    for (int t : {4, 2, 1})
      if (ring_fits(M, ks, t)) { T = t; break; }
  }
  if (!ring_fits(M, ks, T)) return false;
  const int pitch = ks * 64 + 64;
  const int stage = ring_stage_bytes(ks, T, pitch);
  const size_t fixed = ring_smem_bytes((int)M, ks, 0, stage);
  const int n_tiles = (int)((N + 15) / 16);
  const int n_su = (n_tiles + T - 1) / T;
  int gx = std::min(sm, n_su);
  if (max_ctas > 0) gx = std::max(1, std::min(gx, max_ctas));
  const int per_cta = (n_su + gx - 1) / gx;
  int stages = (int)std::min<size_t>(kRingMaxStages, (kRingSmemCap - fixed) / stage);
  stages = std::max(2, std::min(stages, per_cta));
  p->kernel = LI4_KERNEL_RING;
  p->rt = 1;
  p->nt = 1;
  p->scale_in_a = false;
  p->n_ks = ks;
  p->split = 1;
  p->ks_per_split = ks;
  p->n_tiles = n_tiles;
  p->grid_x = gx;
  p->auto_grid = false;
  p->sm = sm;
  p->smem = ring_smem_bytes((int)M, ks, stages, stage);
  p->stream_ksplit = false;
  p->stages = stages;
  p->slots = T;
  p->pitch = pitch;
  p->ws_counters = 0;
  p->ws_bytes = 0;
  return true;
}

static int make_plan(int64_t M, int64_t N, int64_t K, int64_t group, int sm, int kernel_req, int rows_req,
                     int split_req, int max_ctas, Plan* p, bool fused = false) {
  if (M < 1 || M > LI4_MAX_M)
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear: M=%lld outside 1..%d", (long long)M, LI4_MAX_M);
  if (N < 1) return set_error(LI4_ERR_INVALID_ARG, "int4_linear: N=%lld < 1", (long long)N);
  if (K < 0 || K % 128 != 0)
    return set_error(LI4_ERR_UNSUPPORTED, "int4_linear: K=%lld must be a multiple of 128", (long long)K);
  if (!is_pow2(group) || group < 32 || (K > 0 && K % group != 0))
    return set_error(LI4_ERR_UNSUPPORTED,
                     "int4_linear: group_size=%lld must be a power of two >= 32 dividing K=%lld", (long long)group,
                     (long long)K);
  if (N > (int64_t(1) << 30) || K > (int64_t(1) << 24))
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear: N=%lld K=%lld too large", (long long)N, (long long)K);
  if (sm <= 0) sm = 148;

  int kernel = kernel_req;
  // (The slab and register-rows families are taken only when forced: in graphs of back-to-back
  // launches on B200 they measured slower than the choices below at every decode shape, e.g.
  // q_proj at M = 1 2.73 / 3.34 against 2.41 us, gate_proj 5.70 / 7.35 against 4.44 us.)
  if (kernel == LI4_KERNEL_AUTO) {
    // By a measured B200 sweep of every family and split over the Llama-3.2-1B shapes at
    // M = 1..16 (graphs of back-to-back launches, weights streaming from HBM): tile
    // streaming when every warp slot gets several 16-row x 2048-k tiles (lm_head-sized N)
    // at M <= 8; the bulk-copy ring when the 16-row tiles alone give each SM two or more
    // at M >= 2 (gate / up / fused gate-up, lm_head at M = 16) or four or more at M = 1
    // (fused gate-up: 6.47 against 8.91 us); streaming warps for everything narrower
    // (q / k / v / o / fused qkv / down at every M: k_proj at M = 8 3.82 against 6.85 us
    // on the bulk ring, down_proj at M = 2 7.0 against 10.9 us); CUDA-core / MMA kernels
    // for groups below 128.  Launches with a prologue or epilogue keep the bulk ring for
    // 2 <= M <= 8 and, at M > 8, wherever the 2048-k tiles give each SM two or more: the
    // streaming kernel's fused variants spill at M > 8, and the fused decode step at batch
    // 16 measured 0.97 ms with these choices against 1.04 ms with the plain ones.
    const int64_t tiles = (N + 15) / 16;
    const int64_t tiles_2048 = tiles * std::max<int64_t>(1, K / 2048);
    const bool bulk_plain = (M >= 2 && tiles >= 2LL * sm) || tiles >= 4LL * sm;
    const bool bulk_fused = (M >= 2 && M <= 8) || tiles_2048 >= 4LL * sm || (M > 8 && tiles_2048 >= 2LL * sm);
    // Long K over few row tiles (down_proj: 2048 x 8192) at M = 1 and, without a prologue or
    // epilogue, M <= 4: the shared-memory ring with one 16-row x 8192-k stage per CTA and no
    // split-K (M = 1 5.4 against 6.4 us on the streaming warps, M = 2 5.6 against 7.0, M = 4 6.9
    // against 8.5).  Everywhere else the ring measured slower (lm_head 36.6 against 33.7 us).
    Plan rp = {};
    const bool ring_long_k = group == 128 && K >= 4096 && tiles <= sm && (M == 1 || (!fused && M <= 4)) &&
                             split_req <= 1 && rows_req == 0 && ring_shape(M, N, K, sm, 0, max_ctas, &rp);
    if (group == 128 && K > 0 && K % 2048 == 0 && tiles_2048 >= 32LL * sm && M <= 8) kernel = LI4_KERNEL_TILE;
    else if (ring_long_k) kernel = LI4_KERNEL_RING;
    else if (group == 128 && K > 0 && K % 1024 == 0 && (fused ? bulk_fused : bulk_plain))
      kernel = LI4_KERNEL_BULK;
    else if (group >= 128 && K > 0) kernel = LI4_KERNEL_STREAM;
    else kernel = (M <= 8) ? LI4_KERNEL_CUDA_CORE : LI4_KERNEL_MMA;
  }
  if (fused && kernel != LI4_KERNEL_STREAM && kernel != LI4_KERNEL_TILE && kernel != LI4_KERNEL_BULK &&
      kernel != LI4_KERNEL_SLAB && kernel != LI4_KERNEL_ROWS && kernel != LI4_KERNEL_RING)
    return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_fused: fused prologues / epilogues run on the streaming-warp, "
                     "tile, bulk-copy, slab and ring kernels (group_size >= 128)");
  if (kernel == LI4_KERNEL_CUDA_CORE && M > 8)
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear: CUDA-core kernel takes M <= 8 (M=%lld)", (long long)M);
  if (kernel == LI4_KERNEL_STREAM && (group < 128 || K == 0))
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear: the streaming kernel needs group_size >= 128 and K > 0");
  if (kernel == LI4_KERNEL_TILE && (group != 128 || K == 0 || (K / 128) % kTileKs != 0))
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear: the tile kernel needs group_size 128 and K a multiple of %d",
                     kTileKs * 128);
  if (kernel == LI4_KERNEL_BULK && (group != 128 || K == 0 || (K / 128) % 8 != 0))
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear: the bulk-copy kernel needs group_size 128 and K a multiple "
                     "of 1024");
  if (kernel < LI4_KERNEL_CUDA_CORE || kernel > LI4_KERNEL_RING)
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear: unknown kernel %d", kernel);
  if (kernel == LI4_KERNEL_RING) {
    if (group != 128 || split_req > 1 || !ring_shape(M, N, K, sm, rows_req, max_ctas, p))
      return set_error(LI4_ERR_UNSUPPORTED, "int4_linear: M=%lld N=%lld K=%lld (rows %d, split %d) does not fit the "
                       "ring kernel (group 128, M <= 8, K a multiple of 1024, M x K <= 32768, 16 / 32 / 64 rows per "
                       "stage, one K range)", (long long)M, (long long)N, (long long)K, rows_req, split_req);
    return LI4_OK;
  }
  if (kernel == LI4_KERNEL_ROWS) {
    if (M != 1 || group != 128 || (K != 1024 && K != 2048))
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear: the register-rows kernel takes M = 1, group_size 128 and "
                       "K = 1024 or 2048 (M=%lld K=%lld)", (long long)M, (long long)K);
    p->kernel = kernel;
    p->rt = 1;
    p->nt = 1;
    p->scale_in_a = false;
    p->n_ks = (int)(K / 128);
    p->split = 1;
    p->ks_per_split = p->n_ks;
    p->n_tiles = (int)((N + 15) / 16);
    p->grid_x = p->n_tiles;
    p->auto_grid = false;
    p->sm = sm;
    p->smem = 0;
    p->stream_ksplit = false;
    p->ws_counters = 0;
    p->ws_bytes = 0;
    return LI4_OK;
  }
  if (kernel == LI4_KERNEL_SLAB) {
    if (group != 128 || K == 0)
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear: the slab kernel needs group_size 128 and K > 0");
    if (!slab_shape(M, N, K, sm, split_req, max_ctas, p))
      return set_error(LI4_ERR_UNSUPPORTED, "int4_linear: M=%lld N=%lld K=%lld (split %d) does not fit the slab "
                       "kernel (at most %d row tiles and %zu bytes of shared memory per CTA)", (long long)M,
                       (long long)N, (long long)K, split_req, kSlabMaxTiles, kSlabSmemMax);
    if (p->split > 1) {
      if ((size_t)p->n_tiles * sizeof(unsigned) > LI4_WORKSPACE_COUNTER_BYTES)
        return set_error(LI4_ERR_UNSUPPORTED, "int4_linear: N=%lld needs %d split-K row tiles, more than the %d "
                         "arrival counters of the workspace", (long long)N, p->n_tiles,
                         (int)(LI4_WORKSPACE_COUNTER_BYTES / sizeof(unsigned)));
      p->ws_counters = LI4_WORKSPACE_COUNTER_BYTES;
      p->ws_bytes = p->ws_counters + (size_t)p->split * M * N * sizeof(float);
    } else {
      p->ws_counters = 0;
      p->ws_bytes = 0;
    }
    return LI4_OK;
  }
  p->stream_ksplit = false;
  p->kernel = kernel;
  p->nt = (M <= 8) ? 1 : 2;
  p->scale_in_a = group < 128;

  if (rows_req == 16) p->rt = 1;
  else if (rows_req == 32) p->rt = 2;
  else if (rows_req == 0) p->rt = (N >= 4096) ? 2 : 1;
  else return set_error(LI4_ERR_INVALID_ARG, "int4_linear: rows_per_cta=%d must be 0, 16 or 32", rows_req);
  const int rows = 16 * p->rt;
  p->n_tiles = (int)((N + rows - 1) / rows);
  p->n_ks = (int)(K / 128);

  // K range of one CTA: 16 ksteps, or (streaming warps) as many as keep the staged x within 32 KiB
  int max_ks = kMaxKsPerCta;
  if (kernel == LI4_KERNEL_STREAM) max_ks = std::max(kMaxKsPerCta, 32768 / (p->nt * (p->nt == 1 ? (int)M : 8) * 256));
  int split = 1;
  if (split_req > 0) {
    split = split_req;
    if (p->n_ks == 0 || p->n_ks % split != 0 || p->n_ks / split > max_ks)
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear: split=%d must divide K/128=%d into ranges of <= %d",
                       split, p->n_ks, max_ks);
  } else if (p->n_ks > 0) {
    // smallest divisor of n_ks giving K ranges of at most kMaxKsPerCta ksteps
    while (p->n_ks % split != 0 || p->n_ks / split > kMaxKsPerCta) ++split;
    // more K ranges while the row tiles alone leave SMs idle and every warp keeps >= 1 kstep
    while ((int64_t)p->n_tiles * split < 2 * sm && p->n_ks % (2 * split) == 0 &&
           p->n_ks / (2 * split) >= kWarps)
      split *= 2;
  }
  if (kernel == LI4_KERNEL_STREAM) {  // 16-row tiles; rows mode for many tiles, K-split mode for few
    p->rt = 1;
    p->n_tiles = (int)((N + 15) / 16);
    if (split_req <= 0) {
      split = 1;
      while (p->n_ks % split != 0 || p->n_ks / split > max_ks) ++split;
    }
    p->stream_ksplit = (int64_t)p->n_tiles < 4LL * sm && p->n_ks / split >= kStreamWarps;
    // more K ranges while the CTAs stay resident (two per SM) and every warp keeps >= 2 ksteps
    if (split_req <= 0 && p->stream_ksplit)
      while ((int64_t)p->n_tiles * split * 2 <= 2LL * sm && p->n_ks % (2 * split) == 0 &&
             p->n_ks / (2 * split) >= 2 * kStreamWarps)
        split *= 2;
  }
  if (kernel == LI4_KERNEL_TILE) {  // K ranges of exactly kTileKs ksteps; 16 or 32 rows per warp tile
    if (split_req > 0 && split_req != p->n_ks / kTileKs)
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear: the tile kernel takes split=%d for K=%lld",
                       p->n_ks / kTileKs, (long long)K);
    split = p->n_ks / kTileKs;
    p->rt = (rows_req == 32) ? 2 : 1;
    p->n_tiles = (int)((N + 16 * p->rt - 1) / (16 * p->rt));
  }
  if (kernel == LI4_KERNEL_BULK) {  // 16-row tiles of K ranges of 16 (or 8) ksteps through a shared-memory ring
    p->rt = 1;
    p->n_tiles = (int)((N + 15) / 16);
    int ks = (p->n_ks % 16 == 0) ? 16 : 8;
    if (split_req > 0) {
      if (p->n_ks % split_req != 0 || (p->n_ks / split_req != 16 && p->n_ks / split_req != 8))
        return set_error(LI4_ERR_INVALID_ARG, "int4_linear: the bulk-copy kernel takes K ranges of 8 or 16 ksteps "
                         "(split=%d, K/128=%d)", split_req, p->n_ks);
      ks = p->n_ks / split_req;
    } else if (ks == 16 && (int64_t)p->n_tiles * (p->n_ks / 16) * 2 <= sm) {
      ks = 8;  // few tiles: shorter K ranges put more CTAs to work
    }
    split = p->n_ks / ks;
  }
  p->split = split;
  p->ks_per_split = (p->n_ks == 0) ? 0 : p->n_ks / split;

  p->sm = sm;
  p->auto_grid = (max_ctas <= 0);
  const int cap = (max_ctas > 0) ? max_ctas : sm * 4;
  int gx = cap / split;
  if (gx < 1) gx = 1;
  if (gx > p->n_tiles) gx = p->n_tiles;
  p->grid_x = gx;

  const int m8 = (p->kernel == LI4_KERNEL_CUDA_CORE) ? (int)M : (p->nt == 1 ? (int)M : 8);
  const int nt = (p->kernel == LI4_KERNEL_CUDA_CORE) ? 1 : p->nt;
  const int cols = 8 * nt;
  p->smem = round_up((size_t)p->ks_per_split * nt * m8 * 256, 128) + (size_t)kWarps * rows * cols * sizeof(float);
  if (kernel == LI4_KERNEL_STREAM) {
    p->smem = round_up((size_t)p->ks_per_split * p->nt * (p->nt == 1 ? (int)M : 8) * 256, 128) +
              (p->stream_ksplit ? (size_t)2 * kStreamWarps * 16 * 8 * p->nt * sizeof(float) : 0);
    int gx = p->stream_ksplit ? p->n_tiles : (p->n_tiles + kStreamWarps - 1) / kStreamWarps;
    if (max_ctas > 0 && gx > max_ctas / split) gx = max_ctas / split > 0 ? max_ctas / split : 1;
    p->grid_x = gx;  // capped by occupancy at launch
  }
  if (kernel == LI4_KERNEL_BULK) {
    const int max_stages = (p->nt == 1) ? kBulkMaxStages : 8;
    int gx = std::max(1, sm / split);
    if (max_ctas > 0) gx = std::max(1, std::min(gx, max_ctas / split));
    gx = std::min(gx, p->n_tiles);
    const int per_cta = (p->n_tiles + gx - 1) / gx;
    p->stages = std::min(max_stages, per_cta);
    p->grid_x = gx;
    const BulkLayout L = bulk_layout(p->ks_per_split, false);  // the padded layout: an upper bound
    p->smem = (size_t)p->stages * L.stage + (size_t)p->ks_per_split * p->nt * 8 * 256 +
              2 * kBulkMaxStages * sizeof(uint64_t);
  }
  if (kernel == LI4_KERNEL_TILE) {
    p->smem = (size_t)kTileKs * p->nt * 8 * 256;
    int gx = (p->n_tiles + kStreamWarps - 1) / kStreamWarps;
    if (max_ctas > 0 && gx > max_ctas / split) gx = max_ctas / split > 0 ? max_ctas / split : 1;
    p->grid_x = gx;  // capped by occupancy at launch
  }

  if (split > 1) {
    // Counters live in a fixed region at the start of the workspace that no
    // launch ever uses for partial sums, so they stay zero between launches
    // of different shapes sharing the workspace.
    if ((size_t)p->n_tiles * sizeof(unsigned) > LI4_WORKSPACE_COUNTER_BYTES)
      return set_error(LI4_ERR_UNSUPPORTED, "int4_linear: N=%lld needs %d split-K row tiles, more than the %d "
                       "arrival counters of the workspace", (long long)N, p->n_tiles,
                       (int)(LI4_WORKSPACE_COUNTER_BYTES / sizeof(unsigned)));
    p->ws_counters = LI4_WORKSPACE_COUNTER_BYTES;
    p->ws_bytes = p->ws_counters + (size_t)split * M * N * sizeof(float);
  } else {
    p->ws_counters = 0;
    p->ws_bytes = 0;
  }
  return LI4_OK;
}

// CTAs of `kernel` that fit on one SM with `smem` bytes of dynamic shared
// memory (cached; the answer depends only on the kernel and smem size).
template <typename KernelT>
static int ctas_per_sm(KernelT kernel, size_t smem) {
  struct Entry { const void* fn; size_t smem; int dev; int n; };
  static std::mutex mu;
  static std::vector<Entry> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& e : cache)
    if (e.fn == (const void*)kernel && e.smem == smem && e.dev == dev) return e.n;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreads, smem) != cudaSuccess || n < 1) n = 1;
  cache.push_back(Entry{(const void*)kernel, smem, dev, n});
  return n;
}

// Raise the kernel's dynamic shared memory limit once per (kernel, device)
// to the largest size requested so far, so launches after the first (for
// example inside CUDA-graph capture) make no attribute call.
template <typename KernelT>
static int ensure_smem_limit(KernelT kernel, size_t smem) {
  // the kernels also hold a little static shared memory (RMSNorm partials): raise the limit well
  // before dynamic + static reaches the 48 KiB default
  if (smem + 4096 <= 48 * 1024) return LI4_OK;
  struct Entry { const void* fn; int dev; size_t limit; };
  static std::mutex mu;
  static std::vector<Entry> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (Entry& e : cache)
    if (e.fn == (const void*)kernel && e.dev == dev) {
      if (e.limit >= smem) return LI4_OK;
      const int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                                "int4_linear: cudaFuncSetAttribute");
      if (rc == LI4_OK) e.limit = smem;
      return rc;
    }
  const int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "int4_linear: cudaFuncSetAttribute");
  if (rc == LI4_OK) cache.push_back(Entry{(const void*)kernel, dev, smem});
  return rc;
}

template <typename KernelT>
static int launch(KernelT kernel, const Plan& p, const GemvArgs& args, cudaStream_t stream) {
  int rc = ensure_smem_limit(kernel, p.smem);
  if (rc != LI4_OK) return rc;
  int grid_x = p.grid_x;
  if (p.auto_grid) {  // persistent grid: every CTA resident at once
    const int cap = ctas_per_sm(kernel, p.smem) * p.sm;
    grid_x = cap / p.split;
    if (grid_x < 1) grid_x = 1;
    if (grid_x > p.n_tiles) grid_x = p.n_tiles;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid_x, (unsigned)p.split, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, args), "int4_linear: kernel launch");
}

template <int M>
static int launch_cc(const Plan& p, const GemvArgs& args, cudaStream_t s) {
  return p.rt == 1 ? launch(gemv_cc_kernel<M, 1>, p, args, s) : launch(gemv_cc_kernel<M, 2>, p, args, s);
}

template <typename KernelT>
static int launch_stream_kernel(KernelT kernel, const Plan& p, const GemvArgs& args, cudaStream_t stream) {
  int rc = ensure_smem_limit(kernel, p.smem);
  if (rc != LI4_OK) return rc;
  int occ = 0;
  {
    static std::mutex mu;
    struct Entry { const void* fn; size_t smem; int dev; int n; };
    static std::vector<Entry> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry& e : cache)
      if (e.fn == (const void*)kernel && e.smem == p.smem && e.dev == dev) occ = e.n;
    if (occ == 0) {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kStreamThreads, p.smem) != cudaSuccess || occ < 1)
        occ = 1;
      cache.push_back(Entry{(const void*)kernel, p.smem, dev, occ});
    }
  }
  int gx = p.grid_x;
  const int cap = occ * p.sm / p.split;
  if (gx > cap) gx = cap > 0 ? cap : 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)gx, (unsigned)p.split, 1);
  cfg.blockDim = dim3(kStreamThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, args), "int4_linear: streaming kernel launch");
}

template <typename KernelT>
static int launch_bulk_kernel(KernelT kernel, const Plan& p, const GemvArgs& args, cudaStream_t stream) {
  int rc = ensure_smem_limit(kernel, p.smem);
  if (rc != LI4_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid_x, (unsigned)p.split, 1);
  cfg.blockDim = dim3(bulk_threads(p.nt), 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // contiguous tiles: one K range, rows back to back in packed / scale / zero, and N >= 16
  const int contig = (p.split == 1 && args.spn == args.K / 2 && args.ssn == args.K / 128 && args.N >= 16) ? 1 : 0;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, args, p.stages, contig), "int4_linear: bulk-copy kernel launch");
}

static int launch_plan(const Plan& p, const GemvArgs& args, cudaStream_t s) {
  const bool fused = args.norm_w != nullptr || args.epi != LI4_EPI_STORE;
  if (p.kernel == LI4_KERNEL_RING)
    return launch_ring(args, fused, p.grid_x, p.slots, p.stages, p.pitch, p.smem, s);
  if (p.kernel == LI4_KERNEL_SLAB)
    return launch_slab(args, p.nt, fused, p.grid_x, p.stages, p.slots, p.pitch, p.smem, s);
  if (p.kernel == LI4_KERNEL_ROWS) return launch_rows(args, fused, s);
  if (p.kernel == LI4_KERNEL_BULK) {
    const int sel = (p.nt - 1) * 2 + (fused ? 1 : 0);
    switch (sel) {
      case 0: return launch_bulk_kernel(gemv_bulk_kernel<1, false>, p, args, s);
      case 1: return launch_bulk_kernel(gemv_bulk_kernel<1, true>, p, args, s);
      case 2: return launch_bulk_kernel(gemv_bulk_kernel<2, false>, p, args, s);
      default: return launch_bulk_kernel(gemv_bulk_kernel<2, true>, p, args, s);
    }
  }
  if (p.kernel == LI4_KERNEL_TILE) {
    const int sel = (p.nt - 1) * 4 + (p.rt - 1) * 2 + (fused ? 1 : 0);
    switch (sel) {
      case 0: return launch_stream_kernel(gemv_tile_kernel<1, 1, false>, p, args, s);
      case 1: return launch_stream_kernel(gemv_tile_kernel<1, 1, true>, p, args, s);
      case 2: return launch_stream_kernel(gemv_tile_kernel<1, 2, false>, p, args, s);
      case 3: return launch_stream_kernel(gemv_tile_kernel<1, 2, true>, p, args, s);
      case 4: return launch_stream_kernel(gemv_tile_kernel<2, 1, false>, p, args, s);
      case 5: return launch_stream_kernel(gemv_tile_kernel<2, 1, true>, p, args, s);
      case 6: return launch_stream_kernel(gemv_tile_kernel<2, 2, false>, p, args, s);
      default: return launch_stream_kernel(gemv_tile_kernel<2, 2, true>, p, args, s);
    }
  }
  if (p.kernel == LI4_KERNEL_STREAM && args.epi == LI4_EPI_ALLREDUCE_RESIDUAL) {
    // the all-reduce epilogue: its own instantiations, so the others keep their registers
    const int sel = (p.nt - 1) * 2 + (p.stream_ksplit ? 1 : 0);
    switch (sel) {
      case 0: return launch_stream_kernel(gemv_stream_kernel<1, false, true, true>, p, args, s);
      case 1: return launch_stream_kernel(gemv_stream_kernel<1, true, true, true>, p, args, s);
      case 2: return launch_stream_kernel(gemv_stream_kernel<2, false, true, true>, p, args, s);
      default: return launch_stream_kernel(gemv_stream_kernel<2, true, true, true>, p, args, s);
    }
  }
  if (p.kernel == LI4_KERNEL_STREAM) {
    const int sel = (p.nt - 1) * 4 + (p.stream_ksplit ? 2 : 0) + (fused ? 1 : 0);
    switch (sel) {
      case 0: return launch_stream_kernel(gemv_stream_kernel<1, false, false>, p, args, s);
      case 1: return launch_stream_kernel(gemv_stream_kernel<1, false, true>, p, args, s);
      case 2: return launch_stream_kernel(gemv_stream_kernel<1, true, false>, p, args, s);
      case 3: return launch_stream_kernel(gemv_stream_kernel<1, true, true>, p, args, s);
      case 4: return launch_stream_kernel(gemv_stream_kernel<2, false, false>, p, args, s);
      case 5: return launch_stream_kernel(gemv_stream_kernel<2, false, true>, p, args, s);
      case 6: return launch_stream_kernel(gemv_stream_kernel<2, true, false>, p, args, s);
      default: return launch_stream_kernel(gemv_stream_kernel<2, true, true>, p, args, s);
    }
  }
  if (p.kernel == LI4_KERNEL_CUDA_CORE) {
    switch (args.M) {
      case 1: return launch_cc<1>(p, args, s);
      case 2: return launch_cc<2>(p, args, s);
      case 3: return launch_cc<3>(p, args, s);
      case 4: return launch_cc<4>(p, args, s);
      case 5: return launch_cc<5>(p, args, s);
      case 6: return launch_cc<6>(p, args, s);
      case 7: return launch_cc<7>(p, args, s);
      case 8: return launch_cc<8>(p, args, s);
      default: return set_error(LI4_ERR_INVALID_ARG, "int4_linear: CUDA-core kernel M=%d", args.M);
    }
  }
  const int sel = (p.rt - 1) * 4 + (p.nt - 1) * 2 + (p.scale_in_a ? 1 : 0);
  switch (sel) {
    case 0: return launch(gemv_mma_kernel<1, 1, false>, p, args, s);
    case 1: return launch(gemv_mma_kernel<1, 1, true>, p, args, s);
    case 2: return launch(gemv_mma_kernel<1, 2, false>, p, args, s);
    case 3: return launch(gemv_mma_kernel<1, 2, true>, p, args, s);
    case 4: return launch(gemv_mma_kernel<2, 1, false>, p, args, s);
    case 5: return launch(gemv_mma_kernel<2, 1, true>, p, args, s);
    case 6: return launch(gemv_mma_kernel<2, 2, false>, p, args, s);
    default: return launch(gemv_mma_kernel<2, 2, true>, p, args, s);
  }
}

static bool aligned4(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 3u) == 0; }

// Preconditions of the fused prologue / epilogues (li4_fusion).
static int check_fusion(const li4_fusion& f, int64_t M, int64_t N, int64_t K) {
  if (f.sumsq_out != nullptr && (f.epilogue != LI4_EPI_RESIDUAL || !aligned4(f.sumsq_out)))
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: sumsq_out goes with the residual epilogue (4-byte "
                     "aligned, [ceil(N/16)][M] floats)");
  if (f.sumsq_in != nullptr &&
      (f.norm_weight == nullptr || !aligned4(f.sumsq_in) || f.sumsq_tiles != (K + 15) / 16))
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: sumsq_in needs the RMSNorm prologue and "
                     "sumsq_tiles = ceil(K/16) = %lld (got %lld)", (long long)((K + 15) / 16),
                     (long long)f.sumsq_tiles);
  if (f.norm_weight != nullptr) {
    if (!aligned16(f.norm_weight))
      return set_error(LI4_ERR_ALIGNMENT, "int4_linear_fused: norm_weight must be 16-byte aligned");
    if (!(f.norm_eps >= 0.f)) return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: norm_eps must be >= 0");
  }
  switch (f.epilogue) {
    case LI4_EPI_STORE:
    case LI4_EPI_STORE_F32:
      return LI4_OK;
    case LI4_EPI_RESIDUAL:
      if (!f.residual || f.stride_rm < N || (reinterpret_cast<uintptr_t>(f.residual) & 1u))
        return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: residual epilogue needs a residual [M, N] "
                         "(row stride >= N)");
      return LI4_OK;
    case LI4_EPI_SWIGLU:
      if (N % 16 != 0)
        return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: SwiGLU pairs need N %% 16 == 0 (N=%lld)",
                         (long long)N);
      return LI4_OK;
    case LI4_EPI_ALLREDUCE_RESIDUAL: {
      if (!f.residual || f.stride_rm < N || (reinterpret_cast<uintptr_t>(f.residual) & 1u) || N % 16 != 0)
        return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: the all-reduce epilogue needs a residual [M, N] "
                         "(row stride >= N) and N %% 16 == 0 (N=%lld)", (long long)N);
      if (f.ar_world < 1 || f.ar_world > 8 || f.ar_rank < 0 || f.ar_rank >= f.ar_world || !f.ar_recv ||
          !f.ar_epochs || !aligned4(f.ar_epochs))
        return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: all-reduce epilogue: world=%d rank=%d (1..8 ranks), "
                         "receive buffers and a 4-byte aligned epoch array", f.ar_world, f.ar_rank);
      const size_t need = (size_t)f.ar_world * (size_t)(N / 16) * (size_t)M * 8 * sizeof(unsigned long long);
      if (f.ar_recv_bytes < need)
        return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: all-reduce receive buffers of %zu bytes, %zu needed "
                         "(world x N/16 x M x 8 words of 8 bytes)", f.ar_recv_bytes, need);
      for (int r = 0; r < f.ar_world; ++r)
        if (!f.ar_recv[r] || (reinterpret_cast<uintptr_t>(f.ar_recv[r]) & 7u))
          return set_error(LI4_ERR_ALIGNMENT, "int4_linear_fused: all-reduce receive buffer %d is null or not 8-byte "
                           "aligned", r);
      if (f.sumsq_out != nullptr || f.argmax_out != nullptr)
        return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_fused: the all-reduce epilogue takes neither sumsq_out nor "
                         "the fused argmax");
      return LI4_OK;
    }
    case LI4_EPI_QKV_ROPE: {
      const int64_t v_rows = N - f.q_rows - f.k_rows;
      if (f.head_dim < 2 || f.head_dim % 2 != 0 || f.q_rows < 0 || f.k_rows <= 0 || f.q_rows % 16 != 0 ||
          f.k_rows % 16 != 0 || f.q_rows % f.head_dim != 0 || f.k_rows % f.head_dim != 0 || v_rows != f.k_rows)
        return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: QKV epilogue needs q_rows, k_rows multiples of "
                         "16 and of head_dim, and N = q_rows + 2 k_rows (N=%lld q=%lld k=%lld head_dim=%lld)",
                         (long long)N, (long long)f.q_rows, (long long)f.k_rows, (long long)f.head_dim);
      if (!f.pos || !f.rope_cos || !f.rope_sin || (f.q_rows > 0 && !f.q_out) || !f.cache_k || !f.cache_v)
        return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: QKV epilogue needs pos, rope_cos/sin, q_out and "
                         "cache_k/v");
      if (f.rope_stride < f.head_dim / 2 || f.stride_qm < f.q_rows || f.cache_stride_s < f.k_rows ||
          f.cache_stride_b < f.cache_stride_s)
        return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: QKV epilogue strides smaller than the rows");
      if (!aligned4(f.cache_k) || !aligned4(f.cache_v) || (f.q_rows > 0 && !aligned4(f.q_out)) ||
          f.stride_qm % 2 != 0 || f.cache_stride_b % 2 != 0 || f.cache_stride_s % 2 != 0)
        return set_error(LI4_ERR_ALIGNMENT, "int4_linear_fused: q_out / cache rows must be 4-byte aligned "
                         "(pairs are stored as half2)");
      (void)M;
      (void)K;
      return LI4_OK;
    }
    default:
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: unknown epilogue %d", f.epilogue);
  }
}

int prepare_linear(const void* x, const void* packed, const void* scale, const void* zero, void* y, int64_t M,
                   int64_t N, int64_t K, int64_t group, int64_t sxm, int64_t spn, int64_t ssn, int64_t sym,
                   const li4_fusion* f, GemvArgs* out) {
  const bool fused = f != nullptr && (f->norm_weight != nullptr || f->epilogue != LI4_EPI_STORE);
  const int epi = f ? f->epilogue : LI4_EPI_STORE;
  // columns of y: N, N/2 for SwiGLU pairs, none for the QKV epilogue (outputs go to q_out and the cache)
  const int64_t y_cols = epi == LI4_EPI_SWIGLU ? N / 2 : (epi == LI4_EPI_QKV_ROPE ? 0 : N);
  if (fused) {
    const int rc = check_fusion(*f, M, N, K);
    if (rc != LI4_OK) return rc;
  }
  if (!x || !packed || !scale || !zero || (!y && y_cols > 0))
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear: null tensor pointer");
  if (sxm < K || sym < y_cols || spn < K / 2 || ssn < (K > 0 ? K / group : 0))
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear: row strides (x %lld, packed %lld, scale %lld, y %lld) "
                     "smaller than the rows", (long long)sxm, (long long)spn, (long long)ssn, (long long)sym);
  if (!aligned16(packed) || spn % 16 != 0)
    return set_error(LI4_ERR_ALIGNMENT, "int4_linear: packed rows must start on 16-byte boundaries "
                     "(base %p, row stride %lld bytes)", packed, (long long)spn);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(scale) |
       reinterpret_cast<uintptr_t>(zero)) & 1u)
    return set_error(LI4_ERR_ALIGNMENT, "int4_linear: fp16 tensors must be 2-byte aligned");
  if (epi == LI4_EPI_STORE_F32 && (reinterpret_cast<uintptr_t>(y) & 3u))
    return set_error(LI4_ERR_ALIGNMENT, "int4_linear_fused: an fp32 output must be 4-byte aligned");
  if (f && f->argmax_out) {
    if (epi != LI4_EPI_STORE_F32 || !f->argmax_scratch || f->argmax_stride < 1)
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear_fused: the fused argmax takes LI4_EPI_STORE_F32, an "
                       "argmax_scratch and argmax_stride >= 1");
    if ((reinterpret_cast<uintptr_t>(f->argmax_out) | reinterpret_cast<uintptr_t>(f->argmax_scratch)) & 7u)
      return set_error(LI4_ERR_ALIGNMENT, "int4_linear_fused: argmax_out / argmax_scratch must be 8-byte aligned");
  }
  GemvArgs args = {};
  if (fused) {
    args.norm_w = static_cast<const __half*>(f->norm_weight);
    args.norm_eps = f->norm_eps;
    args.epi = epi;
    args.res = static_cast<const __half*>(f->residual);
    args.srm = f->stride_rm;
    args.q_rows = (int)f->q_rows;
    args.k_rows = (int)f->k_rows;
    args.head_dim = (int)f->head_dim;
    args.pos = reinterpret_cast<const long long*>(f->pos);
    args.rope_cos = f->rope_cos;
    args.rope_sin = f->rope_sin;
    args.rope_stride = f->rope_stride;
    args.q_out = static_cast<__half*>(f->q_out);
    args.sqm = f->stride_qm;
    args.cache_k = static_cast<__half*>(f->cache_k);
    args.cache_v = static_cast<__half*>(f->cache_v);
    args.cache_sb = f->cache_stride_b;
    args.cache_ss = f->cache_stride_s;
    args.ssq_out = f->sumsq_out;
    args.ssq_in = f->sumsq_in;
    args.ssq_tiles = (int)f->sumsq_tiles;
    if (epi == LI4_EPI_ALLREDUCE_RESIDUAL) {
      for (int r = 0; r < f->ar_world; ++r) args.ar_recv[r] = static_cast<unsigned long long*>(f->ar_recv[r]);
      args.ar_epochs = f->ar_epochs;
      args.ar_words = (N / 16) * M * 8;
      args.ar_world = f->ar_world;
      args.ar_rank = f->ar_rank;
    }
    if (f->argmax_out != nullptr) {
      args.am_keys = static_cast<unsigned long long*>(f->argmax_scratch);
      args.am_count = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(f->argmax_scratch) + 8 * M);
      args.am_out = reinterpret_cast<long long*>(f->argmax_out);
      args.am_stride = f->argmax_stride;
    }
  }
  args.x = static_cast<const __half*>(x);
  args.packed = static_cast<const uint8_t*>(packed);
  args.scale = static_cast<const __half*>(scale);
  args.zero = static_cast<const __half*>(zero);
  args.y = static_cast<__half*>(y);
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.log2_group = ilog2(group);
  args.sxm = sxm;
  args.spn = spn;
  args.ssn = ssn;
  args.sym = sym;
  *out = args;
  return LI4_OK;
}

static int int4_linear_impl(const void* x, const void* packed, const void* scale, const void* zero, void* y,
                            int64_t M, int64_t N, int64_t K, int64_t group, int64_t sxm, int64_t spn, int64_t ssn,
                            int64_t sym, void* workspace, size_t workspace_bytes, void* stream, int kernel,
                            int rows_req, int split_req, int max_ctas, const li4_fusion* f = nullptr) {
  Plan p = {};
  const int sm = current_sm_count();
  const bool fused = f != nullptr && (f->norm_weight != nullptr || f->epilogue != LI4_EPI_STORE);
  int rc = make_plan(M, N, K, group, sm, kernel, rows_req, split_req, max_ctas, &p, fused);
  if (rc != LI4_OK) return rc;
  if (p.kernel == LI4_KERNEL_ROWS &&
      (!aligned16(x) || (f != nullptr && (f->norm_weight != nullptr || f->argmax_out != nullptr)))) {
    // the register-rows kernel reads x in 16-byte pieces and has no RMSNorm prologue or argmax
    if (kernel != LI4_KERNEL_AUTO)
      return set_error(LI4_ERR_UNSUPPORTED, "int4_linear: the register-rows kernel needs a 16-byte aligned x and "
                       "no RMSNorm prologue or fused argmax");
    rc = make_plan(M, N, K, group, sm, LI4_KERNEL_STREAM, rows_req, split_req, max_ctas, &p, fused);
    if (rc != LI4_OK) return rc;
  }
  if (f != nullptr && f->epilogue == LI4_EPI_ALLREDUCE_RESIDUAL && p.kernel != LI4_KERNEL_STREAM) {
    // the all-reduce epilogue runs on the streaming-warp kernel
    if (kernel != LI4_KERNEL_AUTO)
      return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_fused: the all-reduce epilogue runs on the streaming-warp "
                       "kernel only");
    rc = make_plan(M, N, K, group, sm, LI4_KERNEL_STREAM, rows_req, split_req, max_ctas, &p, fused);
    if (rc != LI4_OK) return rc;
  }
  if (kernel == LI4_KERNEL_AUTO && f != nullptr && f->argmax_out != nullptr && p.kernel != LI4_KERNEL_TILE &&
      p.kernel != LI4_KERNEL_RING && M <= 8) {
    // the fused greedy argmax runs on the tile kernel at M <= 8; where that does not take the
    // problem, the check below reports the fusion as unsupported (callers then run the argmax
    // separately)
    Plan tp = {};
    if (make_plan(M, N, K, group, sm, LI4_KERNEL_TILE, rows_req, split_req, max_ctas, &tp, fused) == LI4_OK) p = tp;
  }
  GemvArgs args = {};
  rc = prepare_linear(x, packed, scale, zero, y, M, N, K, group, sxm, spn, ssn, sym, f, &args);
  if (rc != LI4_OK) return rc;
  if (p.kernel == LI4_KERNEL_TILE && ((N - 1) * spn + K / 2 > (int64_t)UINT32_MAX ||
                                      (N - 1) * ssn + K / group > (int64_t)UINT32_MAX)) {
    // the tile kernel addresses rows with 32-bit offsets
    if (kernel != LI4_KERNEL_AUTO)
      return set_error(LI4_ERR_UNSUPPORTED, "int4_linear: the tile kernel needs packed / scale offsets below 2^32");
    rc = make_plan(M, N, K, group, sm, LI4_KERNEL_STREAM, rows_req, split_req, max_ctas, &p, fused);
    if (rc != LI4_OK) return rc;
  }
  if (p.kernel == LI4_KERNEL_BULK && (!aligned16(scale) || !aligned16(zero) || ssn % 8 != 0)) {
    // the scale / zero rows move as 16-byte-aligned bulk copies
    if (kernel != LI4_KERNEL_AUTO)
      return set_error(LI4_ERR_ALIGNMENT, "int4_linear: the bulk-copy kernel needs 16-byte aligned scale / zero "
                       "rows (row stride %% 8 == 0)");
    rc = make_plan(M, N, K, group, sm, LI4_KERNEL_STREAM, rows_req, split_req, max_ctas, &p, fused);
    if (rc != LI4_OK) return rc;
  }
  if (p.kernel == LI4_KERNEL_RING &&
      (!aligned16(packed) || spn % 16 != 0 || !aligned16(scale) || !aligned16(zero) || ssn % 8 != 0)) {
    // packed rows and scale / zero rows move as 16-byte-aligned bulk copies
    if (kernel != LI4_KERNEL_AUTO)
      return set_error(LI4_ERR_ALIGNMENT, "int4_linear: the ring kernel needs 16-byte aligned packed, scale and "
                       "zero rows (packed row stride %% 16 == 0, scale row stride %% 8 == 0)");
    rc = make_plan(M, N, K, group, sm, LI4_KERNEL_STREAM, rows_req, split_req, max_ctas, &p, fused);
    if (rc != LI4_OK) return rc;
  }
  if (args.am_keys != nullptr && ((p.kernel != LI4_KERNEL_TILE && p.kernel != LI4_KERNEL_RING) || p.split != 1))
    return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_fused: the fused argmax runs on the tile and ring kernels "
                     "without a K split (lm_head-sized N at M <= 8); this launch plan has neither");
  if (p.ws_bytes > 0) {
    if (!workspace || workspace_bytes < p.ws_bytes)
      return set_error(LI4_ERR_WORKSPACE, "int4_linear: split-K (%d ranges) needs a %zu-byte zero-initialised "
                       "workspace, got %zu", p.split, p.ws_bytes, workspace ? workspace_bytes : (size_t)0);
    if (!aligned16(workspace)) return set_error(LI4_ERR_ALIGNMENT, "int4_linear: workspace must be 16-byte aligned");
  }
  args.n_tiles = p.n_tiles;
  args.split = p.split;
  args.ks_per_split = p.ks_per_split;
  args.counters = p.ws_bytes ? static_cast<unsigned*>(workspace) : nullptr;
  args.partial = p.ws_bytes ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + p.ws_counters) : nullptr;
  rc = launch_plan(p, args, static_cast<cudaStream_t>(stream));
  if (rc == LI4_OK) clear_error();
  return rc;
}

}  // namespace li4

extern "C" size_t li4_int4_linear_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t group_size, int sm_count) {
  li4::Plan p = {};
  const int sm = sm_count > 0 ? sm_count : li4::current_sm_count();
  if (li4::make_plan(M, N, K, group_size, sm, LI4_KERNEL_AUTO, 0, 0, 0, &p) != LI4_OK) return 0;
  // Enough for every kernel family and launch shape the dispatcher may pick.
  size_t best = p.ws_bytes;
  for (int kernel = LI4_KERNEL_CUDA_CORE; kernel <= LI4_KERNEL_ROWS; ++kernel) {
    if (kernel == LI4_KERNEL_CUDA_CORE && M > 8) continue;
    if (li4::make_plan(M, N, K, group_size, sm, kernel, 0, 0, 0, &p) == LI4_OK && p.ws_bytes > best) best = p.ws_bytes;
  }
  return best;
}

extern "C" int li4_int4_linear_plan(int64_t M, int64_t N, int64_t K, int64_t group_size, int sm_count, int* kernel,
                                    int* split, int* grid_x, size_t* smem_bytes) {
  li4::Plan p = {};
  const int sm = sm_count > 0 ? sm_count : li4::current_sm_count();
  const int rc = li4::make_plan(M, N, K, group_size, sm, LI4_KERNEL_AUTO, 0, 0, 0, &p);
  if (rc != LI4_OK) return rc;
  if (kernel) *kernel = p.kernel;
  if (split) *split = p.split;
  if (grid_x) *grid_x = p.grid_x;
  if (smem_bytes) *smem_bytes = p.smem;
  li4::clear_error();
  return LI4_OK;
}

extern "C" int li4_int4_linear(const void* x, const void* packed, const void* scale, const void* zero, void* y,
                               int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t stride_xm,
                               int64_t stride_pn, int64_t stride_sn, int64_t stride_ym, void* workspace,
                               size_t workspace_bytes, void* stream) {
  return li4::int4_linear_impl(x, packed, scale, zero, y, M, N, K, group_size, stride_xm, stride_pn, stride_sn,
                               stride_ym, workspace, workspace_bytes, stream, LI4_KERNEL_AUTO, 0, 0, 0);
}

extern "C" int li4_int4_linear_ex(const void* x, const void* packed, const void* scale, const void* zero, void* y,
                                  int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t stride_xm,
                                  int64_t stride_pn, int64_t stride_sn, int64_t stride_ym, void* workspace,
                                  size_t workspace_bytes, void* stream, int kernel, int rows_per_cta, int split,
                                  int max_ctas) {
  return li4::int4_linear_impl(x, packed, scale, zero, y, M, N, K, group_size, stride_xm, stride_pn, stride_sn,
                               stride_ym, workspace, workspace_bytes, stream, kernel, rows_per_cta, split, max_ctas);
}

extern "C" int li4_device_errors(unsigned* flags, int reset) {
  if (!flags) return li4::set_error(LI4_ERR_INVALID_ARG, "device_errors: null output");
  int rc = li4::check_cuda(cudaMemcpyFromSymbol(flags, li4::g_li4_device_error, sizeof(unsigned)),
                           "device_errors: reading the flags");
  if (rc == LI4_OK && reset) {
    const unsigned zero = 0;
    rc = li4::check_cuda(cudaMemcpyToSymbol(li4::g_li4_device_error, &zero, sizeof(unsigned)),
                         "device_errors: clearing the flags");
  }
  unsigned comm = 0;
  if (rc == LI4_OK) rc = li4::comm_device_errors(&comm, reset != 0);
  if (rc == LI4_OK) *flags |= comm;
  unsigned prog = 0;
  if (rc == LI4_OK) rc = li4::program_device_errors(&prog, reset != 0);
  if (rc == LI4_OK) *flags |= prog;
  unsigned gemm = 0;
  if (rc == LI4_OK) rc = li4::gemm_device_errors(&gemm, reset != 0);
  if (rc == LI4_OK) *flags |= gemm;
  // the error words of the other translation units (GEMV code, the argmax key exchange)
  int (*const readers[])(unsigned*, bool) = {li4::slab_device_errors, li4::rows_device_errors,
                                             li4::ring_device_errors, li4::program_gemv_device_errors,
                                             li4::sample_device_errors};
  for (auto read : readers) {
    unsigned f = 0;
    if (rc == LI4_OK) rc = read(&f, reset != 0);
    if (rc == LI4_OK) *flags |= f;
  }
  if (rc == LI4_OK) li4::clear_error();
  return rc;
}

extern "C" int li4_int4_linear_fused(const void* x, const void* packed, const void* scale, const void* zero, void* y,
                                     int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t stride_xm,
                                     int64_t stride_pn, int64_t stride_sn, int64_t stride_ym, const li4_fusion* fusion,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  return li4::int4_linear_impl(x, packed, scale, zero, y, M, N, K, group_size, stride_xm, stride_pn, stride_sn,
                               stride_ym, workspace, workspace_bytes, stream, LI4_KERNEL_AUTO, 0, 0, 0, fusion);
}

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot hand this library a workspace: code that runs while a
// CUDA graph is being captured or under an allocator that forbids new device
// allocations after warm-up (cudaMalloc can synchronise the device), and hosts
// that bind only this C ABI and own no device allocator of their own.  For
// them the split-K partial sums and arrival counters live in one static device
// array of this translation unit, sized once for the decode shapes.  The
// array exists on every GPU that loads the library, for the life of the
// process.  All calls share it, so two calls that may overlap on the GPU (for
// example on two streams) race; keep such calls on one stream.
// ---------------------------------------------------------------------------
namespace li4 {

constexpr size_t kNoAllocScratchBytes = LI4_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.  The host-side
// symbol is only a stand-in for the array, so the address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* by_device[64] = {};
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "int4_linear_noalloc: cudaGetDevice");
  if (rc != LI4_OK) return rc;
  if (dev < 0 || dev >= 64) return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_noalloc: device ordinal %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (by_device[dev] == nullptr) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "int4_linear_noalloc: cudaGetSymbolAddress");
    if (rc != LI4_OK) return rc;
    by_device[dev] = p;
  }
  *out = by_device[dev];
  return LI4_OK;
}

}  // namespace li4

extern "C" int li4_int4_linear_noalloc(const void* x, const void* packed, const void* scale, const void* zero,
                                       void* y, int64_t M, int64_t N, int64_t K, int64_t group_size,
                                       int64_t stride_xm, int64_t stride_pn, int64_t stride_sn, int64_t stride_ym,
                                       void* stream) {
  using namespace li4;
  Plan p = {};
  int rc = make_plan(M, N, K, group_size, current_sm_count(), LI4_KERNEL_AUTO, 0, 0, 0, &p);
  if (rc != LI4_OK) return rc;
  void* scratch = nullptr;
  if (p.ws_bytes > 0) {
    if (p.ws_bytes > kNoAllocScratchBytes)
      return set_error(LI4_ERR_WORKSPACE, "int4_linear_noalloc: M=%lld N=%lld K=%lld needs %zu bytes of split-K "
                       "scratch, more than the %zu-byte static scratch of this entry point; call li4_int4_linear "
                       "with a workspace instead", (long long)M, (long long)N, (long long)K, p.ws_bytes,
                       kNoAllocScratchBytes);
    rc = noalloc_scratch(&scratch);
    if (rc != LI4_OK) return rc;
    // The counters must start at zero and the array keeps whatever the previous call left in
    // it: clear the whole counter region, whichever launch plan runs.
    rc = check_cuda(cudaMemsetAsync(scratch, 0, LI4_WORKSPACE_COUNTER_BYTES, static_cast<cudaStream_t>(stream)),
                    "int4_linear_noalloc: clearing the arrival counters");
    if (rc != LI4_OK) return rc;
  }
  return int4_linear_impl(x, packed, scale, zero, y, M, N, K, group_size, stride_xm, stride_pn, stride_sn, stride_ym,
                          scratch, scratch ? kNoAllocScratchBytes : 0, stream, LI4_KERNEL_AUTO, 0, 0, 0);
}
