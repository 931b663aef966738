// li4_gemv_device.cuh -- device-side pieces of the INT4 GEMV shared by the per-launch kernels
// (li4_gemv.cu) and the persistent decode program (li4_program.cu), sm_100a: the launch
// arguments, the fused epilogues, the RMSNorm prologue, the x staging layout, the
// tensor-core unit of one 16-row x 128-k weight slab, and the mbarrier / bulk-copy helpers.
#pragma once

#include "li4_common.cuh"
#include "li4_internal.h"
#include "../../include/llama_int4_b200.h"

namespace li4 {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxKsPerCta = 16;  // K range of one CTA <= 16 * 128 = 2048 (x staging)
constexpr int kBatch = 4;         // ksteps one warp loads before it computes

struct GemvArgs {
  const __half* x;
  const uint8_t* packed;
  const __half* scale;
  const __half* zero;
  __half* y;
  int M, N, K;
  int log2_group;
  long long sxm, spn, ssn, sym;  // strides: x, scale/zero, y in elements; packed in bytes
  int n_tiles;                   // ceil(N / ROWS)
  int split;                     // number of K ranges (grid.y)
  int ks_per_split;              // ksteps per K range
  float* partial;                // [split][M][N] fp32, split > 1 only
  unsigned* counters;            // [n_tiles] arrival counters, split > 1 only
  // li4_int4_linear_fused (zero / null otherwise)
  const __half* norm_w;          // RMSNorm weight [K] applied while staging x
  float norm_eps;
  int epi;                       // li4_epilogue_kind
  const __half* res;             // LI4_EPI_RESIDUAL
  long long srm;
  int q_rows, k_rows, head_dim;  // LI4_EPI_QKV_ROPE
  const long long* pos;
  const float* rope_cos;
  const float* rope_sin;
  long long rope_stride;
  __half* q_out;
  long long sqm;
  __half* cache_k;
  __half* cache_v;
  long long cache_sb, cache_ss;
  float* ssq_out;                // LI4_EPI_RESIDUAL: per 16-row tile, per row m, sum of the written values squared
  const float* ssq_in;           // RMSNorm prologue: the producer's ssq_out, [ssq_tiles][M]
  int ssq_tiles;
  unsigned long long* am_keys;   // greedy argmax (LI4_EPI_STORE_F32, tile kernel): [M] running keys,
  unsigned* am_count;            // then the CTA arrival count (li4_fusion.argmax_scratch)
  long long* am_out;
  long long am_stride;
  // LI4_EPI_ALLREDUCE_RESIDUAL: every rank's receive buffer [world][ar_words] (peer pointers),
  // this rank's per-tile call counts, words per sender (N / 16 * M * 8)
  unsigned long long* ar_recv[8];
  unsigned* ar_epochs;
  long long ar_words;
  int ar_world, ar_rank;
};

// ---------------------------------------------------------------------------
// Fused epilogues.  Every GEMV output is rounded to fp16 first, as the
// reference's fp16 Linear output is, and each later fp16 intermediate of the
// reference is rounded again at the same point.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool epi_paired(const GemvArgs& a) {
  return a.epi == LI4_EPI_SWIGLU || a.epi == LI4_EPI_QKV_ROPE;
}

// One output y[m, row] (LI4_EPI_STORE / LI4_EPI_RESIDUAL / LI4_EPI_STORE_F32); returns the value written.
__device__ __forceinline__ float emit_one(const GemvArgs& a, int m, int row, float v) {
  __half h = __float2half_rn(v);
  if (a.epi == LI4_EPI_STORE_F32) {  // fp16 Linear output widened: logits = output(h).float() (llama/model.py:455)
    reinterpret_cast<float*>(a.y)[(long long)m * a.sym + row] = __half2float(h);
    return __half2float(h);
  }
  if (a.epi == LI4_EPI_RESIDUAL)  // h = x + wo(...): fp16 + fp16 (llama/model.py:358-362)
    h = __float2half_rn(__half2float(h) + __half2float(a.res[(long long)m * a.srm + row]));
  a.y[(long long)m * a.sym + row] = h;
  return __half2float(h);
}

// Pair `pair` of a paired-row weight: v0 from tile row j, v1 from tile row j + 8.
__device__ __forceinline__ void emit_pair(const GemvArgs& a, int m, int pair, float v0, float v1) {
  const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
  if (a.epi == LI4_EPI_SWIGLU) {  // F.silu(w1(x)) * w3(x) (llama/model.py:315)
    const float g = __half2float(h0);
    const float sg = __half2float(__float2half_rn(g / (1.0f + expf(-g))));
    a.y[(long long)m * a.sym + pair] = __float2half_rn(sg * __half2float(h1));
    return;
  }
  // LI4_EPI_QKV_ROPE: rows (2 pair, 2 pair + 1) of [q | k | v]
  const int row = 2 * pair;
  const long long p = *a.pos;
  if (row < a.q_rows + a.k_rows) {  // (even, odd) as one complex number times e^{i pos f_i} (llama/model.py:126-152)
    const int d = row < a.q_rows ? row : row - a.q_rows;
    const int i = (d % a.head_dim) >> 1;
    const float c = a.rope_cos[p * a.rope_stride + i], s = a.rope_sin[p * a.rope_stride + i];
    const float x0 = __half2float(h0), x1 = __half2float(h1);
    const __half2 o = __floats2half2_rn(x0 * c - x1 * s, x0 * s + x1 * c);
    __half* dst = row < a.q_rows ? a.q_out + (long long)m * a.sqm + d
                                 : a.cache_k + (long long)m * a.cache_sb + p * a.cache_ss + d;
    *reinterpret_cast<__half2*>(dst) = o;
  } else {  // v goes to the cache unrotated (llama/model.py:257-258)
    const int d = row - a.q_rows - a.k_rows;
    *reinterpret_cast<__half2*>(a.cache_v + (long long)m * a.cache_sb + p * a.cache_ss + d) = __halves2half2(h0, h1);
  }
}

// The reduced outputs of one 16-row tile, value(r, m) for local row r, emitted
// by threads tid = 0 .. nthr-1 of the caller's group.
// value(r, m) of a tile reduced over the split-K partial sums (fixed order).
struct PartialSum {
  const float* base;  // partial + first row of the tile
  int M;
  long long N;
  int split;
  __device__ __forceinline__ float operator()(int r, int m) const {
    float v = 0.f;
    for (int sp = 0; sp < split; ++sp) v += __ldcg(&base[((long long)sp * M + m) * N + r]);
    return v;
  }
};

// value(r, m) of a tile reduced over the warps' partial tiles in shared memory.
template <int COLS, int WARPS>
struct WarpTileSum {
  const float* rb;  // [warps][16][COLS]
  __device__ __forceinline__ float operator()(int r, int m) const {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) v += rb[(w * 16 + r) * COLS + m];
    return v;
  }
};

// Pull the residual rows a tile's epilogue will read into L1 while x is being staged, so the
// epilogue's loads do not add an L2 round trip to the end of the launch.  Threads tid < M of
// the group prefetch one 32-byte segment each (rows tile*16 .. +16 of row m).
template <bool FUSED>
__device__ __forceinline__ void prefetch_residual(const GemvArgs& a, int tile16, int tid) {
  if (FUSED && (a.epi == LI4_EPI_RESIDUAL || a.epi == LI4_EPI_ALLREDUCE_RESIDUAL) && tid < a.M && tile16 >= 0 &&
      tile16 * 16 < a.N)
    asm volatile("prefetch.global.L1 [%0];" ::"l"(a.res + (long long)tid * a.srm + tile16 * 16));
}

// One output through the epilogue (FUSED) or as a plain fp16 store.
template <bool FUSED>
__device__ __forceinline__ void emit_value(const GemvArgs& a, int m, int row, float v) {
  if constexpr (FUSED) emit_one(a, m, row, v);
  else a.y[(long long)m * a.sym + row] = __float2half_rn(v);
}

template <bool FUSED, typename F>
__device__ __forceinline__ void emit_tile(const GemvArgs& a, int tile, int tid, int nthr, F value) {
  const int row0 = tile * 16;
  if (FUSED && a.ssq_out != nullptr) {
    // (row m, tile row r) in half-warp groups of 16 rows: each group also leaves the sum of its
    // written values squared for the next kernel's RMSNorm.  nthr is a multiple of 32 and the
    // loop bound is uniform, so every lane reaches the shuffles.
    const int rows = min(16, a.N - row0);
    for (int base = 0; base < 16 * a.M; base += nthr) {
      const int idx = base + tid, m = idx >> 4, r = idx & 15;
      const bool live = idx < 16 * a.M;
      float sq = 0.f;
      if (live && r < rows) {
        const float h = emit_one(a, m, row0 + r, value(r, m));
        sq = h * h;
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      if (live && r == 0) a.ssq_out[(long long)tile * a.M + m] = sq;
    }
    return;
  }
  if (FUSED && epi_paired(a)) {  // N is a multiple of 16: full tiles
    for (int idx = tid; idx < 8 * a.M; idx += nthr) {
      const int j = idx / a.M, m = idx - j * a.M;
      emit_pair(a, m, tile * 8 + j, value(j, m), value(j + 8, m));
    }
  } else {
    const int rows = min(16, a.N - row0);
    for (int idx = tid; idx < rows * a.M; idx += nthr) {
      const int r = idx / a.M, m = idx - r * a.M;
      emit_value<FUSED>(a, m, row0 + r, value(r, m));
    }
  }
}

// emit_one with the residual value already loaded (rv; LI4_EPI_RESIDUAL only).
__device__ __forceinline__ void emit_one_pre(const GemvArgs& a, int m, int row, float v, float rv) {
  __half h = __float2half_rn(v);
  if (a.epi == LI4_EPI_STORE_F32) {
    reinterpret_cast<float*>(a.y)[(long long)m * a.sym + row] = __half2float(h);
    return;
  }
  if (a.epi == LI4_EPI_RESIDUAL) h = __float2half_rn(__half2float(h) + rv);
  a.y[(long long)m * a.sym + row] = h;
}

// The split-K reduction of one 16-row tile by one warp, for M > 8 (up to 8 outputs per lane):
// every partial the lane sums (four K ranges at a time, in the fixed order of PartialSum) and
// every residual it adds are loaded before it stores anything, so the epilogue costs a few L2
// round trips instead of one per output (two K ranges per round: more would spill registers in
// the register-ring kernels).  The paired and sum-of-squares epilogues take emit_tile.
template <bool FUSED>
__device__ __forceinline__ void emit_partial_tile(const GemvArgs& a, int tile, int lane, const PartialSum& ps) {
  if ((FUSED && (a.ssq_out != nullptr || epi_paired(a))) || (long long)ps.M * ps.N > 0x7FFFFFFFLL) {
    emit_tile<FUSED>(a, tile, lane, 32, ps);  // (and partial blocks beyond 32-bit offsets)
    return;
  }
  const int row0 = tile * 16, rows = min(16, a.N - row0), n = rows * a.M;
  int off[8];  // offset of output i of this lane in a K range's partial block (M * N < 2^31, above)
  float acc[8], rv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = lane + 32 * i, r = idx / a.M, m = idx - r * a.M;
    off[i] = idx < n ? m * (int)ps.N + r : 0;
    acc[i] = 0.f;
    rv[i] = (FUSED && a.epi == LI4_EPI_RESIDUAL && idx < n) ? __half2float(a.res[(long long)m * a.srm + row0 + r]) : 0.f;
  }
  const long long range = (long long)ps.M * ps.N;
  int sp = 0;
  for (; sp + 2 <= ps.split; sp += 2) {
    float t[2][8];
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
      for (int i = 0; i < 8; ++i) t[q][i] = lane + 32 * i < n ? __ldcg(ps.base + (sp + q) * range + off[i]) : 0.f;
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += t[q][i];
  }
  for (; sp < ps.split; ++sp) {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += lane + 32 * i < n ? __ldcg(ps.base + sp * range + off[i]) : 0.f;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = lane + 32 * i;
    if (idx >= n) continue;
    const int r = idx / a.M, m = idx - r * a.M;
    if constexpr (FUSED) emit_one_pre(a, m, row0 + r, acc[i], rv[i]);
    else a.y[(long long)m * a.sym + row0 + r] = __float2half_rn(acc[i]);
  }
}

// Rows mode: a warp's 16-row tile `tile16` straight from its lanes' accumulators (lane (grp, quad)
// holds rows grp and grp + 8, columns nt*8 + 2*quad + {0, 1}); split == 1.
template <bool FUSED, int NT>
__device__ __forceinline__ void emit_warp_tile(const GemvArgs& a, int tile16, const float (&acc)[NT][4], int grp,
                                               int quad) {
  const int row0 = tile16 * 16;
  const int rows = min(16, a.N - row0);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    if (FUSED && epi_paired(a)) {  // rows grp and grp + 8 of the tile are a pair
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int m = nt * 8 + 2 * quad + e;
        if (m < a.M && row0 < a.N) emit_pair(a, m, tile16 * 8 + grp, acc[nt][e], acc[nt][e + 2]);
      }
      continue;
    }
    float sq[2] = {0.f, 0.f};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = grp + 8 * (e >> 1), m = nt * 8 + 2 * quad + (e & 1);
      if (r < rows && m < a.M) {
        if constexpr (FUSED) {
          const float h = emit_one(a, m, row0 + r, acc[nt][e]);
          sq[e & 1] += h * h;
        } else {
          a.y[(long long)m * a.sym + row0 + r] = __float2half_rn(acc[nt][e]);
        }
      }
    }
    if (FUSED && a.ssq_out != nullptr) {  // sum over the tile's rows: the 8 lanes of a quad column
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        sq[0] += __shfl_xor_sync(0xffffffffu, sq[0], o);
        sq[1] += __shfl_xor_sync(0xffffffffu, sq[1], o);
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int m = nt * 8 + 2 * quad + e;
        if (grp == 0 && m < a.M && row0 < a.N) a.ssq_out[(long long)tile16 * a.M + m] = sq[e];
      }
    }
  }
}

// 1 / rms from the producer's per-tile sums of squares (fusion.sumsq_in): one warp per row.
template <int WARPS>
__device__ __forceinline__ void rms_from_ssq(const GemvArgs& a, float* s_rstd, int warp, int lane) {
  for (int m = warp; m < a.M; m += WARPS) {
    float ss = 0.f;
    for (int t = lane; t < a.ssq_tiles; t += 32) ss += a.ssq_in[(long long)t * a.M + m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) s_rstd[m] = rsqrtf(ss / (float)a.K + a.norm_eps);
  }
}

// Per-row 1 / rms of x for the RMSNorm prologue: s_rstd[m] = rsqrt(mean_k x[m,k]^2 + eps),
// the mean in fp32 over all K columns (llama/model.py:61).  One warp per row, 16-byte loads
// unrolled so a row's loads are in flight together; the caller synchronises before use.
template <int WARPS>
__device__ __forceinline__ void rms_factors(const GemvArgs& a, float* s_rstd, int warp, int lane) {
  const bool vec = ((reinterpret_cast<uintptr_t>(a.x) & 15u) == 0) && ((a.sxm & 7) == 0);
#pragma unroll 2
  for (int m = warp; m < a.M; m += WARPS) {
    const __half* row = a.x + (long long)m * a.sxm;
    float ss = 0.f;
    if (vec) {
      const uint4* r4 = reinterpret_cast<const uint4*>(row);
      const int n4 = a.K >> 3;
#pragma unroll 4
      for (int c = lane; c < n4; c += 32) {
        const uint4 u = r4[c];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
          ss = fmaf(f.x, f.x, ss);
          ss = fmaf(f.y, f.y, ss);
        }
      }
    } else {
      for (int k = lane; k < a.K; k += 32) {
        const float v = __half2float(row[k]);
        ss = fmaf(v, v, ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) s_rstd[m] = rsqrtf(ss / (float)a.K + a.norm_eps);
  }
}

// fp16(fp16(x * rstd) * w): RMSNorm's output cast (type_as) and its fp16 weight product.
// The fp16 x fp16 product is exact before its one rounding, so the half2 multiply gives the same
// bits as the reference's float multiply rounded to fp16.
__device__ __forceinline__ uint32_t norm_pair(uint32_t xv, uint32_t wv, float rstd) {
  const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xv));
  const __half2 n = __floats2half2_rn(xf.x * rstd, xf.y * rstd);
  const __half2 o = __hmul2(n, *reinterpret_cast<const __half2*>(&wv));
  return *reinterpret_cast<const uint32_t*>(&o);
}

// ---------------------------------------------------------------------------
// x staging.  Block b = ((ks * NT + nt) * M8 + m8) * 4 + quad holds the 32
// values x[m][k0 .. k0+32), m = nt*8 + m8, k0 = kstep*128 + 32*quad, as 16
// half2 words; word 4w + i = (x[k0 + 8w + i], x[k0 + 8w + i + 4]).  Chunk w
// (16 bytes) of block b sits at b*64 + ((w ^ key) << 4) with
// key = (2*m8 + (quad >> 1)) & 3, which keeps the 128-bit reads of 8
// consecutive blocks on distinct banks and does not depend on the kstep (so a
// reader can precompute its offsets).
// ---------------------------------------------------------------------------
__device__ __forceinline__ int xs_key(int m8, int quad) { return (2 * m8 + (quad >> 1)) & 3; }

// block = ((kstep * NT + nt) * M8 + m8) * 4 + quad
__device__ __forceinline__ int xs_chunk_offset(int block, int w, int m8) {
  return block * 64 + ((w ^ xs_key(m8, block & 3)) << 4);
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// The same load as an ordered instruction: loop-invariant B fragments stay in
// shared memory instead of being hoisted into registers across tiles.
__device__ __forceinline__ uint4 lds128_ordered(const uint8_t* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
  return r;
}

// s_rstd: per-row RMSNorm factors (rms_factors) when a.norm_w is set, else unused.
template <int NT, int THREADS = kThreads, bool NORM = false>
__device__ __forceinline__ void stage_x(const GemvArgs& a, int ks0, int nks, int M8, uint8_t* xs,
                                        const float* s_rstd = nullptr) {
  // One thread per 16-byte k-chunk (k = 8 values) and every row of it: the RMSNorm weight chunk
  // is read once.
  const int chunks = nks * 16;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(a.x) & 15u) == 0) && ((a.sxm & 7) == 0);
  for (int c = threadIdx.x; c < chunks; c += THREADS) {
    const int ks = c >> 4, quad = (c >> 2) & 3, w = c & 3;
    const long long k = (long long)(ks0 + ks) * 128 + 32 * quad + 8 * w;
    uint4 wn = make_uint4(0u, 0u, 0u, 0u);
    if (NORM && a.norm_w != nullptr) wn = *reinterpret_cast<const uint4*>(a.norm_w + k);  // 16-byte aligned
    // M > 8 (two n-tiles): the rows' loads in flight together, 8 at a time.  M <= 8 keeps the
    // loop below, measured faster at M = 1 (where it has one load per chunk) -- the batched
    // form in the same kernel slowed the M = 1 launches by up to 0.3 us.
    if (NT == 2 && vec_ok) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {  // the 8 rows of an n-tile in flight together
      uint4 v[8];
#pragma unroll
      for (int m8 = 0; m8 < 8; ++m8) {
        const int i = nt * 8 + m8;
        v[m8] = (m8 < M8 && i < a.M) ? *reinterpret_cast<const uint4*>(a.x + (long long)i * a.sxm + k)
                                     : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int m8 = 0; m8 < 8; ++m8) {
        const int i = nt * 8 + m8;
        if (m8 >= M8) continue;
        uint32_t u[4] = {v[m8].x, v[m8].y, v[m8].z, v[m8].w};
        if (NORM && a.norm_w != nullptr && i < a.M) {
          const float r = s_rstd[i];
          u[0] = norm_pair(u[0], wn.x, r);
          u[1] = norm_pair(u[1], wn.y, r);
          u[2] = norm_pair(u[2], wn.z, r);
          u[3] = norm_pair(u[3], wn.w, r);
        }
        uint4 out;
        out.x = __byte_perm(u[0], u[2], 0x5410);  // (x0, x4)
        out.y = __byte_perm(u[0], u[2], 0x7632);  // (x1, x5)
        out.z = __byte_perm(u[1], u[3], 0x5410);  // (x2, x6)
        out.w = __byte_perm(u[1], u[3], 0x7632);  // (x3, x7)
        *reinterpret_cast<uint4*>(xs + xs_chunk_offset(((ks * NT + nt) * M8 + m8) * 4 + quad, w, m8)) = out;
      }
      }
      continue;
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int m8 = 0; m8 < 8; ++m8) {
        if (m8 >= M8) break;
        const int m = nt * 8 + m8;
        const int block = ((ks * NT + nt) * M8 + m8) * 4 + quad;
        uint4 out = make_uint4(0u, 0u, 0u, 0u);
        if (m < a.M) {
          const __half* src = a.x + (long long)m * a.sxm + k;
          uint32_t u[4];
          if (vec_ok) {
            const uint4 v = *reinterpret_cast<const uint4*>(src);
            u[0] = v.x; u[1] = v.y; u[2] = v.z; u[3] = v.w;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              u[e] = (uint32_t)__half_as_ushort(src[2 * e]) | ((uint32_t)__half_as_ushort(src[2 * e + 1]) << 16);
          }
          if (NORM && a.norm_w != nullptr) {
            const float r = s_rstd[m];
            u[0] = norm_pair(u[0], wn.x, r);
            u[1] = norm_pair(u[1], wn.y, r);
            u[2] = norm_pair(u[2], wn.z, r);
            u[3] = norm_pair(u[3], wn.w, r);
          }
          out.x = __byte_perm(u[0], u[2], 0x5410);  // (x0, x4)
          out.y = __byte_perm(u[0], u[2], 0x7632);  // (x1, x5)
          out.z = __byte_perm(u[1], u[3], 0x5410);  // (x2, x6)
          out.w = __byte_perm(u[1], u[3], 0x7632);  // (x3, x7)
        }
        *reinterpret_cast<uint4*>(xs + xs_chunk_offset(block, w, m8)) = out;
      }
    }
  }
}

// torch.argmax order as one 64-bit key: the value's order-preserving bits (NaN above every
// number, -0 as +0) above the complement of the index (the first index wins a tie).
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
  unsigned u = __float_as_uint(v);
  unsigned ord;
  if (v != v) {
    ord = 0xFFFFFFFFu;
  } else {
    if (v == 0.f) u = 0u;
    ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)i);
}

// The fused greedy argmax's end of launch: after every warp of the CTA has issued its
// atomicMax (sync), the CTA counts itself in; the last one writes the indices and leaves the
// keys and the count at zero for the next launch.
template <typename Sync>
__device__ __forceinline__ void argmax_finish(const GemvArgs& a, Sync sync) {
  sync();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned total = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(a.am_count, 1u) == total - 1u) {
      __threadfence();
      for (int m = 0; m < a.M; ++m) {
        const unsigned long long k = atomicExch(&a.am_keys[m], 0ull);
        a.am_out[(long long)m * a.am_stride] = (long long)(0xFFFFFFFFu - (unsigned)(k & 0xFFFFFFFFull));
      }
      atomicExch(a.am_count, 0u);
    }
  }
}

struct StreamUnit {
  uint4 lo, hi;          // bytes [16 quad, +16) of the kstep for rows grp and grp + 8
  uint32_t sz_lo, sz_hi; // fp16 bits: scale | zero << 16, for the two rows
};

// Base pointers of a warp-thread for one tile (rows grp, grp + 8).
struct StreamRows {
  const uint8_t* p_lo;
  const uint8_t* p_hi;
  const unsigned short* s_lo;
  const unsigned short* s_hi;
  const unsigned short* z_lo;
  const unsigned short* z_hi;
};

__device__ __forceinline__ StreamRows stream_rows(const GemvArgs& a, int tile, int ks0, int grp, int quad) {
  int r0 = tile * 16 + grp, r1 = r0 + 8;
  r0 = r0 < a.N ? r0 : a.N - 1;
  r1 = r1 < a.N ? r1 : a.N - 1;
  const long long off = (long long)ks0 * 64 + quad * 16;
  const int g0 = (ks0 * 128) >> a.log2_group;
  StreamRows r;
  r.p_lo = a.packed + (long long)r0 * a.spn + off;
  r.p_hi = a.packed + (long long)r1 * a.spn + off;
  r.s_lo = reinterpret_cast<const unsigned short*>(a.scale) + (long long)r0 * a.ssn + g0;
  r.s_hi = reinterpret_cast<const unsigned short*>(a.scale) + (long long)r1 * a.ssn + g0;
  r.z_lo = reinterpret_cast<const unsigned short*>(a.zero) + (long long)r0 * a.ssn + g0;
  r.z_hi = reinterpret_cast<const unsigned short*>(a.zero) + (long long)r1 * a.ssn + g0;
  return r;
}

__device__ __forceinline__ uint32_t ldg_u16(const unsigned short* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ void stream_load(const GemvArgs& a, StreamUnit& u, const StreamRows& r, int ks) {
  u.lo = ldg_stream_v4(r.p_lo + ks * 64);
  u.hi = ldg_stream_v4(r.p_hi + ks * 64);
  const int g = (ks * 128) >> a.log2_group;
  u.sz_lo = ldg_u16(r.s_lo + g) | (ldg_u16(r.z_lo + g) << 16);
  u.sz_hi = ldg_u16(r.s_hi + g) | (ldg_u16(r.z_hi + g) << 16);
}

// acc += s * (W[rows] . x) for one unit.  xs_ks: the unit's kstep in the x
// staging; n-tile nt of it starts nt * nt_stride bytes further.
template <int NT>
__device__ __forceinline__ void stream_compute(const StreamUnit& u, const uint8_t* xs_ks, int nt_stride,
                                               const int boff[4], bool bvalid, float acc[NT][4]) {
  const ZeroConsts zl = make_zero_consts(__ushort_as_half((unsigned short)(u.sz_lo >> 16)));
  const ZeroConsts zh = make_zero_consts(__ushort_as_half((unsigned short)(u.sz_hi >> 16)));
  float c[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) c[nt][e] = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    __half2 pl[4], ph[4];
    unpack8_qz((w == 0) ? u.lo.x : (w == 1) ? u.lo.y : (w == 2) ? u.lo.z : u.lo.w, zl, pl);
    unpack8_qz((w == 0) ? u.hi.x : (w == 1) ? u.hi.y : (w == 2) ? u.hi.z : u.hi.w, zh, ph);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint4 bq = make_uint4(0u, 0u, 0u, 0u);
      if (bvalid) bq = lds128(xs_ks + nt * nt_stride + boff[w]);
      mma_16816(c[nt], h2_as_u32(pl[0]), h2_as_u32(ph[0]), h2_as_u32(pl[1]), h2_as_u32(ph[1]), bq.x, bq.y);
      mma_16816(c[nt], h2_as_u32(pl[2]), h2_as_u32(ph[2]), h2_as_u32(pl[3]), h2_as_u32(ph[3]), bq.z, bq.w);
    }
  }
  const float sl = __half2float(__ushort_as_half((unsigned short)(u.sz_lo & 0xFFFFu)));
  const float sh = __half2float(__ushort_as_half((unsigned short)(u.sz_hi & 0xFFFFu)));
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    acc[nt][0] = fmaf(sl, c[nt][0], acc[nt][0]);
    acc[nt][1] = fmaf(sl, c[nt][1], acc[nt][1]);
    acc[nt][2] = fmaf(sh, c[nt][2], acc[nt][2]);
    acc[nt][3] = fmaf(sh, c[nt][3], acc[nt][3]);
  }
}

constexpr unsigned kBulkWaitLimit = 1u << 22;  // try_wait rounds: well under a second of polling, never forever

// Device error word of the translation unit that includes this header (each has its own copy,
// read through tu_device_errors; li4_device_errors collects them).  Bit 0: a bounded pipeline
// wait ran out; bit 5: a fused all-reduce epilogue's wait ran out.
static __device__ unsigned g_li4_device_error;

// Host side: this translation unit's copy of the device error word, cleared when reset.
static inline int tu_device_errors(unsigned* flags, bool reset) {
  int rc = check_cuda(cudaMemcpyFromSymbol(flags, g_li4_device_error, sizeof(unsigned)), "device_errors: reading");
  if (rc == LI4_OK && reset) {
    const unsigned zero = 0;
    rc = check_cuda(cudaMemcpyToSymbol(g_li4_device_error, &zero, sizeof(unsigned)), "device_errors: clearing");
  }
  return rc;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` with the non-blocking test (a completed phase costs one
// test), at most kBulkWaitLimit polls; a wait that runs out sets bit 0 of the device error word.
__device__ __forceinline__ bool mbar_spin_bounded(uint64_t* bar, unsigned parity) {
  for (unsigned i = 0; i < kBulkWaitLimit; ++i)
    if (mbar_test_wait(bar, parity)) return true;
  atomicOr(&g_li4_device_error, 1u);
  return false;
}

// Wait for phase `parity` of `bar` to complete, at most kBulkWaitLimit rounds.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity) {
  for (unsigned i = 0; i < kBulkWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicOr(&g_li4_device_error, 1u);
  return false;
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` on `bar`; the weight
// bytes it moves are marked evict-first in L2 (weight_l2_policy).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(weight_l2_policy())
      : "memory");
}

// Shared-memory layout of one stage: 16 packed rows of K-range/2 bytes, then
// 16 scale rows and 16 zero rows of KS fp16 values.  When the tile's rows are
// one contiguous block of HBM (contiguous tensors, one K range) a stage is
// three bulk copies and the rows sit back to back; otherwise each row is its
// own copy and the row pitch is K-range/2 + 64, which keeps the 16-byte reads
// of the eight row pairs of a quarter warp on distinct banks.
struct BulkLayout {
  int ks;       // ksteps per K range (8 or 16)
  int pitch;    // bytes between packed rows
  int sz_off;   // scale rows, then zero rows at + 16 * ks * 2
  int stage;    // bytes per stage (multiple of 128)
};

__host__ __device__ inline BulkLayout bulk_layout(int ks, bool contig) {
  BulkLayout L;
  L.ks = ks;
  L.pitch = ks * 64 + (contig ? 0 : 64);
  L.sz_off = 16 * L.pitch;
  L.stage = (L.sz_off + 2 * 16 * ks * 2 + 127) & ~127;
  return L;
}


// Slab kernel (li4_slab.cu): most 16-row tiles one CTA stages in shared memory.
constexpr int kSlabMaxTiles = 16;

// Host: shared-memory bytes of one slab CTA (mbarriers, tile stages, x staging, warp partials).
size_t slab_smem_bytes(int M, int nt, int ks, int tiles_max, int slots, int pitch);

// Host: launch the slab kernel for a.ks_per_split ksteps per K range (a.split ranges on grid.y).
int launch_slab(const GemvArgs& a, int nt, bool fused, int grid_x, int tiles_max, int slots, int pitch,
                size_t smem, cudaStream_t stream);

// Host: launch the register-rows kernel (li4_rows.cu): M = 1, K = 1024 or 2048, 16-byte aligned x.
int launch_rows(const GemvArgs& a, bool fused, cudaStream_t stream);

// Ring kernel (li4_ring.cu): 16 consumer warps and one bulk-copy producer warp per CTA, one CTA
// per SM, a ring of up to kRingMaxStages shared-memory stages of T 16-row tiles each.
constexpr int kRingWarps = 16;
constexpr int kRingThreads = (kRingWarps + 1) * 32;
constexpr int kRingMaxStages = 8;
constexpr size_t kRingSmemCap = 227 * 1024;  // dynamic shared memory one ring CTA may take

// Host: bytes of one ring stage (T tiles of `ks` ksteps at a row pitch of `pitch` bytes) and of
// the whole dynamic shared memory of one ring CTA.
int ring_stage_bytes(int ks, int T, int pitch);
size_t ring_smem_bytes(int M, int ks, int stages, int stage_bytes);

// Host: launch the ring kernel (group 128, M <= 8, one K range: a.ks_per_split == K / 128).
int launch_ring(const GemvArgs& a, bool fused, int grid_x, int T, int stages, int pitch, size_t smem,
                cudaStream_t stream);

// Host: validate one linear (and its fusion) as li4_int4_linear_fused does and fill the
// GemvArgs fields that do not depend on the launch plan (li4_gemv.cu).
int prepare_linear(const void* x, const void* packed, const void* scale, const void* zero, void* y, int64_t M,
                   int64_t N, int64_t K, int64_t group, int64_t sxm, int64_t spn, int64_t ssn, int64_t sym,
                   const li4_fusion* f, GemvArgs* out);

}  // namespace li4
