// li4_slab.cu -- the slab GEMV kernel (sm_100a): every CTA stages its whole weight slice in
// shared memory with bulk copies issued before the dependency wait, and all warps of the CTA
// split the K range of each 16-row tile.
//
// Why this shape.  In a decode step the linears run back to back, each reading an x that the
// preceding kernel wrote.  With programmatic dependent launch a kernel can start while its
// predecessor still runs, but only on SMs where the predecessor leaves room.  The slab kernel
// keeps one CTA at 256 threads (<= 128 registers) and, for the Llama-3.2-1B layer shapes, at
// most about 100 KB of shared memory, so the next launch's CTA fits beside it on the same SM:
// the next linear's weights stream from HBM into its shared memory while this one computes.
// After the wait only x staging, the tensor-core work on resident weights, one shared-memory
// reduction and the stores remain on the launch chain.
//
// Work split.  A CTA owns a contiguous range of 16-row tiles (ceil(n_tiles / grid_x) at most)
// and one K range (grid.y; split-K only where x would not fit).  Each tile is one
// shared-memory stage with its own mbarrier: 16 packed rows of ks*64 bytes, then 16 scale
// rows and 16 zero rows of ks fp16 values.  The warps form `slots` x (8 / slots) groups:
// warp w takes ksteps w % slots, + slots, ... of tiles w / slots, + 8 / slots, ..., so every
// warp works on every tile when slots == 8.  The per-warp partial sums meet in shared memory
// and the epilogue sums them in a fixed order (bitwise deterministic).
//
// Math per 16-row x 128-k unit as in the other GEMV kernels (stream_compute): exact q - zero
// in fp16 from the magic-number unpack, m16n8k16 with fp32 accumulation, group scale in fp32.
#include "li4_common.cuh"
#include "li4_gemv_device.cuh"
#include "li4_internal.h"

#include <mutex>
#include <vector>

namespace li4 {

constexpr int kSlabWarps = 8;
constexpr int kSlabThreads = kSlabWarps * 32;
constexpr int kSlabBarBytes = 8 * kSlabMaxTiles;  // one mbarrier per tile stage

struct SlabArgs {
  int tiles_max;  // most tiles one CTA owns (stages in shared memory)
  int slots;      // warps sharing one tile's ksteps: a power of two <= 8 dividing ks
  int pitch;      // bytes between packed rows of a stage (ks*64, or ks*64 + 64 against bank conflicts)
  int stage;      // bytes per stage, a multiple of 128
  int sz_mode;    // scale / zero rows: 0 one block copy per tile, 1 a copy per row, 2 plain loads
};

__host__ __device__ inline int slab_stage_bytes(int ks, int pitch) {
  return (16 * pitch + 2 * 16 * ks * 2 + 127) & ~127;
}

// value(r, m) of one tile: the warps' partials summed in slot order.
struct SlabSum {
  const float* base;  // red + tile * slots * 16 * M
  int slots, M;
  __device__ __forceinline__ float operator()(int r, int m) const {
    float p[8];
#pragma unroll
    for (int s = 0; s < 8; ++s) p[s] = s < slots ? base[(s * 16 + r) * M + m] : 0.f;
    float v = 0.f;
#pragma unroll
    for (int s = 0; s < 8; ++s) v += p[s];  // slot order (the zero tail adds nothing)
    return v;
  }
};

// x for the CTA's K range into the staging layout of stage_x (li4_gemv_device.cuh), with up
// to U 16-byte loads in flight per thread (one L2 round trip per U items): item i = (k-chunk c,
// staged row j), j fastest.
template <int NT, bool NORM>
__device__ __forceinline__ void slab_stage_x(const GemvArgs& a, int ks0, int nks, int M8, uint8_t* xs,
                                             const float* s_rstd) {
  constexpr int U = 4;
  const int rows = NT * M8;
  const int items = nks * 16 * rows;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(a.x) & 15u) == 0) && ((a.sxm & 7) == 0);
  for (int i0 = threadIdx.x; i0 < items; i0 += U * kSlabThreads) {
    uint4 v[U];
    if (vec_ok) {
      // every load of the round issued before any is used: out-of-range items read x[0][k0]
      // (in bounds) and are zeroed afterwards, so there is no branch between the loads
      const __half* src[U];
      bool live[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * kSlabThreads;
        const int c = i / rows, j = i - c * rows;
        const int m = (j / M8) * 8 + (j % M8);
        live[u] = i < items && m < a.M;
        src[u] = live[u] ? a.x + (long long)m * a.sxm + (long long)ks0 * 128 + (long long)c * 8 : a.x;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = *reinterpret_cast<const uint4*>(src[u]);
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (!live[u]) v[u] = make_uint4(0u, 0u, 0u, 0u);
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * kSlabThreads;
        v[u] = make_uint4(0u, 0u, 0u, 0u);
        if (i < items) {
          const int c = i / rows, j = i - c * rows;
          const int m = (j / M8) * 8 + (j % M8);
          if (m < a.M) {
            const __half* src = a.x + (long long)m * a.sxm + (long long)ks0 * 128 + (long long)c * 8;
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = (uint32_t)__half_as_ushort(src[2 * e]) | ((uint32_t)__half_as_ushort(src[2 * e + 1]) << 16);
            v[u] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * kSlabThreads;
      if (i >= items) break;
      const int c = i / rows, j = i - c * rows;
      const int nt = j / M8, m8 = j % M8, m = nt * 8 + m8;
      const int ks = c >> 4, quad = (c >> 2) & 3, w = c & 3;
      uint32_t q[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      if (NORM && m < a.M) {
        const long long k = (long long)ks0 * 128 + (long long)c * 8;
        const uint4 wn = *reinterpret_cast<const uint4*>(a.norm_w + k);
        const float r = s_rstd[m];
        q[0] = norm_pair(q[0], wn.x, r);
        q[1] = norm_pair(q[1], wn.y, r);
        q[2] = norm_pair(q[2], wn.z, r);
        q[3] = norm_pair(q[3], wn.w, r);
      }
      uint4 out;
      out.x = __byte_perm(q[0], q[2], 0x5410);  // (x0, x4)
      out.y = __byte_perm(q[0], q[2], 0x7632);  // (x1, x5)
      out.z = __byte_perm(q[1], q[3], 0x5410);  // (x2, x6)
      out.w = __byte_perm(q[1], q[3], 0x7632);  // (x3, x7)
      *reinterpret_cast<uint4*>(xs + xs_chunk_offset(((ks * NT + nt) * M8 + m8) * 4 + quad, w, m8)) = out;
    }
  }
}

// The A fragments of one 16-row x 128-k unit (exact q - zero in fp16, mma.m16n8k16 order: word
// 8w + {0..3} / {4..7} are the A registers of the unit's two MMAs on 16-byte chunk w) and the two
// row scales.  Unpacking needs no x, so a warp builds its first units' fragments before the
// dependency wait, while the preceding kernel still runs.
struct SlabFrag {
  uint32_t a[32];
  float s_lo, s_hi;
};

__device__ __forceinline__ void slab_unpack(SlabFrag& f, const uint8_t* row_lo, const uint8_t* row_hi,
                                            const unsigned short* sc, const unsigned short* ze, int grp, int ks,
                                            int ks_n) {
  const uint4 lo = lds128(row_lo + ks * 64), hi = lds128(row_hi + ks * 64);
  const unsigned short zlo = ze[grp * ks_n + ks], zhi = ze[(grp + 8) * ks_n + ks];
  f.s_lo = __half2float(__ushort_as_half(sc[grp * ks_n + ks]));
  f.s_hi = __half2float(__ushort_as_half(sc[(grp + 8) * ks_n + ks]));
  const ZeroConsts zl = make_zero_consts(__ushort_as_half(zlo)), zh = make_zero_consts(__ushort_as_half(zhi));
  const uint32_t wl[4] = {lo.x, lo.y, lo.z, lo.w}, wh[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    __half2 pl[4], ph[4];
    unpack8_qz(wl[w], zl, pl);
    unpack8_qz(wh[w], zh, ph);
    f.a[8 * w + 0] = h2_as_u32(pl[0]);
    f.a[8 * w + 1] = h2_as_u32(ph[0]);
    f.a[8 * w + 2] = h2_as_u32(pl[1]);
    f.a[8 * w + 3] = h2_as_u32(ph[1]);
    f.a[8 * w + 4] = h2_as_u32(pl[2]);
    f.a[8 * w + 5] = h2_as_u32(ph[2]);
    f.a[8 * w + 6] = h2_as_u32(pl[3]);
    f.a[8 * w + 7] = h2_as_u32(ph[3]);
  }
}

// acc += s * (W[unit rows] . x[kstep]): the unit's 8 MMAs on four independent accumulators
// (dependency depth 2), summed pairwise, then scaled per row in fp32.
template <int NT>
__device__ __forceinline__ void slab_mma(const SlabFrag& f, const uint8_t* xs_ks, int nt_stride, const int boff[4],
                                         bool bvalid, float acc[NT][4]) {
  float c[4][NT][4];
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) c[w][nt][e] = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint4 bq = make_uint4(0u, 0u, 0u, 0u);
      if (bvalid) bq = lds128(xs_ks + nt * nt_stride + boff[w]);
      mma_16816(c[w][nt], f.a[8 * w + 0], f.a[8 * w + 1], f.a[8 * w + 2], f.a[8 * w + 3], bq.x, bq.y);
      mma_16816(c[w][nt], f.a[8 * w + 4], f.a[8 * w + 5], f.a[8 * w + 6], f.a[8 * w + 7], bq.z, bq.w);
    }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = (c[0][nt][e] + c[1][nt][e]) + (c[2][nt][e] + c[3][nt][e]);
    acc[nt][0] = fmaf(f.s_lo, v[0], acc[nt][0]);
    acc[nt][1] = fmaf(f.s_lo, v[1], acc[nt][1]);
    acc[nt][2] = fmaf(f.s_hi, v[2], acc[nt][2]);
    acc[nt][3] = fmaf(f.s_hi, v[3], acc[nt][3]);
  }
}

template <int NT, bool FUSED>
__global__ void __launch_bounds__(kSlabThreads, 2) gemv_slab_kernel(const __grid_constant__ GemvArgs a,
                                                                   const __grid_constant__ SlabArgs sa) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int ks_n = a.ks_per_split;
  const int ks0 = blockIdx.y * ks_n;
  const int M8 = (NT == 1) ? a.M : 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 2, quad = lane & 3;
  const int t_begin = (int)((long long)blockIdx.x * a.n_tiles / gridDim.x);
  const int t_end = (int)((long long)(blockIdx.x + 1) * a.n_tiles / gridDim.x);
  const int my_tiles = t_end - t_begin;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint8_t* stages = smem + kSlabBarBytes;
  uint8_t* xs = stages + (size_t)sa.tiles_max * sa.stage;
  float* red = reinterpret_cast<float*>(xs + (size_t)ks_n * NT * M8 * 256);
  __shared__ float s_rstd[LI4_MAX_M];

  if (threadIdx.x == 0) {
    for (int t = 0; t < my_tiles; ++t) mbar_init(&bars[t], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_launch_dependents();

  // ---- weights: bulk copies before the dependency wait (weights never come from the preceding kernel)
  if (warp == 0) {
    const unsigned row_bytes = (unsigned)ks_n * 64;
    const unsigned sz_row = (unsigned)ks_n * 2;
    for (int t = 0; t < my_tiles; ++t) {
      const int tile = t_begin + t;
      const int valid = min(16, a.N - tile * 16);
      uint8_t* st = stages + (size_t)t * sa.stage;
      uint8_t* sc = st + 16 * sa.pitch;
      uint8_t* ze = sc + 16 * sz_row;
      unsigned bytes = 16u * row_bytes;
      if (sa.sz_mode == 0) bytes += 2u * (unsigned)valid * sz_row;
      else if (sa.sz_mode == 1) bytes += 2u * 16u * sz_row;
      if (lane == 0) mbar_arrive_expect_tx(&bars[t], bytes);
      __syncwarp();
      if (lane < 16) {
        const int r = min(tile * 16 + lane, a.N - 1);  // rows past N repeat row N-1 (outputs discarded)
        bulk_g2s(st + lane * sa.pitch, a.packed + (long long)r * a.spn + (long long)ks0 * 64, row_bytes, &bars[t]);
      } else if (sa.sz_mode == 0) {  // the tile's scale (zero) rows are one block: rows tile*16 .. +valid
        if (lane == 16)
          bulk_g2s(sc, a.scale + (long long)tile * 16 * a.ssn, (unsigned)valid * sz_row, &bars[t]);
        else if (lane == 17)
          bulk_g2s(ze, a.zero + (long long)tile * 16 * a.ssn, (unsigned)valid * sz_row, &bars[t]);
      } else if (sa.sz_mode == 1) {
        const int j = lane - 16;
        const int r = min(tile * 16 + j, a.N - 1);
        bulk_g2s(sc + j * sz_row, a.scale + (long long)r * a.ssn + ks0, sz_row, &bars[t]);
        bulk_g2s(ze + j * sz_row, a.zero + (long long)r * a.ssn + ks0, sz_row, &bars[t]);
      } else {  // rows not 16-byte aligned: plain loads (seen by the other warps through the barrier below)
        const int j = lane - 16;
        const int r = min(tile * 16 + j, a.N - 1);
        const unsigned short* gs = reinterpret_cast<const unsigned short*>(a.scale) + (long long)r * a.ssn + ks0;
        const unsigned short* gz = reinterpret_cast<const unsigned short*>(a.zero) + (long long)r * a.ssn + ks0;
        unsigned short* ss = reinterpret_cast<unsigned short*>(sc) + j * ks_n;
        unsigned short* sz = reinterpret_cast<unsigned short*>(ze) + j * ks_n;
        for (int q = 0; q < ks_n; ++q) {
          ss[q] = __ldg(gs + q);
          sz[q] = __ldg(gz + q);
        }
      }
    }
  } else {
    // x into L2 while the preceding kernel finishes: harmless if that kernel is still writing
    // it (L2 is the point of coherence), and a hit instead of an HBM read after the wait when x
    // was written long before.
    const int lines_per_row = (ks_n * 256 + 127) / 128;
    const int lines = lines_per_row * a.M;
    for (int l = (int)threadIdx.x - 32; l < lines; l += kSlabThreads - 32) {
      const int m = l / lines_per_row, c = l - m * lines_per_row;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const uint8_t*>(a.x + (long long)m * a.sxm +
                                                                                       (long long)ks0 * 128) + c * 128));
    }
  }
  if (sa.sz_mode == 2) __syncthreads();  // scale / zero rows written by plain stores above

  // ---- this warp's units: tiles phase, phase + P, ...; ksteps slot, slot + S, ... of each
  const int S = sa.slots, P = kSlabWarps / S;
  const int slot = warp & (S - 1), phase = warp / S;
  const int per_tile = ks_n / S;  // ksteps of one tile this warp takes (S divides ks_n)
  const int warp_tiles = my_tiles > phase ? (my_tiles - phase + P - 1) / P : 0;
  const int n_units = warp_tiles * per_tile;
  const uint8_t* row_lo0 = stages + grp * sa.pitch + quad * 16;
  auto unit_tile = [&](int u) { return phase + (u / per_tile) * P; };
  auto unit_ks = [&](int u) { return slot + (u % per_tile) * S; };
  auto unpack_unit = [&](SlabFrag& f, int u) {
    const int t = unit_tile(u);
    const uint8_t* st = stages + (size_t)t * sa.stage;
    const unsigned short* sc = reinterpret_cast<const unsigned short*>(st + 16 * sa.pitch);
    const uint8_t* rl = row_lo0 + (size_t)t * sa.stage;
    slab_unpack(f, rl, rl + 8 * sa.pitch, sc, sc + 16 * ks_n, grp, unit_ks(u), ks_n);
  };

  // Before the dependency wait: every tile this warp reads has landed (its weights were
  // requested at entry, so this overlaps the preceding kernel), and the first two units are
  // unpacked into registers.
  bool ok = true;
  for (int t = phase; t < my_tiles && ok; t += P) ok = mbar_spin_bounded(&bars[t], 0);
  SlabFrag f0, f1;
  if (ok && n_units > 0) unpack_unit(f0, 0);
  if (ok && n_units > 1) unpack_unit(f1, 1);
  {
    // Keep the unpack above the dependency wait (the compiler would sink it below to save
    // registers): a branch on every unpacked word, taken only when N < 1 (never), must be
    // evaluated before the wait.
    uint32_t fold = 0u;
#pragma unroll
    for (int i = 0; i < 32; ++i) fold ^= f0.a[i] ^ f1.a[i];
    if (a.N < 1 && fold == 0u) atomicOr(&g_li4_device_error, 0u);
  }

  pdl_wait_primary();  // x (and the residual) come from the preceding kernel
  if (a.split == 1) {
    for (int t = warp; t < my_tiles; t += kSlabWarps) prefetch_residual<FUSED>(a, t_begin + t, lane);
  }
  if (FUSED && a.norm_w != nullptr) {
    if (a.ssq_in != nullptr) rms_from_ssq<kSlabWarps>(a, s_rstd, warp, lane);
    else rms_factors<kSlabWarps>(a, s_rstd, warp, lane);
    __syncthreads();
    slab_stage_x<NT, true>(a, ks0, ks_n, M8, xs, s_rstd);
  } else {
    slab_stage_x<NT, false>(a, ks0, ks_n, M8, xs, s_rstd);
  }
  __syncthreads();

  // ---- tensor-core work on the resident tiles
  const bool bvalid = grp < M8;
  int boff[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) boff[w] = (grp * 4 + quad) * 64 + ((w ^ xs_key(grp, quad)) << 4);
  const int nt_stride = M8 * 256;
  const int ks_stride = NT * nt_stride;
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
  // after unit u: a finished tile's partial goes to red[(t * S + slot) * 16 + r][m]
  auto finish_unit = [&](int u) {
    if (u % per_tile != per_tile - 1) return;
    float* rb = red + (size_t)(unit_tile(u) * S + slot) * 16 * a.M;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = grp + 8 * (e >> 1), m = nt * 8 + 2 * quad + (e & 1);
        if (m < a.M) rb[r * a.M + m] = acc[nt][e];
        acc[nt][e] = 0.f;
      }
  };
  if (ok) {
    if (n_units > 0) {
      slab_mma<NT>(f0, xs + unit_ks(0) * ks_stride, nt_stride, boff, bvalid, acc);
      finish_unit(0);
    }
    if (n_units > 1) {
      slab_mma<NT>(f1, xs + unit_ks(1) * ks_stride, nt_stride, boff, bvalid, acc);
      finish_unit(1);
    }
    for (int u = 2; u < n_units; u += 2) {  // two units in flight: both unpacked, then both multiplied
      const bool two = u + 1 < n_units;
      unpack_unit(f0, u);
      if (two) unpack_unit(f1, u + 1);
      slab_mma<NT>(f0, xs + unit_ks(u) * ks_stride, nt_stride, boff, bvalid, acc);
      finish_unit(u);
      if (two) {
        slab_mma<NT>(f1, xs + unit_ks(u + 1) * ks_stride, nt_stride, boff, bvalid, acc);
        finish_unit(u + 1);
      }
    }
  }
  const bool any_failed = __syncthreads_or(!ok);

  // ---- epilogue: warp w finishes tiles w, w + 8, ...
  for (int t = warp; t < my_tiles; t += kSlabWarps) {
    const int tile = t_begin + t;
    const SlabSum sum{red + (size_t)t * S * 16 * a.M, S, a.M};
    if (a.split == 1) {
      emit_tile<FUSED>(a, tile, lane, 32, sum);
      continue;
    }
    // split-K: this K range's partial of the tile, then the last range to arrive reduces
    const int row0 = tile * 16, rows = min(16, a.N - row0);
    for (int idx = lane; idx < rows * a.M; idx += 32) {
      const int r = idx / a.M, m = idx - r * a.M;
      a.partial[((long long)blockIdx.y * a.M + m) * a.N + row0 + r] = sum(r, m);
    }
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
  // No copy may still be writing this CTA's shared memory when it exits.  On the normal path
  // every stage was waited for (by the warps that read it, before the barrier above); after a
  // failed wait this drains, bounded, what is left.
  if (any_failed && threadIdx.x == 0)
    for (int t = 0; t < my_tiles; ++t) mbar_spin_bounded(&bars[t], 0);
}

size_t slab_smem_bytes(int M, int nt, int ks, int tiles_max, int slots, int pitch) {
  const int m8 = (nt == 1) ? M : 8;
  return (size_t)kSlabBarBytes + (size_t)tiles_max * slab_stage_bytes(ks, pitch) + (size_t)ks * nt * m8 * 256 +
         (size_t)tiles_max * slots * 16 * M * sizeof(float);
}

template <typename KernelT>
static int slab_smem_limit(KernelT kernel, size_t smem) {
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
                                "int4_linear: slab kernel shared-memory limit");
      if (rc == LI4_OK) e.limit = smem;
      return rc;
    }
  const int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "int4_linear: slab kernel shared-memory limit");
  if (rc == LI4_OK) cache.push_back(Entry{(const void*)kernel, dev, smem});
  return rc;
}

int launch_slab(const GemvArgs& a, int nt, bool fused, int grid_x, int tiles_max, int slots, int pitch,
                size_t smem, cudaStream_t stream) {
  SlabArgs sa;
  sa.tiles_max = tiles_max;
  sa.slots = slots;
  sa.pitch = pitch;
  sa.stage = slab_stage_bytes(a.ks_per_split, pitch);
  // scale / zero rows: one block per tile when the tile's rows are back to back and the launch
  // covers all of K; a copy per row when each row is 16-byte aligned; plain loads otherwise
  const unsigned sz_row = (unsigned)a.ks_per_split * 2;
  const bool base_al = aligned16(a.scale) && aligned16(a.zero);
  if (a.split == 1 && a.ssn == a.ks_per_split && base_al && sz_row % 16 == 0) sa.sz_mode = 0;
  else if (base_al && sz_row % 16 == 0 && (a.ssn * 2) % 16 == 0) sa.sz_mode = 1;
  else sa.sz_mode = 2;
  auto kernel = nt == 1 ? (fused ? gemv_slab_kernel<1, true> : gemv_slab_kernel<1, false>)
                        : (fused ? gemv_slab_kernel<2, true> : gemv_slab_kernel<2, false>);
  int rc = slab_smem_limit(kernel, smem);
  if (rc != LI4_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid_x, (unsigned)a.split, 1);
  cfg.blockDim = dim3(kSlabThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, a, sa), "int4_linear: slab kernel launch");
}

int slab_device_errors(unsigned* flags, bool reset) { return tu_device_errors(flags, reset); }

}  // namespace li4
