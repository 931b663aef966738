// li4_grouped.cu -- many independent INT4 GEMVs in one persistent launch, sm_100a.
//
// A decode step's linears depend on each other, so each is its own launch and pays the
// launch-chain latency.  Independent GEMVs (different weights, inputs and outputs) need not:
// here one launch streams all of them.  The problems' 16-row tiles, in problem order, are cut
// into contiguous ranges of about equal weight bytes, one per CTA of a full wave (two CTAs per
// SM); a range stages the x of the few problems it touches once, and each of its 8 warps takes
// tiles w, w + 8, ... of the range and streams their (tile, kstep) units through ONE register
// ring D units deep that runs on across tile and problem boundaries -- the next tile's first
// weights are in flight while the last ksteps of the current one are computed, and nothing
// waits on a barrier between tiles.  The first units are requested before the dependency wait.
// Math: m16n8k16 MMAs on the biased unpack below (1024 + q halves straight from the LOP3, the
// zero and the bias taken off in fp32 per kstep), fp32 accumulation, the group scale in fp32, one
// fp16 rounding per output.
//
// The problems and the ranges live in a caller-owned device table built once
// (li4_int4_linear_grouped_build); a launch needs no host data, writes nothing but the outputs
// and can be repeated or captured in a CUDA graph.
#include "li4_common.cuh"
#include "li4_gemv_device.cuh"
#include "li4_internal.h"

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

namespace li4 {

constexpr int kGroupWarps = 8;
constexpr int kGroupThreads = kGroupWarps * 32;
constexpr int kGroupDepth = 4;                 // ring units (16 rows x 128 k) in flight per warp
constexpr int kGroupProblemX = 32768;          // x of one problem: M * K * 2 bytes at most
constexpr int kGroupXBytes = 65536;            // x staging of one range (all its problems)
constexpr int kGroupRangeProblems = 16;        // problems one range may touch
constexpr int kGroupMinRangeUnits = 64;        // a range moves at least ~64 KB of weights
constexpr int kGroupCtasPerSm = 2;

struct GroupedProblem {
  const __half* x;
  const uint8_t* packed;
  const __half* scale;
  const __half* zero;
  __half* y;
  int N, K;
  long long sxm, spn, ssn, sym;
  int tile0;  // first flattened 16-row tile of this problem
  int pad;
};

struct GroupedHeader {
  int n_problems, n_ranges, M, pad;
};

// One CTA's work: flattened tiles [t0, t1), of problems p0 .. p1.
struct GroupedRange {
  int t0, t1, p0, p1;
};

// Table layout: header, problems[n_problems], ranges[n_ranges].
struct GroupedArgs {
  const GroupedProblem* problems;
  const GroupedRange* ranges;
  int n_ranges, M;
};

__device__ __forceinline__ GemvArgs grouped_problem_args(const GroupedProblem& p, int M) {
  GemvArgs a = {};
  a.x = p.x;
  a.packed = p.packed;
  a.scale = p.scale;
  a.zero = p.zero;
  a.y = p.y;
  a.M = M;
  a.N = p.N;
  a.K = p.K;
  a.log2_group = 7;
  a.sxm = p.sxm;
  a.spn = p.spn;
  a.ssn = p.ssn;
  a.sym = p.sym;
  return a;
}

// Staging of one problem's x in a range: the permuted x (the streaming kernel's layout, odd-k halves
// scaled by 1/16), then per kstep and row m < 8 the sums the biased unpack needs (float2 [ks][8]).
__host__ __device__ inline int grouped_x_bytes(int K, int M) {
  return (((K / 128) * M * 256 + 127) & ~127) + (K / 128) * 8 * (int)sizeof(float2);
}
__host__ __device__ inline int grouped_sums_offset(int K, int M) { return ((K / 128) * M * 256 + 127) & ~127; }

// ---------------------------------------------------------------------------
// Biased unpack.  The exact unpack of the other kernels forms q - z in fp16 with a LOP3 and a
// half2 subtract / FMA per pair of nibbles (9 instructions per 8 weights).  Here the MMA takes the
// magic-number halves as they come out of the LOP3 -- 1024 + q for a low nibble (even k) and
// 1024 + 16 q for a high nibble (odd k), both exact in fp16 -- against x with its odd-k entries
// scaled by 1/16 (exact for |x| >= 2^-10), so a unit costs 5 instructions per 8 weights, and the
// bias comes off in fp32 afterwards:
//   sum_k (q_k - z) x_k = C - P - z Q,  C = the MMA result,
//   P = 1024 (S_even + S'_odd),  Q = S_even + 16 S'_odd,
// with S_even the kstep's even-k x and S'_odd its scaled odd-k x, summed in fp32 at staging.
// C carries the bias (about 1024 |x| per term), so the fp32 sums of a unit lose ~10 bits to the
// cancellation: absolute errors of ~1e-3 per unit before the group scale, far inside the
// acceptance bound.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grouped_stage_x(const GemvArgs& a, int M, uint8_t* xs, float2* sums) {
  const int nks = a.K / 128;
  const __half2 inv16 = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(a.x) & 15u) == 0) && ((a.sxm & 7) == 0);
  for (int i = threadIdx.x; i < nks * 8; i += kGroupThreads)  // rows past M read as zero sums
    if ((i & 7) >= M) sums[i] = make_float2(0.f, 0.f);
  // item (ks, m, j), j = 16-byte chunk of the kstep (quad * 4 + w) fastest: the 16 chunks of one
  // (kstep, row) sit on 16 consecutive lanes, which sum them with a fixed butterfly
  const int items = nks * M * 16;
  for (int base = 0; base < items; base += kGroupThreads) {
    const int i = base + (int)threadIdx.x;
    const bool live = i < items;
    const int j = i & 15, km = i >> 4;
    const int ks = km / M, m = km - ks * M;
    const int quad = j >> 2, w = j & 3;
    float se = 0.f, so = 0.f;
    if (live) {
      const __half* src = a.x + (long long)m * a.sxm + ks * 128 + 32 * quad + 8 * w;
      uint32_t u[4];
      if (vec_ok) {
        const uint4 v = *reinterpret_cast<const uint4*>(src);
        u[0] = v.x; u[1] = v.y; u[2] = v.z; u[3] = v.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          u[e] = (uint32_t)__half_as_ushort(src[2 * e]) | ((uint32_t)__half_as_ushort(src[2 * e + 1]) << 16);
      }
      uint4 out;
      out.x = __byte_perm(u[0], u[2], 0x5410);                                     // (x0, x4)
      out.y = h2_as_u32(__hmul2(u32_as_h2(__byte_perm(u[0], u[2], 0x7632)), inv16));  // (x1, x5) / 16
      out.z = __byte_perm(u[1], u[3], 0x5410);                                     // (x2, x6)
      out.w = h2_as_u32(__hmul2(u32_as_h2(__byte_perm(u[1], u[3], 0x7632)), inv16));  // (x3, x7) / 16
      const float2 e0 = __half22float2(u32_as_h2(out.x)), e1 = __half22float2(u32_as_h2(out.z));
      const float2 o0 = __half22float2(u32_as_h2(out.y)), o1 = __half22float2(u32_as_h2(out.w));
      se = (e0.x + e0.y) + (e1.x + e1.y);
      so = (o0.x + o0.y) + (o1.x + o1.y);
      *reinterpret_cast<uint4*>(xs + xs_chunk_offset((ks * M + m) * 4 + quad, w, m)) = out;
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      se += __shfl_xor_sync(0xffffffffu, se, o);
      so += __shfl_xor_sync(0xffffffffu, so, o);
    }
    if (live && j == 0) sums[ks * 8 + m] = make_float2(1024.f * (se + so), se + 16.f * so);
  }
}

// acc += s * sum_k (q - z) x over one 16-row x 128-k unit with the biased unpack; sums_ks: the
// kstep's (P, Q) for rows 0..7 of x.
__device__ __forceinline__ void grouped_compute(const StreamUnit& u, const uint8_t* xs_ks, const float2* sums_ks,
                                                const int boff[4], bool bvalid, int quad, float acc[4]) {
  constexpr uint32_t MAGIC = 0x64006400u;
  float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t wl = (w == 0) ? u.lo.x : (w == 1) ? u.lo.y : (w == 2) ? u.lo.z : u.lo.w;
    const uint32_t wh = (w == 0) ? u.hi.x : (w == 1) ? u.hi.y : (w == 2) ? u.hi.z : u.hi.w;
    const uint32_t wl8 = wl >> 8, wh8 = wh >> 8;
    uint4 bq = make_uint4(0u, 0u, 0u, 0u);
    if (bvalid) bq = lds128(xs_ks + boff[w]);
    mma_16816(c, lop3_and_or(wl, 0x000F000Fu, MAGIC), lop3_and_or(wh, 0x000F000Fu, MAGIC),
              lop3_and_or(wl, 0x00F000F0u, MAGIC), lop3_and_or(wh, 0x00F000F0u, MAGIC), bq.x, bq.y);
    mma_16816(c, lop3_and_or(wl8, 0x000F000Fu, MAGIC), lop3_and_or(wh8, 0x000F000Fu, MAGIC),
              lop3_and_or(wl8, 0x00F000F0u, MAGIC), lop3_and_or(wh8, 0x00F000F0u, MAGIC), bq.z, bq.w);
  }
  const float4 pq = *reinterpret_cast<const float4*>(sums_ks + 2 * quad);  // (P, Q) of x rows 2 quad, 2 quad + 1
  const float sl = __half2float(__ushort_as_half((unsigned short)(u.sz_lo & 0xFFFFu)));
  const float sh = __half2float(__ushort_as_half((unsigned short)(u.sz_hi & 0xFFFFu)));
  const float zl = __half2float(__ushort_as_half((unsigned short)(u.sz_lo >> 16)));
  const float zh = __half2float(__ushort_as_half((unsigned short)(u.sz_hi >> 16)));
  acc[0] = fmaf(sl, fmaf(-zl, pq.y, c[0] - pq.x), acc[0]);
  acc[1] = fmaf(sl, fmaf(-zl, pq.w, c[1] - pq.z), acc[1]);
  acc[2] = fmaf(sh, fmaf(-zh, pq.y, c[2] - pq.x), acc[2]);
  acc[3] = fmaf(sh, fmaf(-zh, pq.w, c[3] - pq.z), acc[3]);
}

// A warp's walk over its (tile, kstep) units of one range: tiles first, first + 8, ... < end.
struct GroupCursor {
  int tile;       // flattened tile (>= end: done)
  int ks, nks;    // kstep and ksteps of the tile's problem
  int p;          // problem of `tile`
  int tile0;      // its first flattened tile
  int tile_end;   // one past its last
  int xoff;       // its x in the range's staging
  int sums;       // its (P, Q) sums, bytes after xoff
  StreamRows rows;
};

__device__ __forceinline__ void cursor_problem(GroupCursor& c, const GroupedArgs& g, int M) {
  const GroupedProblem& pr = g.problems[c.p];
  c.tile0 = pr.tile0;
  c.nks = pr.K / 128;
  c.tile_end = pr.tile0 + (pr.N + 15) / 16;
  c.sums = grouped_sums_offset(pr.K, M);
}

__device__ __forceinline__ void cursor_rows(GroupCursor& c, const GroupedArgs& g, int M, int grp, int quad) {
  const GemvArgs a = grouped_problem_args(g.problems[c.p], M);
  c.rows = stream_rows(a, c.tile - c.tile0, 0, grp, quad);
}

// Move to the warp's next tile (8 tiles on), crossing into later problems of the range.
__device__ __forceinline__ void cursor_next_tile(GroupCursor& c, const GroupedArgs& g, int M, int end, int grp,
                                                 int quad) {
  c.tile += kGroupWarps;
  c.ks = 0;
  if (c.tile >= end) return;
  while (c.tile >= c.tile_end) {
    c.xoff += grouped_x_bytes(c.nks * 128, M);
    ++c.p;
    cursor_problem(c, g, M);
  }
  cursor_rows(c, g, M, grp, quad);
}

__device__ __forceinline__ void cursor_advance(GroupCursor& c, const GroupedArgs& g, int M, int end, int grp,
                                               int quad) {
  if (++c.ks == c.nks) cursor_next_tile(c, g, M, end, grp, quad);
}

__device__ __forceinline__ void group_load(StreamUnit& u, const GroupCursor& c) {
  u.lo = ldg_stream_v4(c.rows.p_lo + c.ks * 64);
  u.hi = ldg_stream_v4(c.rows.p_hi + c.ks * 64);
  u.sz_lo = ldg_u16(c.rows.s_lo + c.ks) | (ldg_u16(c.rows.z_lo + c.ks) << 16);
  u.sz_hi = ldg_u16(c.rows.s_hi + c.ks) | (ldg_u16(c.rows.z_hi + c.ks) << 16);
}

__global__ void __launch_bounds__(kGroupThreads, kGroupCtasPerSm) gemv_grouped_kernel(const __grid_constant__ GroupedArgs g) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int D = kGroupDepth;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 2, quad = lane & 3;
  const int M = g.M;
  const bool bvalid = grp < M;
  int boff[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) boff[w] = (grp * 4 + quad) * 64 + ((w ^ xs_key(grp, quad)) << 4);
  const int nt_stride = M * 256;

  for (int ri = blockIdx.x; ri < g.n_ranges; ri += gridDim.x) {
    const GroupedRange R = g.ranges[ri];
    const bool first = ri == (int)blockIdx.x;
    // this warp's units: the load cursor runs D units ahead of the compute cursor
    GroupCursor cc;
    cc.tile = R.t0 + warp;
    cc.ks = 0;
    cc.p = R.p0;
    cc.xoff = 0;
    cc.nks = 1;
    if (cc.tile < R.t1) {
      cursor_problem(cc, g, M);
      while (cc.tile >= cc.tile_end) {
        cc.xoff += grouped_x_bytes(cc.nks * 128, M);
        ++cc.p;
        cursor_problem(cc, g, M);
      }
      cursor_rows(cc, g, M, grp, quad);
    }
    GroupCursor lc = cc;
    StreamUnit buf[D];
#pragma unroll
    for (int d = 0; d < D; ++d)
      if (lc.tile < R.t1) {
        group_load(buf[d], lc);
        cursor_advance(lc, g, M, R.t1, grp, quad);
      }
    if (first) {
      pdl_launch_dependents();
      pdl_wait_primary();  // the inputs may come from the preceding kernel
    } else {
      __syncthreads();  // every warp is done with the previous range's x
    }
    // x of the range's problems, back to back in the staging layout of the streaming kernel
    {
      int off = 0;
      for (int p = R.p0; p <= R.p1; ++p) {
        const GemvArgs a = grouped_problem_args(g.problems[p], M);
        grouped_stage_x(a, M, smem + off, reinterpret_cast<float2*>(smem + off + grouped_sums_offset(a.K, M)));
        off += grouped_x_bytes(a.K, M);
      }
    }
    __syncthreads();

    float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    while (cc.tile < R.t1) {
#pragma unroll
      for (int d = 0; d < D; ++d) {
        if (cc.tile >= R.t1) break;
        grouped_compute(buf[d], smem + cc.xoff + cc.ks * nt_stride,
                        reinterpret_cast<const float2*>(smem + cc.xoff + cc.sums) + cc.ks * 8, boff, bvalid, quad,
                        acc[0]);
        if (lc.tile < R.t1) {
          group_load(buf[d], lc);
          cursor_advance(lc, g, M, R.t1, grp, quad);
        }
        if (cc.ks == cc.nks - 1) {  // the tile is complete
          const GemvArgs a = grouped_problem_args(g.problems[cc.p], M);
          emit_warp_tile<false, 1>(a, cc.tile - cc.tile0, acc, grp, quad);
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[0][e] = 0.f;
        }
        cursor_advance(cc, g, M, R.t1, grp, quad);
      }
    }
  }
}

// Table layout on the device: header | problems | ranges.
static size_t grouped_offset_problems() { return (sizeof(GroupedHeader) + 15) & ~size_t(15); }
static size_t grouped_offset_ranges(int n) { return grouped_offset_problems() + ((size_t)n * sizeof(GroupedProblem) + 15) / 16 * 16; }
static size_t grouped_bytes(int n, int ranges) { return grouped_offset_ranges(n) + (size_t)ranges * sizeof(GroupedRange); }

static int grouped_check(const li4_gemv_problem* problems, int n, int64_t M) {
  if (!problems || n < 1 || n > 65535)
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear_grouped: %d problems (1..65535, non-null)", n);
  if (M < 1 || M > 8) return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_grouped: M=%lld (1..8)", (long long)M);
  int64_t tiles = 0;
  for (int i = 0; i < n; ++i) {
    const li4_gemv_problem& p = problems[i];
    if (!p.x || !p.packed || !p.scale || !p.zero || !p.y)
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear_grouped: problem %d has a null pointer", i);
    if (p.N < 1 || p.K < 128 || p.K % 128 != 0 || p.N > (int64_t(1) << 30))
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear_grouped: problem %d: N=%lld K=%lld (K a multiple of 128)", i,
                       (long long)p.N, (long long)p.K);
    if (M * p.K * 2 > kGroupProblemX)
      return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_grouped: problem %d: M x K = %lld x %lld is above the %d-byte "
                       "x staging", i, (long long)M, (long long)p.K, kGroupProblemX);
    if (p.stride_xm < p.K || p.stride_pn < p.K / 2 || p.stride_sn < p.K / 128 || p.stride_ym < p.N)
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear_grouped: problem %d: row strides smaller than the rows", i);
    if (!aligned16(p.packed) || p.stride_pn % 16 != 0)
      return set_error(LI4_ERR_ALIGNMENT, "int4_linear_grouped: problem %d: packed rows must start on 16-byte "
                       "boundaries", i);
    if ((reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.y) | reinterpret_cast<uintptr_t>(p.scale) |
         reinterpret_cast<uintptr_t>(p.zero)) & 1u)
      return set_error(LI4_ERR_ALIGNMENT, "int4_linear_grouped: problem %d: fp16 tensors must be 2-byte aligned", i);
    tiles += (p.N + 15) / 16;
  }
  if (tiles > (int64_t(1) << 30)) return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_grouped: too many row tiles");
  return LI4_OK;
}

// CTAs of one full wave on the current device (the SM count of a B200 where no device answers).
static int grouped_wave() {
  const int sm = current_sm_count();
  return kGroupCtasPerSm * (sm > 0 ? sm : 148);
}

// The flattened tiles cut into ranges of about equal weight bytes (a tile of problem p costs its
// K / 128 ksteps), about one per CTA of a wave -- fewer for small lists, so that a range moves at
// least kGroupMinRangeUnits ksteps -- and each range cut again where its problems' x would pass
// the staging limit or their count kGroupRangeProblems.  Deterministic: the same list and device
// give the same ranges.
static std::vector<GroupedRange> grouped_ranges(const li4_gemv_problem* problems, int n, int64_t M,
                                                std::vector<int>* tile0) {
  tile0->assign(n, 0);
  int64_t total = 0;
  int tiles = 0;
  for (int i = 0; i < n; ++i) {
    (*tile0)[i] = tiles;
    const int t = (int)((problems[i].N + 15) / 16);
    tiles += t;
    total += (int64_t)t * (problems[i].K / 128);
  }
  // Range size: the wave's share of the ksteps, rounded up to a multiple of 512 (eight 16-row
  // tiles of K = 8192, or 32 of K = 2048), so that a range of a long-K problem holds whole groups
  // of 8 tiles -- the same number per warp: the Llama-3.2-1B step's 33-tile down_proj ranges gave
  // some warps 5 tiles and others 4, and the slowest range sets the launch's time.
  const int64_t wave = grouped_wave();
  int64_t target = std::max<int64_t>(kGroupMinRangeUnits, (total + wave - 1) / wave);
  if (target >= 512) target = (target + 511) / 512 * 512;
  std::vector<GroupedRange> out;
  GroupedRange cur = {0, 0, 0, 0};
  int64_t cost = 0;        // cost of the tiles before the current one
  int64_t xbytes = 0;      // x staging of the current range
  int part = 0;            // index of the current cost part
  bool open = false;
  for (int p = 0; p < n; ++p) {
    const int nt = (int)((problems[p].N + 15) / 16);
    const int64_t c = problems[p].K / 128;
    const int64_t xb = grouped_x_bytes((int)problems[p].K, (int)M);
    for (int t = 0; t < nt; ++t) {
      const int ft = (*tile0)[p] + t;
      // the part this tile falls in: where its cost starts
      const int tp = (int)(cost / target);
      const bool new_problem = open && cur.p1 != p;
      const bool cut = open && (tp != part || (new_problem && (xbytes + xb > kGroupXBytes ||
                                                               p - cur.p0 + 1 > kGroupRangeProblems)));
      if (cut) {
        out.push_back(cur);
        open = false;
      }
      if (!open) {
        cur = GroupedRange{ft, ft, p, p};
        xbytes = xb;
        part = tp;
        open = true;
      } else if (new_problem) {
        cur.p1 = p;
        xbytes += xb;
      }
      cur.t1 = ft + 1;
      cost += c;
    }
  }
  if (open) out.push_back(cur);
  return out;
}

static int grouped_grid(int ranges, int* grid) {
  static std::mutex mu;
  static std::vector<std::pair<int, int>> cache;  // (device, CTAs per SM)
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "int4_linear_grouped: cudaGetDevice");
  if (rc != LI4_OK) return rc;
  const size_t smem = kGroupXBytes;
  std::lock_guard<std::mutex> lock(mu);
  int occ = 0;
  for (auto& e : cache)
    if (e.first == dev) occ = e.second;
  if (occ == 0) {
    rc = check_cuda(cudaFuncSetAttribute(gemv_grouped_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                    "int4_linear_grouped: cudaFuncSetAttribute");
    if (rc != LI4_OK) return rc;
    rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_grouped_kernel, kGroupThreads, smem),
                    "int4_linear_grouped: occupancy");
    if (rc != LI4_OK) return rc;
    if (occ < 1) return set_error(LI4_ERR_CUDA, "int4_linear_grouped: the kernel does not fit on an SM");
    cache.emplace_back(dev, occ);
  }
  *grid = std::min(ranges, occ * current_sm_count());
  return LI4_OK;
}

}  // namespace li4

extern "C" size_t li4_int4_linear_grouped_table_bytes(const li4_gemv_problem* problems, int n, int64_t M, int* units) {
  if (li4::grouped_check(problems, n, M) != LI4_OK) return 0;
  std::vector<int> tile0;
  const std::vector<li4::GroupedRange> ranges = li4::grouped_ranges(problems, n, M, &tile0);
  if (units) *units = (int)ranges.size();
  li4::clear_error();
  return li4::grouped_bytes(n, (int)ranges.size());
}

extern "C" int li4_int4_linear_grouped_build(const li4_gemv_problem* problems, int n, int64_t M, int64_t group_size,
                                             void* table, size_t table_bytes) {
  using namespace li4;
  if (group_size != 128)
    return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_grouped: group_size=%lld (128)", (long long)group_size);
  int rc = grouped_check(problems, n, M);
  if (rc != LI4_OK) return rc;
  std::vector<int> tile0;
  const std::vector<GroupedRange> ranges = grouped_ranges(problems, n, M, &tile0);
  const size_t bytes = grouped_bytes(n, (int)ranges.size());
  if (!table || table_bytes < bytes || !aligned16(table))
    return set_error(LI4_ERR_WORKSPACE, "int4_linear_grouped: a 16-byte aligned table of %zu bytes is needed (got %zu)",
                     bytes, table ? table_bytes : (size_t)0);
  std::vector<uint8_t> host(bytes, 0);
  GroupedHeader h = {};
  h.n_problems = n;
  h.n_ranges = (int)ranges.size();
  h.M = (int)M;
  memcpy(host.data(), &h, sizeof(h));
  GroupedProblem* gp = reinterpret_cast<GroupedProblem*>(host.data() + grouped_offset_problems());
  for (int i = 0; i < n; ++i) {
    const li4_gemv_problem& p = problems[i];
    gp[i] = GroupedProblem{static_cast<const __half*>(p.x), static_cast<const uint8_t*>(p.packed),
                           static_cast<const __half*>(p.scale), static_cast<const __half*>(p.zero),
                           static_cast<__half*>(p.y), (int)p.N, (int)p.K, p.stride_xm, p.stride_pn, p.stride_sn,
                           p.stride_ym, tile0[i], 0};
  }
  memcpy(host.data() + grouped_offset_ranges(n), ranges.data(), ranges.size() * sizeof(GroupedRange));
  rc = check_cuda(cudaMemcpy(table, host.data(), bytes, cudaMemcpyHostToDevice), "int4_linear_grouped: table upload");
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_int4_linear_grouped(const void* table, int n, int units, int64_t M, void* stream) {
  using namespace li4;
  if (!table || n < 1 || units < 1 || M < 1 || M > 8)
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear_grouped: table=%p n=%d ranges=%d M=%lld", table, n, units,
                     (long long)M);
  int grid = 0;
  int rc = grouped_grid(units, &grid);
  if (rc != LI4_OK) return rc;
  const uint8_t* base = static_cast<const uint8_t*>(table);
  GroupedArgs g;
  g.problems = reinterpret_cast<const GroupedProblem*>(base + grouped_offset_problems());
  g.ranges = reinterpret_cast<const GroupedRange*>(base + grouped_offset_ranges(n));
  g.n_ranges = units;
  g.M = (int)M;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kGroupThreads, 1, 1);
  cfg.dynamicSmemBytes = kGroupXBytes;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  rc = check_cuda(cudaLaunchKernelEx(&cfg, gemv_grouped_kernel, g), "int4_linear_grouped: kernel launch");
  if (rc == LI4_OK) clear_error();
  return rc;
}
