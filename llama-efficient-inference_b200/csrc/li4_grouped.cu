// li4_grouped.cu -- many independent INT4 GEMVs in one persistent launch, sm_100a.
//
// A decode step's linears depend on each other, so each is its own launch and pays the
// launch-chain latency.  Independent GEMVs (different weights, inputs and outputs) need not:
// here one launch streams all of them.  The work is cut into units of one problem's 128 rows
// (8 warps x 16-row tiles) over its whole K; CTAs take units from a queue -- the first from
// their index, the rest from an atomic counter, largest K first -- so the HBM stream runs from
// the first weight byte to the last without a kernel boundary.  Per unit the CTA stages the
// problem's x once in shared memory (the layout of the streaming kernel), each warp walks its
// tile's ksteps through a register ring D units deep (the first units of the first unit are
// requested before the dependency wait), and the math is the streaming kernel's: exact
// q - zero in fp16, m16n8k16 MMAs with fp32 accumulation per kstep, the group scale in fp32,
// one fp16 rounding per output.
//
// The problems, the unit list and the queue counters live in a caller-owned device table built
// once (li4_int4_linear_grouped_build); a launch then needs no host data and can be captured in
// a CUDA graph.  The last CTA to finish resets the counters.
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
constexpr int kGroupDepth = 5;                 // ring units (16 rows x 128 k) in flight per warp
constexpr int kGroupXBytes = 32768;            // x staging per buffer: M * K * 2 bytes at most
constexpr int kGroupUnitRows = 16 * kGroupWarps;

struct GroupedProblem {
  const __half* x;
  const uint8_t* packed;
  const __half* scale;
  const __half* zero;
  __half* y;
  int N, K;
  long long sxm, spn, ssn, sym;
};

struct GroupedHeader {
  int n_problems, n_units, M, pad0;
  unsigned next;  // units handed out after the first `grid` (queue counter)
  unsigned done;  // CTAs finished (the last one resets both)
  unsigned pad[2];
};

// Table layout: header, problems[n_problems], units[n_units] (problem << 16 | 128-row group).
struct GroupedArgs {
  GroupedHeader* hdr;
  const GroupedProblem* problems;
  const unsigned* units;
  int n_units, M, log2_group;
};

__device__ __forceinline__ GemvArgs grouped_problem_args(const GroupedProblem& p, int M, int log2_group) {
  GemvArgs a = {};
  a.x = p.x;
  a.packed = p.packed;
  a.scale = p.scale;
  a.zero = p.zero;
  a.y = p.y;
  a.M = M;
  a.N = p.N;
  a.K = p.K;
  a.log2_group = log2_group;
  a.sxm = p.sxm;
  a.spn = p.spn;
  a.ssn = p.ssn;
  a.sym = p.sym;
  return a;
}

__global__ void __launch_bounds__(kGroupThreads, 2) gemv_grouped_kernel(const __grid_constant__ GroupedArgs g) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int D = kGroupDepth;
  __shared__ unsigned s_unit[2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 2, quad = lane & 3;
  const int M = g.M;

  // this warp's tile of the first unit: its first D ksteps are requested before the wait
  unsigned unit = blockIdx.x;
  StreamUnit buf[D];
  {
    const unsigned u = g.units[unit];
    const GemvArgs a = grouped_problem_args(g.problems[u >> 16], M, g.log2_group);
    const int tile = (int)(u & 0xFFFFu) * kGroupWarps + warp;
    const int nks = a.K / 128;
    if (tile * 16 < a.N) {
      const StreamRows r = stream_rows(a, tile, 0, grp, quad);
#pragma unroll
      for (int d = 0; d < D; ++d)
        if (d < nks) stream_load(a, buf[d], r, d);
    }
  }
  pdl_launch_dependents();
  pdl_wait_primary();  // the inputs may come from the preceding kernel

  const bool bvalid = grp < M;
  int boff[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) boff[w] = (grp * 4 + quad) * 64 + ((w ^ xs_key(grp, quad)) << 4);
  const int ks_stride = M * 256;
  // (Requesting the next unit's first ksteps during this unit's last ones needs a ring depth that
  // divides K / 128; with a 4-deep ring that measured slower than a 5-deep one without it:
  // 0.209 against 0.197 ms for the 113 Llama-3.2-1B GEMVs.)
  for (int it = 0;; ++it) {
    // the unit after this one, taken now (the atomic's wait hides behind the staging); x of this
    // unit staged into its half of the double buffer
    uint8_t* xs = smem + (it & 1) * kGroupXBytes;
    const unsigned u = g.units[unit];
    const GemvArgs a = grouped_problem_args(g.problems[u >> 16], M, g.log2_group);
    if (threadIdx.x == 0) s_unit[it & 1] = gridDim.x + atomicAdd(&g.hdr->next, 1u);
    stage_x<1, kGroupThreads, false>(a, 0, a.K / 128, M, xs);
    __syncthreads();
    const unsigned next = s_unit[it & 1];

    const int tile = (int)(u & 0xFFFFu) * kGroupWarps + warp;
    const int nks = a.K / 128;
    if (tile * 16 < a.N) {
      const StreamRows r = stream_rows(a, tile, 0, grp, quad);
      if (it > 0) {  // (the first unit's first ksteps were requested before the wait)
#pragma unroll
        for (int d = 0; d < D; ++d)
          if (d < nks) stream_load(a, buf[d], r, d);
      }
      float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
      for (int ks0 = 0; ks0 < nks; ks0 += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
          const int ks = ks0 + d;
          if (ks < nks) {
            stream_compute<1>(buf[d], xs + ks * ks_stride, M * 256, boff, bvalid, acc);
            if (ks + D < nks) stream_load(a, buf[d], r, ks + D);
          }
        }
      }
      emit_warp_tile<false, 1>(a, tile, acc, grp, quad);
    }
    if (next >= (unsigned)g.n_units) break;
    unit = next;
  }
  // the last CTA out resets the queue for the next launch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&g.hdr->done, 1u) == (unsigned)gridDim.x - 1) {
      g.hdr->next = 0u;
      g.hdr->done = 0u;
      __threadfence();
    }
  }
}

// Table layout on the device: header | problems | units.
static size_t grouped_offset_problems() { return (sizeof(GroupedHeader) + 15) & ~size_t(15); }
static size_t grouped_offset_units(int n) { return grouped_offset_problems() + ((size_t)n * sizeof(GroupedProblem) + 15) / 16 * 16; }
static size_t grouped_bytes(int n, int units) { return grouped_offset_units(n) + (size_t)units * sizeof(unsigned); }

static int grouped_check(const li4_gemv_problem* problems, int n, int64_t M, int* units) {
  if (!problems || n < 1 || n > 65535)
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear_grouped: %d problems (1..65535, non-null)", n);
  if (M < 1 || M > 8) return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_grouped: M=%lld (1..8)", (long long)M);
  int64_t total = 0;
  for (int i = 0; i < n; ++i) {
    const li4_gemv_problem& p = problems[i];
    if (!p.x || !p.packed || !p.scale || !p.zero || !p.y)
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear_grouped: problem %d has a null pointer", i);
    if (p.N < 1 || p.K < 128 || p.K % 128 != 0 || p.N > (int64_t(1) << 30))
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear_grouped: problem %d: N=%lld K=%lld (K a multiple of 128)", i,
                       (long long)p.N, (long long)p.K);
    if (M * p.K * 2 > kGroupXBytes)
      return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_grouped: problem %d: M x K = %lld x %lld is above the %d-byte "
                       "x staging", i, (long long)M, (long long)p.K, kGroupXBytes);
    if (p.stride_xm < p.K || p.stride_pn < p.K / 2 || p.stride_sn < p.K / 128 || p.stride_ym < p.N)
      return set_error(LI4_ERR_INVALID_ARG, "int4_linear_grouped: problem %d: row strides smaller than the rows", i);
    if (!aligned16(p.packed) || p.stride_pn % 16 != 0)
      return set_error(LI4_ERR_ALIGNMENT, "int4_linear_grouped: problem %d: packed rows must start on 16-byte "
                       "boundaries", i);
    if ((reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.y) | reinterpret_cast<uintptr_t>(p.scale) |
         reinterpret_cast<uintptr_t>(p.zero)) & 1u)
      return set_error(LI4_ERR_ALIGNMENT, "int4_linear_grouped: problem %d: fp16 tensors must be 2-byte aligned", i);
    const int64_t groups = (p.N + kGroupUnitRows - 1) / kGroupUnitRows;
    if (groups > 65536)
      return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_grouped: problem %d: N=%lld above %d rows", i,
                       (long long)p.N, 65536 * kGroupUnitRows);
    total += groups;
  }
  if (total > (int64_t(1) << 30)) return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_grouped: too many units");
  *units = (int)total;
  return LI4_OK;
}

static int grouped_grid(int units, int* grid) {
  static std::mutex mu;
  static std::vector<std::pair<int, int>> cache;  // (device, CTAs per SM)
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "int4_linear_grouped: cudaGetDevice");
  if (rc != LI4_OK) return rc;
  const size_t smem = 2 * (size_t)kGroupXBytes;
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
  *grid = std::min(units, occ * current_sm_count());
  return LI4_OK;
}

}  // namespace li4

extern "C" size_t li4_int4_linear_grouped_table_bytes(const li4_gemv_problem* problems, int n, int64_t M, int* units) {
  int u = 0;
  if (li4::grouped_check(problems, n, M, &u) != LI4_OK) return 0;
  if (units) *units = u;
  li4::clear_error();
  return li4::grouped_bytes(n, u);
}

extern "C" int li4_int4_linear_grouped_build(const li4_gemv_problem* problems, int n, int64_t M, int64_t group_size,
                                             void* table, size_t table_bytes) {
  using namespace li4;
  if (group_size != 128)
    return set_error(LI4_ERR_UNSUPPORTED, "int4_linear_grouped: group_size=%lld (128)", (long long)group_size);
  int units = 0;
  int rc = grouped_check(problems, n, M, &units);
  if (rc != LI4_OK) return rc;
  const size_t bytes = grouped_bytes(n, units);
  if (!table || table_bytes < bytes || !aligned16(table))
    return set_error(LI4_ERR_WORKSPACE, "int4_linear_grouped: a 16-byte aligned table of %zu bytes is needed (got %zu)",
                     bytes, table ? table_bytes : (size_t)0);
  std::vector<uint8_t> host(bytes, 0);
  GroupedHeader h = {};
  h.n_problems = n;
  h.n_units = units;
  h.M = (int)M;
  memcpy(host.data(), &h, sizeof(h));
  GroupedProblem* gp = reinterpret_cast<GroupedProblem*>(host.data() + grouped_offset_problems());
  for (int i = 0; i < n; ++i) {
    const li4_gemv_problem& p = problems[i];
    gp[i] = GroupedProblem{static_cast<const __half*>(p.x), static_cast<const uint8_t*>(p.packed),
                           static_cast<const __half*>(p.scale), static_cast<const __half*>(p.zero),
                           static_cast<__half*>(p.y), (int)p.N, (int)p.K, p.stride_xm, p.stride_pn, p.stride_sn,
                           p.stride_ym};
  }
  // units: largest K first (the long units start early, the short ones fill the tail), then in order
  std::vector<int> order(n);
  for (int i = 0; i < n; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return problems[a].K > problems[b].K; });
  unsigned* up = reinterpret_cast<unsigned*>(host.data() + grouped_offset_units(n));
  int k = 0;
  for (int i : order) {
    const int64_t groups = (problems[i].N + kGroupUnitRows - 1) / kGroupUnitRows;
    for (int64_t gi = 0; gi < groups; ++gi) up[k++] = ((unsigned)i << 16) | (unsigned)gi;
  }
  rc = check_cuda(cudaMemcpy(table, host.data(), bytes, cudaMemcpyHostToDevice), "int4_linear_grouped: table upload");
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_int4_linear_grouped(const void* table, int n, int units, int64_t M, void* stream) {
  using namespace li4;
  if (!table || n < 1 || units < 1 || M < 1 || M > 8)
    return set_error(LI4_ERR_INVALID_ARG, "int4_linear_grouped: table=%p n=%d units=%d M=%lld", table, n, units,
                     (long long)M);
  int grid = 0;
  int rc = grouped_grid(units, &grid);
  if (rc != LI4_OK) return rc;
  uint8_t* base = static_cast<uint8_t*>(const_cast<void*>(table));
  GroupedArgs g;
  g.hdr = reinterpret_cast<GroupedHeader*>(base);
  g.problems = reinterpret_cast<const GroupedProblem*>(base + grouped_offset_problems());
  g.units = reinterpret_cast<const unsigned*>(base + grouped_offset_units(n));
  g.n_units = units;
  g.M = (int)M;
  g.log2_group = 7;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kGroupThreads, 1, 1);
  cfg.dynamicSmemBytes = 2 * (size_t)kGroupXBytes;
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
