// li4_comm.cu -- one-shot all-reduce + residual add over NVLink peer memory, sm_100a.
//
// Tensor-parallel decode all-reduces a [batch, dim] fp16 partial after every
// row-parallel linear (wo, w2) and then adds the residual
// (h = x + allreduce(wo(...)), llama/model.py:358-362 under tensor
// parallelism).  The messages are small (4-64 KiB), so the cost is latency,
// not bandwidth: NCCL's ring / tree steps each cross the switch.  Here every
// rank's GEMV writes its partial straight into a buffer that all ranks have
// mapped (CUDA IPC), and one kernel per rank
//   1. raises its flag in every peer's flag array (system-scope release, which
//      orders the partial the preceding kernel wrote before the flag),
//   2. waits (bounded) until every peer's flag is up (system-scope acquire),
//   3. reads all partials of its slice over NVLink, sums them in fp32 in rank
//      order and writes fp16(residual + fp16(sum)).
// Each call uses the next slot of two, so a rank never overwrites a partial
// that a peer may still be reading: a peer reaches call k+1's flags only after
// finishing call k.  Flags carry a per-CTA call count kept on the device, so
// the kernel can be captured once in a CUDA graph and replayed.  A wait that
// runs out sets bit 1 of the device error word and the kernel carries on.
#include "li4_common.cuh"
#include "li4_internal.h"

#include <cstring>

namespace li4 {

__device__ unsigned g_comm_device_error;  // bit 1 of li4_device_errors

int comm_device_errors(unsigned* flags, bool reset) {
  int rc = check_cuda(cudaMemcpyFromSymbol(flags, g_comm_device_error, sizeof(unsigned)), "device_errors: comm flags");
  if (rc == LI4_OK && reset) {
    const unsigned zero = 0;
    rc = check_cuda(cudaMemcpyToSymbol(g_comm_device_error, &zero, sizeof(unsigned)), "device_errors: clearing");
  }
  return rc;
}

constexpr int kArThreads = 256;
constexpr int kArMaxRanks = 8;
constexpr unsigned kArWaitLimit = 1u << 22;  // polls of a peer flag before giving up (about a second)
__device__ unsigned g_ar_wait_limit = kArWaitLimit;  // li4_debug_set_wait_limits shortens it for tests

int comm_set_wait_limit(unsigned polls) {
  const unsigned v = polls ? polls : kArWaitLimit;
  return check_cuda(cudaMemcpyToSymbol(g_ar_wait_limit, &v, sizeof(v)), "debug_set_wait_limits: all-reduce");
}

struct ArArgs {
  const __half* slots[kArMaxRanks];  // this call's slot on every rank (peer pointers)
  unsigned* flags[kArMaxRanks];      // every rank's flag array [ctas][ranks]
  unsigned* counts;                  // this rank's per-CTA call counts [ctas]
  const __half* residual;
  __half* out;
  long long n;
  int world, rank;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kArThreads) allreduce_add_kernel(const __grid_constant__ ArArgs a) {
  __shared__ unsigned s_epoch;
  const int c = blockIdx.x, C = gridDim.x;
  pdl_launch_dependents();
  pdl_wait_primary();  // this rank's partial was written by the preceding kernel
  // The partial was written by the preceding kernel, whose writes griddepcontrol.wait made visible
  // to this grid; the flag's system-scope release below orders them before the flag for the peers.
  // (A separate fence.sc.sys here measured 14.0 against 9.4 us per call on two B200s.)
  if (threadIdx.x == 0) s_epoch = a.counts[c] + 1;
  __syncthreads();
  const unsigned epoch = s_epoch;
  if (threadIdx.x < a.world) {  // raise our flag in rank t's array, then wait for rank t's flag in ours
    const int t = threadIdx.x;
    st_release_sys(a.flags[t] + c * a.world + a.rank, epoch);
    const unsigned* mine = a.flags[a.rank] + c * a.world + t;
    const unsigned limit = g_ar_wait_limit;
    unsigned i = 0;
    while ((int)(ld_acquire_sys(mine) - epoch) < 0) {
      if (++i == limit) {
        atomicOr(&g_comm_device_error, 2u);
        break;
      }
    }
  }
  __syncthreads();
  // this CTA's slice, 8 halves per step where aligned
  const long long per = ((a.n + C - 1) / C + 7) / 8 * 8;
  const long long e0 = (long long)c * per, e1 = min(a.n, e0 + per);
  for (long long e = e0 + 8LL * threadIdx.x; e < e1; e += 8LL * kArThreads) {
    if (e + 8 <= e1) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < a.world; ++r) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(a.slots[r] + e));  // L2 / NVLink, never a stale L1 line
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[q]));
          acc[2 * q] += f.x;
          acc[2 * q + 1] += f.y;
        }
      }
      const uint4 ru = *reinterpret_cast<const uint4*>(a.residual + e);
      const uint32_t rw[4] = {ru.x, ru.y, ru.z, ru.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 rf = __half22float2(*reinterpret_cast<const __half2*>(&rw[q]));
        const float2 sf = __half22float2(__floats2half2_rn(acc[2 * q], acc[2 * q + 1]));
        const __half2 h = __floats2half2_rn(rf.x + sf.x, rf.y + sf.y);
        o[q] = *reinterpret_cast<const uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(a.out + e) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
      for (long long i = e; i < e1; ++i) {
        float acc = 0.f;
        for (int r = 0; r < a.world; ++r) acc += __half2float(__ldcg(a.slots[r] + i));
        a.out[i] = __float2half_rn(__half2float(a.residual[i]) + __half2float(__float2half_rn(acc)));
      }
    }
  }
  if (threadIdx.x == 0) a.counts[c] = epoch;
}

}  // namespace li4

extern "C" int li4_comm_alloc(size_t bytes, void** dev_ptr) {
  using namespace li4;
  if (!dev_ptr || bytes == 0) return set_error(LI4_ERR_INVALID_ARG, "comm_alloc: null output or zero size");
  *dev_ptr = nullptr;
  int rc = check_cuda(cudaMalloc(dev_ptr, bytes), "comm_alloc: cudaMalloc");
  if (rc == LI4_OK) rc = check_cuda(cudaMemset(*dev_ptr, 0, bytes), "comm_alloc: cudaMemset");
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_comm_free(void* dev_ptr) {
  using namespace li4;
  const int rc = check_cuda(cudaFree(dev_ptr), "comm_free: cudaFree");
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_ipc_get_handle(void* dev_ptr, void* handle) {
  using namespace li4;
  static_assert(sizeof(cudaIpcMemHandle_t) == LI4_IPC_HANDLE_BYTES, "IPC handle size");
  if (!dev_ptr || !handle) return set_error(LI4_ERR_INVALID_ARG, "ipc_get_handle: null pointer");
  const int rc = check_cuda(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), dev_ptr),
                            "ipc_get_handle: cudaIpcGetMemHandle");
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_ipc_open_handle(const void* handle, void** dev_ptr) {
  using namespace li4;
  if (!dev_ptr || !handle) return set_error(LI4_ERR_INVALID_ARG, "ipc_open_handle: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const int rc = check_cuda(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess),
                            "ipc_open_handle: cudaIpcOpenMemHandle");
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_ipc_close(void* dev_ptr) {
  using namespace li4;
  const int rc = check_cuda(cudaIpcCloseMemHandle(dev_ptr), "ipc_close: cudaIpcCloseMemHandle");
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_allreduce_add(const void* const* slots, void* const* flags, void* counts, int ctas, int world,
                                 int rank, int64_t n, const void* residual, void* out, void* stream) {
  using namespace li4;
  if (world < 1 || world > kArMaxRanks || rank < 0 || rank >= world || ctas < 1 || ctas > 1024 || n < 0)
    return set_error(LI4_ERR_INVALID_ARG, "allreduce_add: world=%d rank=%d ctas=%d n=%lld", world, rank, ctas,
                     (long long)n);
  if (!slots || !flags || !counts || !residual || !out)
    return set_error(LI4_ERR_INVALID_ARG, "allreduce_add: null pointer");
  ArArgs a = {};
  for (int r = 0; r < world; ++r) {
    if (!slots[r] || !flags[r]) return set_error(LI4_ERR_INVALID_ARG, "allreduce_add: null peer pointer");
    if (!aligned16(slots[r])) return set_error(LI4_ERR_ALIGNMENT, "allreduce_add: slots must be 16-byte aligned");
    a.slots[r] = static_cast<const __half*>(slots[r]);
    a.flags[r] = static_cast<unsigned*>(flags[r]);
  }
  if (!aligned16(residual) || !aligned16(out))
    return set_error(LI4_ERR_ALIGNMENT, "allreduce_add: residual / out must be 16-byte aligned");
  a.counts = static_cast<unsigned*>(counts);
  a.residual = static_cast<const __half*>(residual);
  a.out = static_cast<__half*>(out);
  a.n = n;
  a.world = world;
  a.rank = rank;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas, 1, 1);
  cfg.blockDim = dim3(kArThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int rc = check_cuda(cudaLaunchKernelEx(&cfg, allreduce_add_kernel, a), "allreduce_add: kernel launch");
  if (rc == LI4_OK) clear_error();
  return rc;
}
