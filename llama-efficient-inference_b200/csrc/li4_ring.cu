// li4_ring.cu -- the shared-memory ring GEMV kernel (sm_100a) for long K over few row tiles.
//
// Why this shape.  The register-ring kernels keep 4-5 KB per warp in flight; here the weights
// move through a ring of shared-memory stages filled with 1-D bulk copies (cp.async.bulk, the
// TMA engine) by one producer warp and drained by 16 consumer warps that all work on every
// stage.  A CTA's whole weight slice can be requested at its first instruction, with no split-K:
// for down_proj (2048 x 8192) one 16-row x 8192-k stage per CTA replaces the streaming kernel's
// two K ranges and their last-arriver reduction (M = 1: 5.4 against 6.4 us per launch).
// Measured on B200, the bulk-copy path moves at most ~25 GB/s per SM even with three 64 KB
// copies in flight (lm_head: 0.57 of the HBM copy peak, against 0.63 for the register-ring tile
// kernel), and its cost grows with the number of copies (per-row 1 KB copies: 0.41), so the
// dispatcher takes this kernel only where the split-K epilogue is the larger cost.
//
// Work split.  A stage holds T 16-row tiles of the whole K range (T = 1, 2 or 4): T * 16 packed
// rows, then their scale rows and zero rows.  Contiguous tensors move as three block copies per
// stage (rows back to back, pitch K/2); strided ones row by row at a padded pitch (K/2 + 64
// bytes, so the 16-byte reads of a quarter warp's two rows fall on distinct banks).  The stages
// of a CTA are the stage units blockIdx.x, + gridDim.x, ...; the ring is `stages` deep, each
// stage with a "full" mbarrier (the producer's copies, counted in bytes) and an "empty" one (one
// arrival per consumer warp).  Consumer warp w takes tile w % T of every stage and its ksteps
// w / T, + 16 / T, ...; each warp's partial sums go to shared memory, and after one named
// barrier the tile's owner warp (w < T) sums the 16 / T partials in warp order (bitwise
// deterministic) and runs the epilogue (every li4_fusion epilogue but the all-reduce one, and
// the fused greedy argmax).
//
// Math per 16-row x 128-k unit as in the other GEMV kernels (stream_compute): exact q - zero in
// fp16 from the magic-number unpack, m16n8k16 with fp32 accumulation, the group scale in fp32.
// Every mbarrier wait is bounded (test_wait polls); a wait that runs out sets bit 0 of the
// device error word, and the producer drains its own copies (bounded) before it leaves.
#include "li4_common.cuh"
#include "li4_gemv_device.cuh"
#include "li4_internal.h"

#include <mutex>
#include <vector>

namespace li4 {

struct RingArgs {
  int T;            // 16-row tiles per stage (1, 2 or 4)
  int stages;       // ring depth (<= kRingMaxStages)
  int pitch;        // bytes between packed rows of a stage
  int stage_bytes;  // bytes per stage (multiple of 128)
  int n_su;         // stage units: ceil(n_tiles / T)
  int contig;       // 1: a stage unit's packed, scale and zero rows are one block copy each
                    // (rows back to back in HBM, pitch = K/2); 0: a copy per row (padded pitch)
};

// value(r, m) of one tile: the partials of the warps that share it, summed in warp order.
struct RingSum {
  const float* base;  // red buffer + (owner warp) * 16 * M
  int n, step, M;     // n partials, `step` warps apart
  __device__ __forceinline__ float operator()(int r, int m) const {
    float v = 0.f;
    for (int q = 0; q < n; ++q) v += base[((long long)q * step * 16 + r) * M + m];
    return v;
  }
};

// The greedy argmax keys of one tile's outputs (the fp16-rounded values the epilogue writes),
// reduced over the warp and folded into the running keys (argmax_finish ends the launch).
template <typename F>
__device__ __forceinline__ void ring_argmax(const GemvArgs& a, int tile, int lane, F value) {
  const int row0 = tile * 16, rows = min(16, a.N - row0);
  for (int m = 0; m < a.M; ++m) {
    unsigned long long k = 0ull;
    if (lane < rows) k = argmax_key(__half2float(__float2half_rn(value(lane, m))), row0 + lane);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
    if (lane == 0 && k != 0ull) atomicMax(&a.am_keys[m], k);
  }
}

__device__ __forceinline__ void ring_consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kRingWarps * 32) : "memory");
}

template <bool FUSED>
__global__ void __launch_bounds__(kRingThreads, 1) gemv_ring_kernel(const __grid_constant__ GemvArgs a,
                                                                    const __grid_constant__ RingArgs r) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nks = a.ks_per_split;  // the whole K (one K range)
  const int M = a.M;               // <= 8: one n-tile, x rows unpadded
  const int rows_st = 16 * r.T;
  uint8_t* ring = smem;
  uint8_t* xs = ring + (size_t)r.stages * r.stage_bytes;
  float* red = reinterpret_cast<float*>(xs + (((size_t)nks * M * 256 + 127) & ~(size_t)127));  // [2][warps][16][M]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * kRingWarps * 16 * M);
  uint64_t* empty = full + kRingMaxStages;
  __shared__ float s_rstd[LI4_MAX_M];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = (int)gridDim.x;
  const int my = (r.n_su - (int)blockIdx.x + G - 1) / G;  // this CTA's stage units

  if (threadIdx.x == 0) {
    for (int s = 0; s < r.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRingWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kRingWarps) {
    // ---------------- producer warp: weights never come from the preceding kernel ----------------
    const unsigned row_bytes = (unsigned)nks * 64;
    const unsigned sz_row = (unsigned)nks * 2;
    bool ok = true;
    int issued = 0;
    for (int j = 0; j < my && ok; ++j) {
      const int s = j % r.stages;
      if (j >= r.stages) ok = mbar_spin_bounded(&empty[s], ((j / r.stages) - 1) & 1);
      if (!ok) break;
      issued = j + 1;
      const int row0 = ((int)blockIdx.x + j * G) * rows_st;
      const int valid = min(rows_st, a.N - row0);
      uint8_t* st = ring + (size_t)s * r.stage_bytes;
      uint8_t* sc = st + (size_t)rows_st * r.pitch;
      uint8_t* ze = sc + (size_t)rows_st * sz_row;
      if (r.contig) {
        // three copies: the valid rows of packed, scale and zero (rows past N keep stale bytes;
        // their outputs are not written)
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], (unsigned)valid * (row_bytes + 2u * sz_row));
          bulk_g2s(st, a.packed + (long long)row0 * a.spn, (unsigned)valid * row_bytes, &full[s]);
          bulk_g2s(sc, a.scale + (long long)row0 * a.ssn, (unsigned)valid * sz_row, &full[s]);
          bulk_g2s(ze, a.zero + (long long)row0 * a.ssn, (unsigned)valid * sz_row, &full[s]);
        }
        __syncwarp();
        continue;
      }
      if (lane == 0) mbar_arrive_expect_tx(&full[s], (unsigned)rows_st * (row_bytes + 2u * sz_row));
      __syncwarp();
      for (int i = lane; i < rows_st; i += 32) {
        const int row = min(row0 + i, a.N - 1);  // rows past N repeat row N-1 (their outputs are not written)
        bulk_g2s(st + (size_t)i * r.pitch, a.packed + (long long)row * a.spn, row_bytes, &full[s]);
        bulk_g2s(sc + (size_t)i * sz_row, a.scale + (long long)row * a.ssn, sz_row, &full[s]);
        bulk_g2s(ze + (size_t)i * sz_row, a.zero + (long long)row * a.ssn, sz_row, &full[s]);
      }
    }
    // Drain: the last fill of every stage has landed before the producer leaves (a stage is
    // refilled only after the consumers released its previous fill, so only these can be in
    // flight; on the normal path they complete as the data arrives).
    for (int j = (issued > r.stages ? issued - r.stages : 0); j < issued; ++j)
      mbar_spin_bounded(&full[j % r.stages], (j / r.stages) & 1);
    pdl_wait_primary();  // every thread of the grid passes the dependency wait
    return;
  }

  // ---------------- consumer warps ----------------
  const int grp = lane >> 2, quad = lane & 3;
  pdl_wait_primary();  // x (and the residual) come from the preceding kernel
  if (FUSED && a.norm_w != nullptr) {  // RMSNorm factors over the consumer warps
    if (a.ssq_in != nullptr) rms_from_ssq<kRingWarps>(a, s_rstd, warp, lane);
    else rms_factors<kRingWarps>(a, s_rstd, warp, lane);
    ring_consumer_sync();
  }
  if (FUSED && a.norm_w != nullptr) stage_x<1, kRingWarps * 32, true>(a, 0, nks, M, xs, s_rstd);
  else stage_x<1, kRingWarps * 32, false>(a, 0, nks, M, xs);
  ring_consumer_sync();

  const bool bvalid = grp < M;
  int boff[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) boff[w] = (grp * 4 + quad) * 64 + ((w ^ xs_key(grp, quad)) << 4);
  const int nt_stride = M * 256;
  const int tt = warp % r.T;               // this warp's tile in every stage
  const int kstride = kRingWarps / r.T;    // warps sharing a tile
  const int upw = nks / kstride;           // units per warp per stage
  const int ra = tt * 16 + grp, rb = ra + 8;
  const int off_lo = ra * r.pitch + quad * 16, off_hi = rb * r.pitch + quad * 16;
  const int sz_lo = ra * nks, sz_hi = rb * nks;

  bool ok = true;
  for (int j = 0; j < my; ++j) {
    const int s = j % r.stages;
    if (ok) ok = mbar_spin_bounded(&full[s], (j / r.stages) & 1);
    float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    if (ok) {
      const uint8_t* st = ring + (size_t)s * r.stage_bytes;
      const unsigned short* sc = reinterpret_cast<const unsigned short*>(st + (size_t)rows_st * r.pitch);
      const unsigned short* ze = sc + rows_st * nks;
#pragma unroll 2
      for (int i = 0; i < upw; ++i) {
        const int ks = warp / r.T + kstride * i;
        StreamUnit u;
        u.lo = lds128(st + off_lo + ks * 64);
        u.hi = lds128(st + off_hi + ks * 64);
        u.sz_lo = (uint32_t)sc[sz_lo + ks] | ((uint32_t)ze[sz_lo + ks] << 16);
        u.sz_hi = (uint32_t)sc[sz_hi + ks] | ((uint32_t)ze[sz_hi + ks] << 16);
        stream_compute<1>(u, xs + ks * nt_stride, nt_stride, boff, bvalid, acc);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done reading the stage
    float* rbuf = red + (size_t)(j & 1) * kRingWarps * 16 * M;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = grp + 8 * (e >> 1), m = 2 * quad + (e & 1);
      if (m < M) rbuf[(warp * 16 + row) * M + m] = acc[0][e];
    }
    ring_consumer_sync();
    if (warp < r.T) {  // the owner warp of tile `warp` of this stage
      const int tile = ((int)blockIdx.x + j * G) * r.T + warp;
      if (tile * 16 < a.N) {
        const RingSum sum{rbuf + warp * 16 * M, kstride, r.T, M};
        emit_tile<FUSED>(a, tile, lane, 32, sum);
        if (FUSED && a.am_keys != nullptr) ring_argmax(a, tile, lane, sum);
      }
    }
  }
  if (FUSED && a.am_keys != nullptr) argmax_finish(a, [] { ring_consumer_sync(); });
}

size_t ring_smem_bytes(int M, int ks, int stages, int stage_bytes) {
  return (size_t)stages * stage_bytes + (((size_t)ks * M * 256 + 127) & ~(size_t)127) +
         (size_t)2 * kRingWarps * 16 * M * sizeof(float) + (size_t)2 * kRingMaxStages * sizeof(uint64_t);
}

int ring_stage_bytes(int ks, int T, int pitch) { return (16 * T * pitch + 2 * 16 * T * ks * 2 + 127) & ~127; }

template <typename KernelT>
static int ring_smem_limit(KernelT kernel, size_t smem) {
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
                                "int4_linear: ring kernel shared-memory limit");
      if (rc == LI4_OK) e.limit = smem;
      return rc;
    }
  const int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "int4_linear: ring kernel shared-memory limit");
  if (rc == LI4_OK) cache.push_back(Entry{(const void*)kernel, dev, smem});
  return rc;
}

int launch_ring(const GemvArgs& a, bool fused, int grid_x, int T, int stages, int pitch, size_t smem,
                cudaStream_t stream) {
  RingArgs r;
  r.T = T;
  r.stages = stages;
  // rows back to back in packed, scale and zero: one block copy each per stage unit, unpadded
  // rows (pitch = K/2; the stage then needs less than the padded size the plan reserved)
  r.contig = (a.spn == (long long)a.ks_per_split * 64 && a.ssn == a.ks_per_split) ? 1 : 0;
  r.pitch = r.contig ? a.ks_per_split * 64 : pitch;
  r.stage_bytes = ring_stage_bytes(a.ks_per_split, T, r.pitch);
  r.n_su = (a.n_tiles + T - 1) / T;
  auto kernel = fused ? gemv_ring_kernel<true> : gemv_ring_kernel<false>;
  int rc = ring_smem_limit(kernel, smem);
  if (rc != LI4_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid_x, 1, 1);
  cfg.blockDim = dim3(kRingThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, a, r), "int4_linear: ring kernel launch");
}

int ring_device_errors(unsigned* flags, bool reset) { return tu_device_errors(flags, reset); }

}  // namespace li4
