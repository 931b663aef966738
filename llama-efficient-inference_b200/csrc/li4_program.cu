// li4_program.cu -- the decode step as one persistent launch, sm_100a.
//
// A decode program is a list of ops (INT4 linears with their fused prologue /
// epilogue, decode attention, the embedding gather, the greedy argmax) that one
// launch of exactly one CTA per SM runs in order.  Per CTA:
//
//   * warp CW (the producer) walks the CTA's weight units of every linear op of
//     the program, in program order, and copies each (16 rows x up to 2048 k of
//     packed nibbles plus their scale and zero rows) into the next stage of a
//     shared-memory ring with cp.async.bulk.  It waits only for a free stage --
//     never for activations -- so while the consumers wait for an op's inputs,
//     the weights of the following ops are already streaming in;
//   * warps 0..CW-1 (the consumers) run the ops.  An op that waits for op j first
//     polls op j's completion counter (bounded), then stages its x in shared
//     memory (RMSNorm applied), and each consumer warp takes the CTA's units of
//     the op whose ring stage it owns (stage w for warp w): wait for the stage,
//     nibble unpack + mma.m16n8k16 as the per-launch kernels do, release the
//     stage, run the epilogue.  When all consumer warps are done with the op, the
//     CTA adds one to the op's completion counter (release); waiters acquire it.
//
// Units of an op go to CTAs round-robin, starting at an offset that rotates with
// the units of the ops before it, so every CTA gets a near-equal share of the
// step's weight bytes.  A linear with K > 2048 is split into K ranges of 2048:
// CTA c takes range c % C (C ranges) for all its units, so it stages one range of
// x; the ranges of a 16-row tile meet in fp32 partials and the last range to
// arrive (arrival counter) sums them in fixed order and runs the epilogue.
//
// Every wait is bounded (mbarrier waits and counter polls): a wait that runs out
// sets a bit of the device error word and marks the launch as failing, after
// which every other wait of the launch gives up at once, so a fault elsewhere
// ends the launch quickly instead of hanging it.  The last CTA to leave resets
// the completion counters for the next launch and applies the program's
// increments (the decode position).
//
// The arithmetic of every op is the per-launch kernels': li4_gemv's emitters for
// the linears, li4_attention's rounding points for the attention, torch.argmax's
// tie rule for the argmax.
#include "li4_common.cuh"
#include "li4_gemv_device.cuh"
#include "li4_internal.h"

#include <algorithm>
#include <cstring>
#include <vector>

namespace li4 {

enum ProgOpKind { kOpLinear = 0, kOpAttention = 1, kOpGather = 2, kOpArgmax = 3 };

constexpr int kProgSlotBytes = 18432;          // one unit: 16 rows x 2048 k (padded pitch) + scale / zero rows
constexpr int kProgKs = 16;                    // ksteps (of 128 k) per unit at most
constexpr unsigned kProgWaitLimit = 1u << 20;  // polls of a completion counter before giving up (~1 s)
constexpr int kProgMaxIncrements = 4;
constexpr int kArgmaxColChunk = 8192;          // columns per argmax unit

__host__ __device__ constexpr int prog_consumer_warps(int nt) { return nt == 1 ? 10 : 8; }  // = ring stages
__host__ __device__ constexpr int prog_threads(int nt) { return (prog_consumer_warps(nt) + 1) * 32; }
__host__ __device__ constexpr int prog_xs_bytes(int nt) { return kProgKs * nt * 8 * 256; }  // x staging
__host__ __device__ constexpr int prog_smem_bytes(int nt) {
  return prog_consumer_warps(nt) * kProgSlotBytes + prog_xs_bytes(nt) + 2 * prog_consumer_warps(nt) * 8;
}

struct AttnOp {
  const __half* q;
  long long sqb;
  const __half* ck;
  const __half* cv;
  long long csb, css;
  __half* out;
  long long sob;
  int n_kv, rep, hd;
  const long long* pos;
  int max_seq;
};

struct GatherOp {
  const __half* table;
  long long table_rows, stride_t;
  const long long* ids;
  int cols;
  __half* out;
  long long stride_o;
};

struct ArgmaxOp {
  const float* logits;
  long long stride;
  int cols, n_chunks;
  long long* out;
  long long out_stride;
  unsigned long long* keys;  // [rows], zero between launches
};

struct alignas(16) ProgOp {
  int kind;
  int wait;      // op whose completion this op waits for, -1: none
  int units;     // work units over all CTAs
  int chunks;    // linear: K ranges (units = n_tiles * chunks)
  int rot;       // first CTA of the round-robin
  int contig;    // linear: a unit's rows are one block of packed / scale / zero (3 copies)
  int finalize;  // argmax: the CTA that completes the op last writes the indices, then publishes
  GemvArgs g;
  AttnOp at;
  GatherOp ga;
  ArgmaxOp am;
};

struct ProgArgs {
  const ProgOp* ops;
  int n_ops;
  unsigned* done;       // [n_ops] completion counters, then the exit counter
  long long* incr[kProgMaxIncrements];
  int n_incr;
  long long* trace;     // optional [n_ops][ctas][4] globaltimer stamps (li4_program_set_trace)
};

__device__ unsigned g_prog_device_error;  // bits 0, 2, 3 of li4_device_errors (this translation unit)
// Set with the error bit by a wait that runs out; cleared by the last CTA to leave the launch.
__device__ unsigned g_prog_failing;

__device__ unsigned g_prog_wait_limit = kProgWaitLimit;  // li4_debug_set_wait_limits shortens it for tests
__device__ unsigned g_prog_wait_extra = 0u;  // > 0 (tests only): no counter wait can be met

int program_set_wait_limits(unsigned polls, unsigned extra) {
  const unsigned v = polls ? polls : kProgWaitLimit;
  int rc = check_cuda(cudaMemcpyToSymbol(g_prog_wait_limit, &v, sizeof(v)), "debug_set_wait_limits: program");
  if (rc == LI4_OK)
    rc = check_cuda(cudaMemcpyToSymbol(g_prog_wait_extra, &extra, sizeof(extra)), "debug_set_wait_limits: program");
  return rc;
}

int program_device_errors(unsigned* flags, bool reset) {
  unsigned a = 0;
  int rc = check_cuda(cudaMemcpyFromSymbol(&a, g_prog_device_error, sizeof(unsigned)), "device_errors: program");
  if (rc == LI4_OK && reset) {
    const unsigned zero = 0;
    rc = check_cuda(cudaMemcpyToSymbol(g_prog_device_error, &zero, sizeof(unsigned)), "device_errors: clearing");
  }
  if (rc == LI4_OK) *flags = a;
  return rc;
}

// ---------------------------------------------------------------------------
// Unit assignment (host and device compute the same).
// ---------------------------------------------------------------------------
// Number of units of `op` that CTA c of G runs.
__host__ __device__ inline int prog_count(const ProgOp& op, int c, int G) {
  if (op.kind == kOpLinear && op.chunks > 1) {
    const int C = op.chunks, per = G / C, T = op.units / C;
    if (c >= per * C || c / C >= T) return 0;
    return (T - c / C + per - 1) / per;
  }
  const int r = ((c - op.rot) % G + G) % G;
  return r < op.units ? (op.units - r + G - 1) / G : 0;
}

// Unit index of CTA c's i-th unit of `op` (linear with chunks: tile * chunks + range).
__host__ __device__ inline int prog_unit(const ProgOp& op, int c, int G, int i) {
  if (op.kind == kOpLinear && op.chunks > 1) {
    const int C = op.chunks, per = G / C;
    return (c / C + i * per) * C + c % C;
  }
  return ((c - op.rot) % G + G) % G + i * G;
}

__device__ __forceinline__ long long globaltimer() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void red_add_release_gpu(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Some bounded wait of this launch already ran out (the launch is failing): later waits give up
// at once instead of each running to its own limit.
__device__ __forceinline__ bool prog_failed() { return *reinterpret_cast<volatile unsigned*>(&g_prog_failing) != 0u; }

__device__ __forceinline__ void prog_fail(unsigned bit) {
  atomicOr(&g_prog_device_error, bit);
  atomicExch(&g_prog_failing, 1u);
}

// mbarrier phase wait, bounded like mbar_wait_bounded, and cut short once the launch is failing.
__device__ __forceinline__ bool prog_mbar_wait(uint64_t* bar, unsigned parity) {
  for (unsigned i = 0; i < kBulkWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && prog_failed()) return false;
  }
  prog_fail(1u);
  return false;
}

template <int CW>
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");
}

// ---------------------------------------------------------------------------
// Producer: the CTA's weight units of every linear op, in program order.
// ---------------------------------------------------------------------------
template <int CW>
__device__ __forceinline__ void program_producer(const ProgArgs& pa, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                                 int lane) {
  const int G = gridDim.x, c = blockIdx.x;
  bool ok = true;
  int seq = 0;
  for (int j = 0; j < pa.n_ops && ok; ++j) {
    const ProgOp& op = pa.ops[j];
    if (op.kind != kOpLinear) continue;
    const GemvArgs& a = op.g;
    const int n = prog_count(op, c, G);
    const int ks_n = a.ks_per_split;
    const BulkLayout L = bulk_layout(ks_n, op.contig != 0);
    const unsigned stage_bytes = 16u * (unsigned)(ks_n * 64) + 2u * 16u * (unsigned)(ks_n * 2);
    for (int i = 0; i < n && ok; ++i, ++seq) {
      const int s = seq % CW;
      if (seq >= CW) ok = prog_mbar_wait(&empty[s], ((seq / CW) - 1) & 1);
      if (!ok) break;
      const int u = prog_unit(op, c, G, i);
      const int tile = u / op.chunks, ks0 = (u % op.chunks) * ks_n;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], stage_bytes);
      __syncwarp();
      uint8_t* st = ring + (size_t)s * kProgSlotBytes;
      if (op.contig) {  // rows tile*16 .. +15: one block of packed, scale and zero each (the last tile clamped)
        if (lane == 0) {
          const long long r0 = min(tile * 16, a.N - 16);
          bulk_g2s(st, a.packed + r0 * a.spn, 16 * ks_n * 64, &full[s]);
          bulk_g2s(st + L.sz_off, a.scale + r0 * a.ssn, 16 * ks_n * 2, &full[s]);
          bulk_g2s(st + L.sz_off + 16 * ks_n * 2, a.zero + r0 * a.ssn, 16 * ks_n * 2, &full[s]);
        }
      } else if (lane < 16) {
        const long long r = min(tile * 16 + lane, a.N - 1);
        bulk_g2s(st + lane * L.pitch, a.packed + r * a.spn + (long long)ks0 * 64, ks_n * 64, &full[s]);
        bulk_g2s(st + L.sz_off + lane * ks_n * 2, a.scale + r * a.ssn + ks0, ks_n * 2, &full[s]);
      } else {
        const long long r = min(tile * 16 + (lane - 16), a.N - 1);
        bulk_g2s(st + L.sz_off + 16 * ks_n * 2 + (lane - 16) * ks_n * 2, a.zero + r * a.ssn + ks0, ks_n * 2,
                 &full[s]);
      }
    }
  }
  // Drain: the last fill of every stage has landed before the producer leaves.
  for (int it = (seq > CW ? seq - CW : 0); it < seq; ++it) prog_mbar_wait(&full[it % CW], (it / CW) & 1);
}

// x staging of the op's K range [ks0, ks0 + nks) in the layout of stage_x, with the RMSNorm
// prologue (NORM: the range is all of K) in the same pass over x.  A thread owns one 16-byte
// k-chunk of every row and loads all of them before it uses any, so one L2 round trip brings
// the whole staging in.  With NORM it also sums the squares of what it loaded; after the
// per-row sums meet in shared memory, it rescales the blocks it wrote --
// fp16(fp16(x * rstd) * w), the weight permuted into the same (k, k+4) pairs.
// x rows are 16-byte aligned (checked on the host).
template <int NT, int CW, bool NORM>
__device__ __forceinline__ void stage_x_prog(const GemvArgs& a, int ks0, int nks, uint8_t* xs, float* s_ssq,
                                             float* s_rstd, int lane) {
  constexpr int THREADS = CW * 32, M8 = 8, R = NT * 8;
  const int chunks = nks * 16;
  const int M = a.M;
  if (NORM && threadIdx.x < LI4_MAX_M) s_ssq[threadIdx.x] = 0.f;
  float ss[R];
#pragma unroll
  for (int m = 0; m < R; ++m) ss[m] = 0.f;
  for (int c = threadIdx.x; c < chunks; c += THREADS) {
    const int ks = c >> 4, quad = (c >> 2) & 3, w = c & 3;
    const __half* src = a.x + (long long)(ks0 + ks) * 128 + 32 * quad + 8 * w;
    uint4 v[R];
#pragma unroll
    for (int m = 0; m < R; ++m)
      v[m] = m < M ? __ldcg(reinterpret_cast<const uint4*>(src + (long long)m * a.sxm)) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int m = 0; m < R; ++m) {
      const uint32_t u[4] = {v[m].x, v[m].y, v[m].z, v[m].w};
      if (NORM) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[e]));
          ss[m] = fmaf(f.x, f.x, ss[m]);
          ss[m] = fmaf(f.y, f.y, ss[m]);
        }
      }
      uint4 out;
      out.x = __byte_perm(u[0], u[2], 0x5410);  // (x0, x4)
      out.y = __byte_perm(u[0], u[2], 0x7632);  // (x1, x5)
      out.z = __byte_perm(u[1], u[3], 0x5410);  // (x2, x6)
      out.w = __byte_perm(u[1], u[3], 0x7632);  // (x3, x7)
      const int nt = m >> 3, m8 = m & 7;
      *reinterpret_cast<uint4*>(xs + xs_chunk_offset(((ks * NT + nt) * M8 + m8) * 4 + quad, w, m8)) = out;
    }
  }
  if (!NORM) return;
  consumers_sync<CW>();  // s_ssq zeroed before any warp adds to it
#pragma unroll
  for (int m = 0; m < R; ++m) {
    if (m >= M) break;
    float t = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) atomicAdd(&s_ssq[m], t);
  }
  consumers_sync<CW>();
  if (threadIdx.x < M) s_rstd[threadIdx.x] = rsqrtf(s_ssq[threadIdx.x] / (float)a.K + a.norm_eps);
  consumers_sync<CW>();
  for (int c = threadIdx.x; c < chunks; c += THREADS) {
    const int ks = c >> 4, quad = (c >> 2) & 3, w = c & 3;
    const uint4 wn = __ldg(reinterpret_cast<const uint4*>(a.norm_w + (long long)(ks0 + ks) * 128 + 32 * quad + 8 * w));
    const uint32_t w0 = __byte_perm(wn.x, wn.z, 0x5410), w1 = __byte_perm(wn.x, wn.z, 0x7632);
    const uint32_t w2 = __byte_perm(wn.y, wn.w, 0x5410), w3 = __byte_perm(wn.y, wn.w, 0x7632);
#pragma unroll
    for (int m = 0; m < R; ++m) {
      if (m >= M) break;
      const int nt = m >> 3, m8 = m & 7;
      uint4* blk = reinterpret_cast<uint4*>(xs + xs_chunk_offset(((ks * NT + nt) * M8 + m8) * 4 + quad, w, m8));
      uint4 v = *blk;
      const float r = s_rstd[m];
      v.x = norm_pair(v.x, w0, r);
      v.y = norm_pair(v.y, w1, r);
      v.z = norm_pair(v.z, w2, r);
      v.w = norm_pair(v.w, w3, r);
      *blk = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Consumers: one linear op.  seq0 = the CTA's ring sequence number of the op's
// first unit (the producer filled the units in the same order).
// ---------------------------------------------------------------------------
template <int NT, int CW>
__device__ __forceinline__ void program_linear(const ProgOp& op, int n, int seq0, uint8_t* ring, uint8_t* xs,
                                               uint64_t* full, uint64_t* empty, float* s_rstd, float* s_ssq,
                                               int warp, int lane, long long* tr) {
  const GemvArgs& a = op.g;
  const int G = gridDim.x, c = blockIdx.x;
  const int ks_n = a.ks_per_split;
  const int ks0 = (op.chunks > 1 ? c % op.chunks : 0) * ks_n;
  constexpr int M8 = 8;
  if (a.norm_w != nullptr && a.ssq_in == nullptr && op.chunks == 1) {
    stage_x_prog<NT, CW, true>(a, 0, ks_n, xs, s_ssq, s_rstd, lane);
  } else if (a.norm_w != nullptr) {  // the mean of squares over all of K, or handed over by the producer op
    if (a.ssq_in != nullptr) rms_from_ssq<CW>(a, s_rstd, warp, lane);
    else rms_factors<CW>(a, s_rstd, warp, lane);
    consumers_sync<CW>();
    stage_x<NT, CW * 32, true>(a, ks0, ks_n, M8, xs, s_rstd);
  } else {
    stage_x_prog<NT, CW, false>(a, ks0, ks_n, xs, s_ssq, s_rstd, lane);
  }
  consumers_sync<CW>();
  if (tr && threadIdx.x == 0) tr[2] = globaltimer();

  const int grp = lane >> 2, quad = lane & 3;
  const bool bvalid = grp < ((NT == 1) ? a.M : 8);
  int boff[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) boff[w] = (grp * 4 + quad) * 64 + ((w ^ xs_key(grp, quad)) << 4);
  constexpr int nt_stride = M8 * 256;
  constexpr int ks_stride = NT * nt_stride;
  const BulkLayout L = bulk_layout(ks_n, op.contig != 0);

  bool ok = true;
  for (int i = (warp - seq0 % CW + CW) % CW; i < n; i += CW) {  // the units whose stage this warp owns
    const int seq = seq0 + i, s = warp;
    const int u = prog_unit(op, c, G, i);
    const int tile = u / op.chunks, chunk = u % op.chunks;
    if (ok) ok = prog_mbar_wait(&full[s], (seq / CW) & 1);
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
    if (ok) {
      const uint8_t* st = ring + (size_t)s * kProgSlotBytes;
      const unsigned short* sc = reinterpret_cast<const unsigned short*>(st + L.sz_off);
      const unsigned short* ze = sc + 16 * ks_n;
      // stage row of tile row j: a clamped contiguous last tile starts `shift` rows early
      const int shift = op.contig ? tile * 16 - min(tile * 16, a.N - 16) : 0;
      const int ra = min(grp + shift, 15), rb = min(grp + 8 + shift, 15);
      const uint8_t* row_lo = st + ra * L.pitch + quad * 16;
      const uint8_t* row_hi = st + rb * L.pitch + quad * 16;
#pragma unroll 4
      for (int ks = 0; ks < ks_n; ++ks) {
        StreamUnit su;
        su.lo = *reinterpret_cast<const uint4*>(row_lo + ks * 64);
        su.hi = *reinterpret_cast<const uint4*>(row_hi + ks * 64);
        su.sz_lo = (uint32_t)sc[ra * ks_n + ks] | ((uint32_t)ze[ra * ks_n + ks] << 16);
        su.sz_hi = (uint32_t)sc[rb * ks_n + ks] | ((uint32_t)ze[rb * ks_n + ks] << 16);
        stream_compute<NT>(su, xs + ks * ks_stride, nt_stride, boff, bvalid, acc);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // the stage is free for the producer
    if (op.chunks == 1) {
      emit_warp_tile<true, NT>(a, tile, acc, grp, quad);
      continue;
    }
    const int row0 = tile * 16;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = grp + 8 * (e >> 1), m = nt * 8 + 2 * quad + (e & 1);
        if (m < a.M && row0 + r < a.N) a.partial[((long long)chunk * a.M + m) * a.N + row0 + r] = acc[nt][e];
      }
    // the last K range to arrive sums the partials (fixed order) and resets the counter
    __threadfence();
    __syncwarp();
    unsigned last = 0;
    if (lane == 0) last = (atomicAdd(&a.counters[tile], 1u) == (unsigned)(op.chunks - 1)) ? 1u : 0u;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence();
      if constexpr (NT == 2) emit_partial_tile<true>(a, tile, lane, PartialSum{a.partial + row0, a.M, a.N, op.chunks});
      else emit_tile<true>(a, tile, lane, 32, PartialSum{a.partial + row0, a.M, a.N, op.chunks});
      __syncwarp();
      if (lane == 0) a.counters[tile] = 0u;
    }
  }
}

// ---------------------------------------------------------------------------
// Consumers: attention for (sequence b, KV head g), the whole CTA.  The
// arithmetic of li4_attention.cu at one CTA per (KV head, sequence):
//   s = fp16(fp16(q . k) / sqrt(d)), p = fp16(exp(s - max) / sum), o = fp16(sum_j p_j v_j).
// Shared memory (the x staging area): q as fp32, the warps' partial P.V, the
// fp16 scores / probabilities of the REP heads over the L keys.  The cache rows
// are read straight from L2 / HBM with many loads in flight per thread.
// ---------------------------------------------------------------------------
template <int REP, int HD, int CW>
__device__ __noinline__ void program_attention(const AttnOp& at, int b, int g, uint8_t* xs, float (*s_red)[8],
                                                float (*s_stat)[8], int warp, int lane) {
  constexpr int T = CW * 32, DPL = HD / 32, CPR = HD / 8;
  const int tid = threadIdx.x;
  float* q_s = reinterpret_cast<float*>(xs);                    // [REP][HD]
  float* red = q_s + REP * HD;                                   // [CW][REP][HD]
  __half* sc = reinterpret_cast<__half*>(red + CW * REP * HD);  // [REP][max_seq]
  const int ls = at.max_seq;
  long long p = *at.pos;
  p = p < 0 ? 0 : (p >= at.max_seq ? at.max_seq - 1 : p);
  const int L = (int)p + 1;
  const __half* kbase = at.ck + (long long)b * at.csb + (long long)g * HD;
  const __half* vbase = at.cv + (long long)b * at.csb + (long long)g * HD;
  const __half* qrow = at.q + (long long)b * at.sqb + (long long)g * REP * HD;
  for (int t = tid; t < REP * HD; t += T) q_s[t] = __half2float(__ldcg(qrow + t));
  consumers_sync<CW>();

  const float inv_scale = 1.0f / sqrtf((float)HD);
  float mx[REP];
#pragma unroll
  for (int r = 0; r < REP; ++r) mx[r] = -INFINITY;
  // scores: JB keys per thread per round, all their 16-byte loads issued before any is used
  constexpr int JB = CPR <= 8 ? 2 : 1;
  for (int jb = tid; jb < L; jb += JB * T) {
    uint4 kv[JB][CPR];
#pragma unroll
    for (int bq = 0; bq < JB; ++bq) {
      const int j = jb + bq * T;
      const uint4* kr = reinterpret_cast<const uint4*>(kbase + (long long)(j < L ? j : 0) * at.css);
#pragma unroll
      for (int cc = 0; cc < CPR; ++cc) kv[bq][cc] = __ldcg(kr + cc);
    }
#pragma unroll
    for (int bq = 0; bq < JB; ++bq) {
      const int j = jb + bq * T;
      if (j >= L) break;
      float dot[REP];
#pragma unroll
      for (int r = 0; r < REP; ++r) dot[r] = 0.f;
#pragma unroll
      for (int cc = 0; cc < CPR; ++cc) {
        const uint32_t w[4] = {kv[bq][cc].x, kv[bq][cc].y, kv[bq][cc].z, kv[bq][cc].w};
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
        const __half sv = __float2half_rn(s16 * inv_scale);  // torch divides by a scalar as a product with its reciprocal
        sc[r * ls + j] = sv;
        mx[r] = fmaxf(mx[r], __half2float(sv));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float v = mx[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) s_red[warp][r] = v;
  }
  consumers_sync<CW>();
  if (tid < REP) {
    float v = s_red[0][tid];
#pragma unroll
    for (int w = 1; w < CW; ++w) v = fmaxf(v, s_red[w][tid]);
    s_stat[0][tid] = v;
  }
  consumers_sync<CW>();
  float sum[REP];
#pragma unroll
  for (int r = 0; r < REP; ++r) sum[r] = 0.f;
  for (int j = tid; j < L; j += T) {
#pragma unroll
    for (int r = 0; r < REP; ++r) sum[r] += expf(__half2float(sc[r * ls + j]) - s_stat[0][r]);
  }
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float v = sum[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) s_red[warp][r] = v;
  }
  consumers_sync<CW>();
  if (tid < REP) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < CW; ++w) v += s_red[w][tid];
    s_stat[1][tid] = v;
  }
  consumers_sync<CW>();
  for (int j = tid; j < L; j += T) {
#pragma unroll
    for (int r = 0; r < REP; ++r)
      sc[r * ls + j] = __float2half_rn(expf(__half2float(sc[r * ls + j]) - s_stat[0][r]) / s_stat[1][r]);
  }
  consumers_sync<CW>();

  // P.V: warp w takes keys w, w + CW, ...; lane holds dims DPL*lane .. +DPL; U value rows in flight
  float acc[REP][DPL];
#pragma unroll
  for (int r = 0; r < REP; ++r)
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[r][e] = 0.f;
  auto load_v = [&](int j, float (&v)[DPL]) {
    const __half* src = vbase + (long long)j * at.css + DPL * lane;
    if constexpr (DPL == 1) {
      v[0] = __half2float(__ldcg(src));
    } else if constexpr (DPL == 2) {
      const float2 f = __half22float2(__ldcg(reinterpret_cast<const __half2*>(src)));
      v[0] = f.x;
      v[1] = f.y;
    } else {
      const uint2 u = __ldcg(reinterpret_cast<const uint2*>(src));
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      v[0] = f0.x;
      v[1] = f0.y;
      v[2] = f1.x;
      v[3] = f1.y;
    }
  };
  constexpr int U = DPL == 4 ? 8 : 16;
  int j = warp;
  for (; j + (U - 1) * CW < L; j += U * CW) {
    float vu[U][DPL];
#pragma unroll
    for (int u = 0; u < U; ++u) load_v(j + u * CW, vu[u]);
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        const float pj = __half2float(sc[r * ls + j + u * CW]);
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[r][e] = fmaf(pj, vu[u][e], acc[r][e]);
      }
  }
  for (; j < L; j += CW) {
    float vv[DPL];
    load_v(j, vv);
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float pj = __half2float(sc[r * ls + j]);
#pragma unroll
      for (int e = 0; e < DPL; ++e) acc[r][e] = fmaf(pj, vv[e], acc[r][e]);
    }
  }
#pragma unroll
  for (int r = 0; r < REP; ++r)
#pragma unroll
    for (int e = 0; e < DPL; ++e) red[(warp * REP + r) * HD + DPL * lane + e] = acc[r][e];
  consumers_sync<CW>();
  __half* orow = at.out + (long long)b * at.sob + (long long)g * REP * HD;
  for (int t = tid; t < REP * HD; t += T) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < CW; ++w) v += red[w * REP * HD + t];
    orow[t] = __float2half_rn(v);
  }
  consumers_sync<CW>();  // the staging area is reused by the next unit
}

template <int REP, int CW>
__device__ __forceinline__ void attention_hd(const AttnOp& at, int b, int g, uint8_t* xs, float (*s_red)[8],
                                             float (*s_stat)[8], int warp, int lane) {
  if (at.hd == 32) program_attention<REP, 32, CW>(at, b, g, xs, s_red, s_stat, warp, lane);
  else if (at.hd == 64) program_attention<REP, 64, CW>(at, b, g, xs, s_red, s_stat, warp, lane);
  else program_attention<REP, 128, CW>(at, b, g, xs, s_red, s_stat, warp, lane);
}

template <int CW>
__device__ __forceinline__ void attention_unit(const AttnOp& at, int u, uint8_t* xs, float (*s_red)[8],
                                               float (*s_stat)[8], int warp, int lane) {
  const int b = u / at.n_kv, g = u % at.n_kv;
  switch (at.rep) {  // (rep, head_dim) pairs with rep * head_dim <= 512 (checked on the host)
    case 1: attention_hd<1, CW>(at, b, g, xs, s_red, s_stat, warp, lane); break;
    case 2: attention_hd<2, CW>(at, b, g, xs, s_red, s_stat, warp, lane); break;
    case 4: attention_hd<4, CW>(at, b, g, xs, s_red, s_stat, warp, lane); break;
    default:
      if (at.hd == 32) program_attention<8, 32, CW>(at, b, g, xs, s_red, s_stat, warp, lane);
      else program_attention<8, 64, CW>(at, b, g, xs, s_red, s_stat, warp, lane);
      break;
  }
}

// out[r, :] = table[ids[r], :] (16-byte vectors: cols % 8 == 0 and aligned rows, checked on the host).
template <int CW>
__device__ __forceinline__ void gather_unit(const GatherOp& ga, int r) {
  long long id = ga.ids[r];
  if (id < 0 || id >= ga.table_rows) {
    if (threadIdx.x == 0) atomicOr(&g_prog_device_error, 8u);
    id = id < 0 ? 0 : ga.table_rows - 1;
  }
  const uint4* src = reinterpret_cast<const uint4*>(ga.table + id * ga.stride_t);
  uint4* dst = reinterpret_cast<uint4*>(ga.out + (long long)r * ga.stride_o);
  for (int t = threadIdx.x; t < ga.cols / 8; t += CW * 32) dst[t] = src[t];
}

template <int CW>
__device__ __forceinline__ void argmax_unit(const ArgmaxOp& am, int u, unsigned long long* s_key, int warp,
                                            int lane) {
  const int row = u / am.n_chunks, ch = u % am.n_chunks;
  const int c0 = ch * kArgmaxColChunk, c1 = min(am.cols, c0 + kArgmaxColChunk);
  const float* x = am.logits + (long long)row * am.stride;
  unsigned long long best = 0ull;
  // the logits come from this launch: L2 loads (16-byte vectors when the row is aligned)
  const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
  int i0 = c0;
  if (vec) {
    const int v1 = c1 / 4;
#pragma unroll 4
    for (int v = c0 / 4 + threadIdx.x; v < v1; v += CW * 32) {
      const float4 f = __ldcg(reinterpret_cast<const float4*>(x) + v);
      best = max(best, argmax_key(f.x, 4 * v));
      best = max(best, argmax_key(f.y, 4 * v + 1));
      best = max(best, argmax_key(f.z, 4 * v + 2));
      best = max(best, argmax_key(f.w, 4 * v + 3));
    }
    i0 = max(c0, 4 * v1);
  }
  for (int i = i0 + threadIdx.x; i < c1; i += CW * 32) best = max(best, argmax_key(__ldcg(x + i), i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  if (lane == 0) s_key[warp] = best;
  consumers_sync<CW>();
  if (threadIdx.x == 0) {
    unsigned long long k = s_key[0];
#pragma unroll
    for (int w = 1; w < CW; ++w) k = max(k, s_key[w]);
    atomicMax(&am.keys[row], k);
  }
  consumers_sync<CW>();
}

// Op finalisation by the CTA that completed it last (one thread).
__device__ __forceinline__ void finalize_op(const ProgOp& op) {
  if (op.kind == kOpArgmax) {
    const int rows = op.units / op.am.n_chunks;
    for (int r = 0; r < rows; ++r) {
      const unsigned long long k = atomicExch(&op.am.keys[r], 0ull);  // read and reset for the next launch
      op.am.out[(long long)r * op.am.out_stride] = (long long)(0xFFFFFFFFu - (unsigned)(k & 0xFFFFFFFFull));
    }
  }
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(prog_threads(NT), 1) decode_program_kernel(const __grid_constant__ ProgArgs pa) {
  constexpr int CW = prog_consumer_warps(NT);
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* xs = ring + (size_t)CW * kProgSlotBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(xs + prog_xs_bytes(NT));
  uint64_t* empty = full + CW;
  __shared__ ProgOp s_op;  // the consumers' copy of the current op
  __shared__ float s_rstd[LI4_MAX_M];
  __shared__ float s_ssq[LI4_MAX_M];
  __shared__ float s_red[CW][8];
  __shared__ float s_stat[2][8];
  __shared__ unsigned long long s_key[CW];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, c = blockIdx.x;
  if (threadIdx.x == 0) {
    for (int s = 0; s < CW; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);  // the consumer warp that owns the stage
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == CW) {
    program_producer<CW>(pa, ring, full, empty, lane);
  } else {
    int seq = 0;  // ring sequence number of the CTA's next linear unit
    for (int j = 0; j < pa.n_ops; ++j) {
      const ProgOp& gop = pa.ops[j];
      const int n = prog_count(gop, c, G);
      long long* tr = pa.trace ? pa.trace + ((long long)j * G + c) * 4 : nullptr;
      if (n > 0) {
        if (tr && threadIdx.x == 0) tr[0] = globaltimer();
        // threads 32.. copy the op into shared memory while thread 0 waits for its input op
        constexpr int kWords = (int)(sizeof(ProgOp) / 16);
        for (int t = (int)threadIdx.x - 32; t >= 0 && t < kWords; t += CW * 32 - 32)
          reinterpret_cast<uint4*>(&s_op)[t] = reinterpret_cast<const uint4*>(&gop)[t];
        if (threadIdx.x == 0 && gop.wait >= 0) {
          // every CTA has finished op `wait`: its writes are visible after this acquire and the barrier below
          const unsigned target = (unsigned)G + (unsigned)pa.ops[gop.wait].finalize + g_prog_wait_extra;
          const unsigned limit = g_prog_wait_limit;
          unsigned it = 0;
          while (ld_acquire_gpu(&pa.done[gop.wait]) < target) {
            if (++it == limit) {
              prog_fail(4u);
              break;
            }
            if ((it & 255u) == 0u && prog_failed()) break;
          }
        }
        consumers_sync<CW>();
        if (tr && threadIdx.x == 0) tr[1] = globaltimer();
        const ProgOp& op = s_op;
        switch (op.kind) {
          case kOpLinear:
            program_linear<NT, CW>(op, n, seq, ring, xs, full, empty, s_rstd, s_ssq, warp, lane, tr);
            seq += n;
            break;
          case kOpAttention:
            for (int i = 0; i < n; ++i)
              attention_unit<CW>(op.at, prog_unit(op, c, G, i), xs, s_red, s_stat, warp, lane);
            break;
          case kOpGather:
            for (int i = 0; i < n; ++i) gather_unit<CW>(op.ga, prog_unit(op, c, G, i));
            break;
          default:
            for (int i = 0; i < n; ++i) argmax_unit<CW>(op.am, prog_unit(op, c, G, i), s_key, warp, lane);
            break;
        }
        consumers_sync<CW>();  // the op's outputs are written and the staging area is free
        if (tr && threadIdx.x == 0) tr[3] = globaltimer();
      }
      if (threadIdx.x == 0) {  // (the op from global memory: s_op may already hold the next op)
        if (gop.finalize) {
          if (atom_add_acq_rel_gpu(&pa.done[j], 1u) == (unsigned)G - 1u) {
            finalize_op(gop);
            red_add_release_gpu(&pa.done[j], 1u);
          }
        } else {
          red_add_release_gpu(&pa.done[j], 1u);
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // the last CTA to leave resets the counters and applies the increments
    if (atom_add_acq_rel_gpu(&pa.done[pa.n_ops], 1u) == (unsigned)G - 1u) {
      for (int j = 0; j < pa.n_ops; ++j) pa.done[j] = 0u;
      for (int k = 0; k < pa.n_incr; ++k) *pa.incr[k] += 1;
      g_prog_failing = 0u;
      __threadfence();
      pa.done[pa.n_ops] = 0u;
    }
  }
}

int program_gemv_device_errors(unsigned* flags, bool reset) { return tu_device_errors(flags, reset); }

}  // namespace li4

namespace li4 {

// ---------------------------------------------------------------------------
// Standalone row gather (the embedding lookup of the per-launch decode step): one CTA per row,
// 16-byte vectors; the ids come from the preceding kernel (read after the dependency wait).
// ---------------------------------------------------------------------------
constexpr int kGatherThreads = 256;

__global__ void __launch_bounds__(kGatherThreads) gather_rows_kernel(const __half* table, long long table_rows,
                                                                     long long stride_t, const long long* ids,
                                                                     __half* out, long long stride_o, int cols) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int r = blockIdx.x;
  long long id = ids[r];
  if (id < 0 || id >= table_rows) {
    if (threadIdx.x == 0) atomicOr(&g_prog_device_error, 8u);
    id = id < 0 ? 0 : table_rows - 1;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + id * stride_t);
  uint4* dst = reinterpret_cast<uint4*>(out + (long long)r * stride_o);
  for (int t = threadIdx.x; t < cols / 8; t += kGatherThreads) dst[t] = src[t];
}

}  // namespace li4

extern "C" int li4_gather_rows(const void* table, int64_t table_rows, int64_t cols, int64_t stride_t,
                               const int64_t* ids, int64_t rows, void* out, int64_t stride_o, void* stream) {
  using namespace li4;
  if (!table || !ids || !out || table_rows < 1 || rows < 0 || rows > 65535 || cols < 8 || cols % 8 != 0 ||
      cols > INT32_MAX / 2 || stride_t < cols || stride_o < cols)
    return set_error(LI4_ERR_INVALID_ARG, "gather_rows: rows=%lld cols=%lld (cols %% 8 == 0) strides %lld, %lld",
                     (long long)rows, (long long)cols, (long long)stride_t, (long long)stride_o);
  if (!aligned16(table) || !aligned16(out) || stride_t % 8 != 0 || stride_o % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(ids) & 7u))
    return set_error(LI4_ERR_ALIGNMENT, "gather_rows: rows must be 16-byte aligned");
  if (rows == 0) return LI4_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)rows, 1, 1);
  cfg.blockDim = dim3(kGatherThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int rc = check_cuda(cudaLaunchKernelEx(&cfg, gather_rows_kernel, static_cast<const __half*>(table),
                                               (long long)table_rows, (long long)stride_t,
                                               reinterpret_cast<const long long*>(ids), static_cast<__half*>(out),
                                               (long long)stride_o, (int)cols),
                            "gather_rows: kernel launch");
  if (rc == LI4_OK) clear_error();
  return rc;
}

// ---------------------------------------------------------------------------
// Host side of the program.
// ---------------------------------------------------------------------------
struct li4_program {
  std::vector<li4::ProgOp> ops;
  std::vector<size_t> scratch_bytes;  // per op: split-K counters + partials, or argmax keys
  std::vector<long long*> incr;
  int device = -1;
  int ctas = 0, nt = 1;
  void* dev = nullptr;  // op table | completion counters | per-op scratch
  li4::ProgArgs args = {};
  bool finalized = false;
};

namespace li4 {

static int add_op(li4_program* prog, const ProgOp& op, size_t scratch, int* index) {
  if (prog->finalized) return set_error(LI4_ERR_INVALID_ARG, "program: finalized programs take no more ops");
  if (op.wait < -1 || op.wait >= (int)prog->ops.size())
    return set_error(LI4_ERR_INVALID_ARG, "program: op %zu waits for op %d (an earlier op or LI4_NO_WAIT)",
                     prog->ops.size(), op.wait);
  if (op.units < 1) return set_error(LI4_ERR_INVALID_ARG, "program: an op without work");
  prog->ops.push_back(op);
  prog->scratch_bytes.push_back(scratch);
  if (index) *index = (int)prog->ops.size() - 1;
  clear_error();
  return LI4_OK;
}

template <int NT>
static int program_occupancy(size_t smem, int* blocks) {
  auto kernel = decode_program_kernel<NT>;
  int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                      "program: shared memory limit");
  if (rc != LI4_OK) return rc;
  return check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kernel, prog_threads(NT), smem),
                    "program: occupancy");
}

}  // namespace li4

extern "C" int li4_program_create(li4_program** prog) {
  using namespace li4;
  if (!prog) return set_error(LI4_ERR_INVALID_ARG, "program_create: null output");
  *prog = new li4_program();
  clear_error();
  return LI4_OK;
}

extern "C" int li4_program_destroy(li4_program* prog) {
  using namespace li4;
  if (!prog) return LI4_OK;
  int rc = LI4_OK;
  if (prog->dev) {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(prog->device);
    rc = check_cuda(cudaFree(prog->dev), "program_destroy: cudaFree");
    cudaSetDevice(cur);
  }
  delete prog;
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_program_add_linear(li4_program* prog, const void* x, const void* packed, const void* scale,
                                      const void* zero, void* y, int64_t M, int64_t N, int64_t K, int64_t group_size,
                                      int64_t stride_xm, int64_t stride_pn, int64_t stride_sn, int64_t stride_ym,
                                      const li4_fusion* fusion, int wait, int* op_index) {
  using namespace li4;
  if (!prog) return set_error(LI4_ERR_INVALID_ARG, "program_add_linear: null program");
  if (M < 1 || M > LI4_MAX_M || N < 16 || N > INT32_MAX / 2 || K < 128 || K % 128 != 0 ||
      (K > 2048 && K % 2048 != 0) || K > (1 << 20))
    return set_error(LI4_ERR_UNSUPPORTED, "program_add_linear: M=%lld N=%lld K=%lld (program linears take "
                     "1 <= M <= 16, N >= 16, K %% 128 == 0 with K <= 2048 or K %% 2048 == 0)",
                     (long long)M, (long long)N, (long long)K);
  if (group_size != 128)
    return set_error(LI4_ERR_UNSUPPORTED, "program_add_linear: group size %lld (program linears take 128)",
                     (long long)group_size);
  if (fusion && fusion->argmax_out)
    return set_error(LI4_ERR_UNSUPPORTED, "program_add_linear: the fused argmax is a per-launch epilogue; "
                     "programs take li4_program_add_argmax");
  ProgOp op = {};
  op.kind = kOpLinear;
  op.wait = wait;
  int rc = prepare_linear(x, packed, scale, zero, y, M, N, K, group_size, stride_xm, stride_pn, stride_sn, stride_ym,
                          fusion, &op.g);
  if (rc != LI4_OK) return rc;
  if (!aligned16(x) || stride_xm % 8 != 0)
    return set_error(LI4_ERR_ALIGNMENT, "program_add_linear: x rows must be 16-byte aligned");
  const int ks_total = (int)(K / 128);
  const int ks_n = std::min(ks_total, kProgKs);
  op.chunks = ks_total / ks_n;
  op.g.n_tiles = (int)((N + 15) / 16);
  op.g.split = op.chunks;
  op.g.ks_per_split = ks_n;
  op.units = op.g.n_tiles * op.chunks;
  // A unit is one bulk copy each of packed, scale and zero when its 16 rows are contiguous (a
  // ragged last tile is copied from row N - 16, whose scale / zero rows must start on 16 bytes);
  // otherwise one copy per row, whose scale / zero pieces (ks_n fp16) must be whole 16-byte blocks.
  op.contig = (op.chunks == 1 && stride_pn == K / 2 && stride_sn == ks_n && (N % 16 == 0 || (N * ks_n) % 8 == 0))
                  ? 1 : 0;
  if (!aligned16(scale) || !aligned16(zero) || (!op.contig && (stride_sn % 8 != 0 || ks_n % 8 != 0)))
    return set_error(LI4_ERR_ALIGNMENT, "program_add_linear: scale / zero rows must be 16-byte aligned "
                     "(contiguous rows, or row stride %% 8 == 0 and K >= 1024)");
  const size_t scratch = op.chunks > 1 ? (size_t)op.g.n_tiles * 4 + (size_t)op.chunks * M * N * 4 : 0;
  return add_op(prog, op, scratch, op_index);
}

extern "C" int li4_program_add_attention(li4_program* prog, const void* q, int64_t stride_qb, const void* cache_k,
                                         const void* cache_v, int64_t cache_stride_b, int64_t cache_stride_s,
                                         void* out, int64_t stride_ob, int64_t batch, int64_t n_heads,
                                         int64_t n_kv_heads, int64_t head_dim, const int64_t* pos, int64_t max_seq,
                                         int wait, int* op_index) {
  using namespace li4;
  if (!prog) return set_error(LI4_ERR_INVALID_ARG, "program_add_attention: null program");
  if (!q || !cache_k || !cache_v || !out || !pos)
    return set_error(LI4_ERR_INVALID_ARG, "program_add_attention: null pointer");
  if (batch < 1 || n_kv_heads < 1 || n_heads < n_kv_heads || n_heads % n_kv_heads != 0 || max_seq < 1 ||
      batch * n_kv_heads > INT32_MAX / 2 || max_seq > INT32_MAX / 16)
    return set_error(LI4_ERR_INVALID_ARG, "program_add_attention: batch=%lld n_heads=%lld n_kv_heads=%lld "
                     "max_seq=%lld", (long long)batch, (long long)n_heads, (long long)n_kv_heads, (long long)max_seq);
  const int64_t rep = n_heads / n_kv_heads;
  if ((rep != 1 && rep != 2 && rep != 4 && rep != 8) || (head_dim != 32 && head_dim != 64 && head_dim != 128) ||
      rep * head_dim > 512)
    return set_error(LI4_ERR_UNSUPPORTED, "program_add_attention: n_heads / n_kv_heads = %lld with head_dim %lld "
                     "(1, 2, 4 or 8 with head_dim 32, 64 or 128, product <= 512)", (long long)rep,
                     (long long)head_dim);
  if (stride_qb < n_heads * head_dim || stride_ob < n_heads * head_dim || cache_stride_s < n_kv_heads * head_dim ||
      cache_stride_b < max_seq * cache_stride_s)
    return set_error(LI4_ERR_INVALID_ARG, "program_add_attention: strides smaller than the rows");
  if (!aligned16(cache_k) || !aligned16(cache_v) || cache_stride_s % 8 != 0 || cache_stride_b % 8 != 0 ||
      ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 1u))
    return set_error(LI4_ERR_ALIGNMENT, "program_add_attention: cache rows must be 16-byte aligned");
  // shared memory: q (fp32), the warps' partial P.V (fp32), the scores (fp16) of every key; the
  // launch shape (and so the staging area) is known at finalize, this rejects what fits neither
  const int64_t need_nt1 = rep * head_dim * 4 * (1 + prog_consumer_warps(1)) + rep * max_seq * 2;
  const int64_t need_nt2 = rep * head_dim * 4 * (1 + prog_consumer_warps(2)) + rep * max_seq * 2;
  if (need_nt1 > prog_xs_bytes(1) && need_nt2 > prog_xs_bytes(2))
    return set_error(LI4_ERR_UNSUPPORTED, "program_add_attention: max_seq=%lld does not fit the CTA's shared memory "
                     "(use li4_decode_attention)", (long long)max_seq);
  ProgOp op = {};
  op.kind = kOpAttention;
  op.wait = wait;
  op.units = (int)(batch * n_kv_heads);
  op.at.q = static_cast<const __half*>(q);
  op.at.sqb = stride_qb;
  op.at.ck = static_cast<const __half*>(cache_k);
  op.at.cv = static_cast<const __half*>(cache_v);
  op.at.csb = cache_stride_b;
  op.at.css = cache_stride_s;
  op.at.out = static_cast<__half*>(out);
  op.at.sob = stride_ob;
  op.at.n_kv = (int)n_kv_heads;
  op.at.rep = (int)rep;
  op.at.hd = (int)head_dim;
  op.at.pos = reinterpret_cast<const long long*>(pos);
  op.at.max_seq = (int)max_seq;
  return add_op(prog, op, 0, op_index);
}

extern "C" int li4_program_add_gather(li4_program* prog, const void* table, int64_t table_rows, int64_t cols,
                                      int64_t stride_t, const int64_t* ids, int64_t rows, void* out, int64_t stride_o,
                                      int wait, int* op_index) {
  using namespace li4;
  if (!prog) return set_error(LI4_ERR_INVALID_ARG, "program_add_gather: null program");
  if (!table || !ids || !out || table_rows < 1 || rows < 1 || rows > INT32_MAX / 2 || cols < 8 || cols % 8 != 0 ||
      cols > INT32_MAX / 2 || stride_t < cols || stride_o < cols)
    return set_error(LI4_ERR_INVALID_ARG, "program_add_gather: rows=%lld cols=%lld (cols %% 8 == 0) strides %lld, %lld",
                     (long long)rows, (long long)cols, (long long)stride_t, (long long)stride_o);
  if (!aligned16(table) || !aligned16(out) || stride_t % 8 != 0 || stride_o % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(ids) & 7u))
    return set_error(LI4_ERR_ALIGNMENT, "program_add_gather: rows must be 16-byte aligned");
  ProgOp op = {};
  op.kind = kOpGather;
  op.wait = wait;
  op.units = (int)rows;
  op.ga.table = static_cast<const __half*>(table);
  op.ga.table_rows = table_rows;
  op.ga.stride_t = stride_t;
  op.ga.ids = reinterpret_cast<const long long*>(ids);
  op.ga.cols = (int)cols;
  op.ga.out = static_cast<__half*>(out);
  op.ga.stride_o = stride_o;
  return add_op(prog, op, 0, op_index);
}

extern "C" int li4_program_add_argmax(li4_program* prog, const float* logits, int64_t rows, int64_t cols,
                                      int64_t stride, int64_t* out, int64_t out_stride, int wait, int* op_index) {
  using namespace li4;
  if (!prog) return set_error(LI4_ERR_INVALID_ARG, "program_add_argmax: null program");
  if (!logits || !out || rows < 1 || cols < 1 || cols > INT32_MAX / 2 || stride < cols || out_stride < 1)
    return set_error(LI4_ERR_INVALID_ARG, "program_add_argmax: rows=%lld cols=%lld stride=%lld out_stride=%lld",
                     (long long)rows, (long long)cols, (long long)stride, (long long)out_stride);
  if ((reinterpret_cast<uintptr_t>(logits) & 3u) || (reinterpret_cast<uintptr_t>(out) & 7u))
    return set_error(LI4_ERR_ALIGNMENT, "program_add_argmax: misaligned logits or output");
  ProgOp op = {};
  op.kind = kOpArgmax;
  op.wait = wait;
  op.finalize = 1;
  op.am.logits = logits;
  op.am.stride = stride;
  op.am.cols = (int)cols;
  op.am.n_chunks = (int)((cols + kArgmaxColChunk - 1) / kArgmaxColChunk);
  op.am.out = reinterpret_cast<long long*>(out);
  op.am.out_stride = out_stride;
  if (rows * op.am.n_chunks > INT32_MAX / 2) return set_error(LI4_ERR_INVALID_ARG, "program_add_argmax: too large");
  op.units = (int)(rows * op.am.n_chunks);
  return add_op(prog, op, (size_t)rows * 8, op_index);
}

extern "C" int li4_program_add_increment(li4_program* prog, int64_t* value) {
  using namespace li4;
  if (!prog || !value) return set_error(LI4_ERR_INVALID_ARG, "program_add_increment: null pointer");
  if (prog->finalized) return set_error(LI4_ERR_INVALID_ARG, "program: finalized programs take no more ops");
  if ((reinterpret_cast<uintptr_t>(value) & 7u)) return set_error(LI4_ERR_ALIGNMENT, "program_add_increment: misaligned");
  if ((int)prog->incr.size() >= kProgMaxIncrements)
    return set_error(LI4_ERR_UNSUPPORTED, "program_add_increment: at most %d increments", kProgMaxIncrements);
  prog->incr.push_back(reinterpret_cast<long long*>(value));
  clear_error();
  return LI4_OK;
}

extern "C" int li4_program_finalize(li4_program* prog) {
  using namespace li4;
  if (!prog) return set_error(LI4_ERR_INVALID_ARG, "program_finalize: null program");
  if (prog->finalized) return set_error(LI4_ERR_INVALID_ARG, "program_finalize: already finalized");
  if (prog->ops.empty()) return set_error(LI4_ERR_INVALID_ARG, "program_finalize: no ops");
  int rc = check_cuda(cudaGetDevice(&prog->device), "program_finalize: cudaGetDevice");
  if (rc != LI4_OK) return rc;
  const int G = current_sm_count();
  int max_m = 1;
  for (const ProgOp& op : prog->ops)
    if (op.kind == kOpLinear) max_m = std::max(max_m, op.g.M);
  prog->nt = max_m <= 8 ? 1 : 2;
  const int cw = prog_consumer_warps(prog->nt);
  const size_t smem = (size_t)prog_smem_bytes(prog->nt);
  int blocks = 0;
  rc = prog->nt == 1 ? program_occupancy<1>(smem, &blocks) : program_occupancy<2>(smem, &blocks);
  if (rc != LI4_OK) return rc;
  if (blocks < 1) return set_error(LI4_ERR_UNSUPPORTED, "program_finalize: the program CTA does not fit an SM");
  prog->ctas = G;  // one CTA per SM: every CTA is resident for the whole launch
  // rotate each op's round-robin by the units before it, and check what depends on the launch shape
  long long before = 0;
  for (size_t j = 0; j < prog->ops.size(); ++j) {
    ProgOp& op = prog->ops[j];
    op.rot = (int)(before % G);
    before += op.units;
    if (op.kind == kOpLinear && op.chunks > G)
      return set_error(LI4_ERR_UNSUPPORTED, "program_finalize: op %zu has %d K ranges, more than %d CTAs", j,
                       op.chunks, G);
    if (op.kind == kOpAttention) {
      const long long need = (long long)op.at.rep * op.at.hd * 4 * (1 + cw) + (long long)op.at.rep * op.at.max_seq * 2;
      if (need > prog_xs_bytes(prog->nt))
        return set_error(LI4_ERR_UNSUPPORTED, "program_finalize: attention op %zu needs %lld bytes of shared memory "
                         "at batch %d (max_seq %d), the CTA has %d", j, need, max_m, op.at.max_seq,
                         prog_xs_bytes(prog->nt));
    }
  }
  // device state: op table | counters (+ exit counter) | per-op scratch, each 256-byte aligned
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  const size_t n = prog->ops.size();
  const size_t off_done = up(n * sizeof(ProgOp));
  size_t total = off_done + up((n + 1) * sizeof(unsigned));
  std::vector<size_t> off(n, 0);
  for (size_t j = 0; j < n; ++j) {
    if (prog->scratch_bytes[j] == 0) continue;
    off[j] = total;
    const ProgOp& op = prog->ops[j];
    total += op.kind == kOpLinear ? up((size_t)op.g.n_tiles * 4) + up((size_t)op.chunks * op.g.M * op.g.N * 4)
                                  : up(prog->scratch_bytes[j]);
  }
  void* dev = nullptr;
  rc = check_cuda(cudaMalloc(&dev, total), "program_finalize: cudaMalloc");
  if (rc != LI4_OK) return rc;
  uint8_t* base = static_cast<uint8_t*>(dev);
  for (size_t j = 0; j < n; ++j) {
    ProgOp& op = prog->ops[j];
    if (op.kind == kOpLinear && op.chunks > 1) {
      op.g.counters = reinterpret_cast<unsigned*>(base + off[j]);
      op.g.partial = reinterpret_cast<float*>(base + off[j] + up((size_t)op.g.n_tiles * 4));
    } else if (op.kind == kOpArgmax) {
      op.am.keys = reinterpret_cast<unsigned long long*>(base + off[j]);
    }
  }
  rc = check_cuda(cudaMemset(dev, 0, total), "program_finalize: cudaMemset");
  if (rc == LI4_OK)
    rc = check_cuda(cudaMemcpy(dev, prog->ops.data(), n * sizeof(ProgOp), cudaMemcpyHostToDevice),
                    "program_finalize: uploading the op table");
  if (rc != LI4_OK) {
    cudaFree(dev);
    return rc;
  }
  prog->dev = dev;
  ProgArgs& a = prog->args;
  a.ops = reinterpret_cast<const ProgOp*>(base);
  a.n_ops = (int)n;
  a.done = reinterpret_cast<unsigned*>(base + off_done);
  a.n_incr = (int)prog->incr.size();
  for (int k = 0; k < a.n_incr; ++k) a.incr[k] = prog->incr[k];
  a.trace = nullptr;
  prog->finalized = true;
  clear_error();
  return LI4_OK;
}

extern "C" int li4_program_launch(li4_program* prog, void* stream) {
  using namespace li4;
  if (!prog || !prog->finalized) return set_error(LI4_ERR_INVALID_ARG, "program_launch: program not finalized");
  int cur = -1;
  int rc = check_cuda(cudaGetDevice(&cur), "program_launch: cudaGetDevice");
  if (rc != LI4_OK) return rc;
  if (cur != prog->device)
    return set_error(LI4_ERR_INVALID_ARG, "program_launch: the program was built on device %d, current is %d",
                     prog->device, cur);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)prog->ctas, 1, 1);
  cfg.blockDim = dim3((unsigned)prog_threads(prog->nt), 1, 1);
  cfg.dynamicSmemBytes = (size_t)prog_smem_bytes(prog->nt);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  rc = prog->nt == 1 ? check_cuda(cudaLaunchKernelEx(&cfg, decode_program_kernel<1>, prog->args), "program_launch")
                     : check_cuda(cudaLaunchKernelEx(&cfg, decode_program_kernel<2>, prog->args), "program_launch");
  if (rc == LI4_OK) clear_error();
  return rc;
}

extern "C" int li4_program_set_trace(li4_program* prog, int64_t* stamps, int64_t capacity) {
  using namespace li4;
  if (!prog || !prog->finalized) return set_error(LI4_ERR_INVALID_ARG, "program_set_trace: program not finalized");
  const int64_t need = (int64_t)prog->ops.size() * prog->ctas * 4;
  if (stamps && capacity < need)
    return set_error(LI4_ERR_INVALID_ARG, "program_set_trace: %lld stamps needed, %lld given", (long long)need,
                     (long long)capacity);
  if ((reinterpret_cast<uintptr_t>(stamps) & 7u)) return set_error(LI4_ERR_ALIGNMENT, "program_set_trace: misaligned");
  prog->args.trace = reinterpret_cast<long long*>(stamps);
  clear_error();
  return LI4_OK;
}

extern "C" int li4_program_info(const li4_program* prog, int* ctas, int* stages, size_t* smem_bytes) {
  using namespace li4;
  if (!prog || !prog->finalized) return set_error(LI4_ERR_INVALID_ARG, "program_info: program not finalized");
  if (ctas) *ctas = prog->ctas;
  if (stages) *stages = prog_consumer_warps(prog->nt);
  if (smem_bytes) *smem_bytes = (size_t)prog_smem_bytes(prog->nt);
  clear_error();
  return LI4_OK;
}
