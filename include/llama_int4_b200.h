/*
 * llama_int4_b200.h -- C ABI of the B200 (sm_100a) INT4 weight-only decode kernels.
 *
 * Weight format (identical to the reference's QuantizedLinear buffers,
 * llama/quantize.py:29-36 and :44-75):
 *   packed [N, K/2] uint8, row-major, row stride `stride_pn` bytes.
 *          byte j of row n = q[n, 2j] | (q[n, 2j+1] << 4)   (low nibble = even k)
 *   scale  [N, K/group] fp16, row stride `stride_sn` elements
 *   zero   [N, K/group] fp16, same row stride as scale; integers 0..15
 *   W[n, k] = fp16((q[n,k] - zero[n, k/group]) * scale[n, k/group])
 *
 * All pointers are device pointers unless stated otherwise; `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  No entry point
 * allocates device memory, synchronises the device or aborts: each returns an
 * li4_status and records a message readable with li4_last_error().
 * fp16 values are passed as raw 16-bit IEEE half storage (uint16_t / void*).
 */
#ifndef LLAMA_INT4_B200_H
#define LLAMA_INT4_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum li4_status {
  LI4_OK = 0,
  LI4_ERR_INVALID_ARG = 1,   /* shape, stride or null-pointer precondition failed   */
  LI4_ERR_ALIGNMENT = 2,     /* a pointer/stride breaks the 16-byte load contract    */
  LI4_ERR_WORKSPACE = 3,     /* split-K workspace missing or too small               */
  LI4_ERR_UNSUPPORTED = 4,   /* valid for the reference, not handled by these kernels */
  LI4_ERR_CUDA = 5           /* a CUDA runtime call or kernel launch failed          */
} li4_status;

typedef enum li4_dtype {
  LI4_F16 = 0,
  LI4_BF16 = 1,
  LI4_F32 = 2
} li4_dtype;

/* Largest M (rows of x) the decode kernels take.
 * Replaces: MAX_M = 16 (llama/int4_gemv.py:29). */
#define LI4_MAX_M 16

/* Kernel families li4_int4_linear_ex can be forced to (LI4_KERNEL_AUTO lets the
 * dispatcher choose from M, N, K and the SM count). */
typedef enum li4_kernel {
  LI4_KERNEL_AUTO = 0,
  LI4_KERNEL_CUDA_CORE = 1,  /* fp32 FMA on CUDA cores, M <= 8                      */
  LI4_KERNEL_MMA = 2,        /* m16n8k16 tensor-core tiles (weights as the A side)  */
  LI4_KERNEL_STREAM = 3,     /* streaming warps, m16n8k16 tiles, groups >= 128      */
  LI4_KERNEL_TILE = 4,       /* tile-streaming warps: group 128, K ranges of 2048  */
  LI4_KERNEL_BULK = 5,       /* bulk-copy ring in shared memory: group 128,
                                K % 1024 == 0, 16-byte aligned scale / zero rows   */
  LI4_KERNEL_SLAB = 6,       /* whole weight slice of a CTA resident in shared
                                memory, K split across its warps: group 128, up to
                                16 row tiles per CTA                              */
  LI4_KERNEL_ROWS = 7,       /* a warp's two rows unpacked in registers before the
                                dependency wait: M = 1, group 128, K = 1024 or 2048,
                                16-byte aligned x; no RMSNorm prologue or argmax  */
  LI4_KERNEL_RING = 8        /* shared-memory ring of 16/32/64-row stages filled by
                                bulk copies, 16 consumer warps per SM: group 128,
                                M <= 8, K % 1024 == 0, M * K <= 32768, 16-byte
                                aligned rows; rows_per_cta picks the stage rows   */
} li4_kernel;

/* Library version, (major << 16) | (minor << 8) | patch.  0.2: li4_fusion has the argmax_*
 * fields (callers built against 0.1 pass a shorter struct); the li4_program_* and
 * li4_gather_rows entry points. */
int li4_version(void);

/* Message describing the last failed call on this host thread ("" if none). */
const char* li4_last_error(void);

/* Split-K workspace layout: the first LI4_WORKSPACE_COUNTER_BYTES bytes hold
 * per-row-tile arrival counters (never used for anything else), fp32 partial
 * sums follow. */
#define LI4_WORKSPACE_COUNTER_BYTES 65536

/* Bytes of split-K workspace li4_int4_linear needs for this problem on a
 * device with `sm_count` SMs (0 = query the current device); 0 when the
 * launch needs none.  The workspace must be zero-filled once when it is
 * allocated; every launch leaves its arrival counters at zero again, so it can
 * be reused by later launches of any shape on the same stream (and inside
 * CUDA graphs) without clearing.  Two launches that may run concurrently must
 * not share a workspace. */
size_t li4_int4_linear_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t group_size, int sm_count);

/* y[M, N] (fp16, row stride stride_ym elements) = x[M, K] (fp16, row stride
 * stride_xm) @ W^T, W given in the packed INT4 format above.  fp32
 * accumulation; one kernel launch (split-K partial sums are reduced by the
 * last-arriving CTA inside the same launch).  M in 1..16, K % 128 == 0,
 * group_size a power of two >= 32 dividing K, packed rows 16-byte aligned.
 * The launch is marked for programmatic dependent launch: its weight loads
 * may overlap the tail of the preceding kernel on the stream; x is read only
 * after that kernel has completed.
 * Replaces: int4_linear (llama/int4_gemv.py:105-140) and its Triton kernel
 * _int4_gemv_kernel (llama/int4_gemv.py:32-89), including the split-K
 * zero-fill / atomic_add / .half() epilogue (llama/int4_gemv.py:126-139). */
int li4_int4_linear(const void* x, const void* packed, const void* scale, const void* zero, void* y,
                    int64_t M, int64_t N, int64_t K, int64_t group_size,
                    int64_t stride_xm, int64_t stride_pn, int64_t stride_sn, int64_t stride_ym,
                    void* workspace, size_t workspace_bytes, void* stream);

/* li4_int4_linear with an explicit kernel family and launch shape, for tuning
 * sweeps: kernel (li4_kernel), rows_per_cta (16 or 32; 0 = auto), split
 * (number of K ranges, 0 = auto), max_ctas (0 = auto).
 * Replaces: the block_n / split_k / num_warps tuning knobs of int4_linear
 * (llama/int4_gemv.py:105, swept by int4_gemv_bench.py:80-90). */
int li4_int4_linear_ex(const void* x, const void* packed, const void* scale, const void* zero, void* y,
                       int64_t M, int64_t N, int64_t K, int64_t group_size,
                       int64_t stride_xm, int64_t stride_pn, int64_t stride_sn, int64_t stride_ym,
                       void* workspace, size_t workspace_bytes, void* stream,
                       int kernel, int rows_per_cta, int split, int max_ctas);

/* The launch plan li4_int4_linear chooses for this problem on a device with
 * `sm_count` SMs (0 = the current device), for contiguous, 16-byte aligned
 * operands: the kernel family (li4_kernel), the number of K ranges (split),
 * the CTAs along N per K range (grid_x; the streaming-warp and tile kernels
 * cap it by occupancy at launch) and the dynamic shared memory per CTA.  Any
 * output pointer may be null.  Launches nothing.
 * Replaces: nothing in the reference, whose int4_linear picks split-K in
 * _split_k (llama/int4_gemv.py:95-102) without reporting it; benchmarks and
 * profiles use it to name the kernel each shape runs on. */
int li4_int4_linear_plan(int64_t M, int64_t N, int64_t K, int64_t group_size, int sm_count,
                         int* kernel, int* split, int* grid_x, size_t* smem_bytes);

/* One problem of a grouped launch: y[M, N] = x[M, K] @ W^T with this problem's own x, packed
 * weights, scales, zeros and y (fp16; strides as li4_int4_linear's). */
typedef struct li4_gemv_problem {
  const void* x;
  const void* packed;
  const void* scale;
  const void* zero;
  void* y;
  int64_t N, K;
  int64_t stride_xm, stride_pn, stride_sn, stride_ym;
} li4_gemv_problem;

/* Many independent INT4 GEMVs in one persistent launch.  The problems' 16-row tiles, in list
 * order, are cut into contiguous ranges of about equal weight bytes, one per CTA of a full wave;
 * a CTA stages the x of the few problems its range touches once and each of its warps streams
 * its tiles through one register ring that runs on across tile and problem boundaries, so the
 * weight stream of every problem runs in one kernel with no launch boundary or barrier between
 * tiles.  Same math and rounding as li4_int4_linear.  M in 1..8, group_size 128, K a multiple
 * of 128 with M * K * 2 <= 32768 bytes, packed rows 16-byte aligned.
 * li4_int4_linear_grouped_table_bytes gives the size of the device table (0 for an invalid
 * list) and in *units the number of ranges (the ranges depend on the current device's SM
 * count: build and launch on the same kind of device); li4_int4_linear_grouped_build validates
 * the list and writes the table (a synchronous host-to-device copy: build once, launch many);
 * li4_int4_linear_grouped launches with that `units` (no host data; a launch writes only the
 * outputs, so launches repeat and overlap freely on one table).
 * Replaces: a sequence of the reference's int4_linear calls (llama/int4_gemv.py:105-140) on
 * independent inputs, one kernel launch each. */
size_t li4_int4_linear_grouped_table_bytes(const li4_gemv_problem* problems, int n, int64_t M, int* units);
int li4_int4_linear_grouped_build(const li4_gemv_problem* problems, int n, int64_t M, int64_t group_size,
                                  void* table, size_t table_bytes);
int li4_int4_linear_grouped(const void* table, int n, int units, int64_t M, void* stream);

/* y[M, N] = x[M, K] @ W^T on the tensor cores (tcgen05, fp32 accumulation in tensor
 * memory) for any M >= 1, meant for prefill (M > 16).  The fp16 weights are rebuilt in
 * shared memory tile by tile, bit-identical to dequantize_packed's fp16((q - zero) * scale),
 * so the result is the reference's dequantize + F.linear up to the order of the fp32 sums.
 * group_size 128, K a multiple of 128, x rows and packed rows 16-byte aligned (stride_xm
 * % 8 == 0).  One launch; no workspace; no host synchronisation.  A bounded wait inside the
 * kernel that runs out sets bit 4 of li4_device_errors.
 * Replaces: the prefill branch of QuantizedLinear.forward, dequant_fn("v3") + F.linear
 * (llama/quantize.py:143-146, 199-202). */
int li4_int4_gemm(const void* x, const void* packed, const void* scale, const void* zero, void* y,
                  int64_t M, int64_t N, int64_t K, int64_t group_size,
                  int64_t stride_xm, int64_t stride_pn, int64_t stride_sn, int64_t stride_ym, void* stream);

/* Size of the static device scratch behind li4_int4_linear_noalloc. */
#define LI4_NOALLOC_SCRATCH_BYTES (4u << 20)

/* li4_int4_linear for callers that cannot allocate device memory: code running
 * while a CUDA graph is captured, runtimes whose allocator refuses new device
 * allocations after warm-up (cudaMalloc may synchronise the device), and
 * hosts that bind only this C ABI and own no device allocator.  The caller
 * still passes x and y; the split-K partial sums and arrival counters live in
 * a static device array of LI4_NOALLOC_SCRATCH_BYTES (4 MiB) that every GPU
 * loading the library holds until the process exits.  This function calls no
 * cudaMalloc / cudaFree; it clears the counters it uses with cudaMemsetAsync
 * on `stream` before each launch.  Problems whose split-K scratch would exceed
 * the array are rejected with LI4_ERR_WORKSPACE (for example M=16, N=32768,
 * K=8192).  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, which may load the module): make that first call
 * before any stream capture.  The address is cached per device ordinal for the
 * life of the process: a device reset (cudaDeviceReset) between calls is not
 * supported.  All calls share the array, so calls that may overlap on the GPU
 * (different streams) race; keep them on one stream.
 * No counterpart in the reference: its int4_linear allocates its split-K
 * buffer with torch.zeros on every call. */
int li4_int4_linear_noalloc(const void* x, const void* packed, const void* scale, const void* zero, void* y,
                            int64_t M, int64_t N, int64_t K, int64_t group_size,
                            int64_t stride_xm, int64_t stride_pn, int64_t stride_sn, int64_t stride_ym,
                            void* stream);

/* ---------------------------------------------------------------------------
 * Fused decode-step operations.  The decode step of a Llama block is
 *   h   = x + wo(attn(rope(wq(norm1(x))), rope(wk(norm1(x))), wv(norm1(x))))
 *   out = h + w2(silu(w1(norm2(h))) * w3(norm2(h)))
 * (llama/model.py:222-277, 310-315, 358-362).  li4_int4_linear_fused folds the
 * RMSNorm into the GEMV's x staging and RoPE + KV-cache write, SwiGLU or the
 * residual add into its epilogue, so a block is five launches: QKV, attention,
 * wo, gate/up, w2.  The rounding points are the reference's: every GEMV output
 * is rounded to fp16 before the epilogue works on it, and every intermediate
 * the reference holds in fp16 is rounded to fp16 here too.
 *
 * Paired rows.  SwiGLU and RoPE combine two GEMV outputs.  These epilogues take
 * the packed weight with its rows arranged so that rows 16t + j and 16t + 8 + j
 * (j < 8) form pair 8t + j, which puts both values in one thread; N must then be
 * a multiple of 16.
 *   LI4_EPI_SWIGLU:   pair p = (row p of w1, row p of w3); y[m, p], y has N/2
 *                     columns.
 *   LI4_EPI_QKV_ROPE: the rows of [wq; wk; wv] (q_rows + k_rows + v_rows = N),
 *                     pair p = rows (2p, 2p + 1), the (even, odd) pair that RoPE
 *                     rotates as one complex number (llama/model.py:126-152).
 * --------------------------------------------------------------------------- */
typedef enum li4_epilogue_kind {
  LI4_EPI_STORE = 0,     /* y = fp16(x W^T)                                          */
  LI4_EPI_RESIDUAL = 1,  /* y = fp16(residual + fp16(x W^T))                         */
  LI4_EPI_SWIGLU = 2,    /* y = fp16(fp16(silu(g)) * u), g, u = fp16 outputs of pair  */
  LI4_EPI_QKV_ROPE = 3,  /* RoPE on q, k pairs at position *pos; q -> q_out,
                            k and v -> cache_k / cache_v at row *pos (y unused)       */
  LI4_EPI_STORE_F32 = 4, /* y is fp32 [M, N] (row stride in fp32 elements):
                            y = (float)fp16(x W^T), the reference's output(h).float() */
  LI4_EPI_ALLREDUCE_RESIDUAL = 5  /* row-parallel linear under tensor parallelism:
                            y = fp16(residual + fp16(sum_r P_r)), P_r = fp16(x W_r^T) of
                            rank r, summed in fp32 in rank order (ar_* fields)          */
} li4_epilogue_kind;

typedef struct li4_fusion {
  /* Prologue: x -> fp16(fp16(x * rsqrt(mean(x^2) + eps)) * norm_weight), the
   * mean over all K columns in fp32 (llama/model.py:61-75).  NULL = no norm. */
  const void* norm_weight;  /* fp16 [K] */
  float norm_eps;
  int epilogue;             /* li4_epilogue_kind */
  /* LI4_EPI_RESIDUAL: fp16 [M, N], row stride stride_rm elements; may equal y. */
  const void* residual;
  int64_t stride_rm;
  /* LI4_EPI_QKV_ROPE (M = batch rows, one new token each, all at *pos). */
  int64_t q_rows, k_rows, head_dim;         /* v_rows = N - q_rows - k_rows           */
  const int64_t* pos;                       /* device scalar                         */
  const float* rope_cos;                    /* [positions, head_dim / 2] fp32         */
  const float* rope_sin;
  int64_t rope_stride;                      /* elements between positions             */
  void* q_out;                              /* fp16 [M, q_rows], row stride stride_qm */
  int64_t stride_qm;
  void* cache_k;                            /* fp16 [batch, seq, k_rows] with strides */
  void* cache_v;                            /* (elements) cache_stride_b / _s         */
  int64_t cache_stride_b, cache_stride_s;
  /* Sums of squares handed from a residual epilogue to the next RMSNorm prologue, so the
   * norm needs no pass over x: with LI4_EPI_RESIDUAL, sumsq_out (fp32 [ceil(N/16)][M])
   * receives, per 16-row tile and row m, the sum of the written fp16 values squared; a
   * launch with norm_weight and sumsq_in = that array (sumsq_tiles = ceil(K/16)) takes its
   * mean of squares from it.  NULL = not used. */
  float* sumsq_out;
  const float* sumsq_in;
  int64_t sumsq_tiles;
  /* Greedy argmax of the written logits (LI4_EPI_STORE_F32 only): argmax_out[m * argmax_stride]
   * = torch.argmax(y[m, :N]) (int64), written by the launch's last CTA.  argmax_scratch: device
   * memory of 8 * M + 8 bytes, zero before the first use; launches leave it zero (launches that
   * may overlap need their own).  Runs on the tile kernel (lm_head-sized N at M <= 8); other
   * launch plans return LI4_ERR_UNSUPPORTED.  NULL = not used. */
  int64_t* argmax_out;
  int64_t argmax_stride;
  void* argmax_scratch;
  /* LI4_EPI_ALLREDUCE_RESIDUAL (also needs residual / stride_rm; N % 16 == 0).  The launch
   * pushes its fp16 partial P_rank to every rank as 8-byte words -- two outputs (rows j and
   * j + 8 of a 16-row tile) and the call's epoch -- stored straight into each rank's receive
   * buffer over NVLink, then waits (bounded) until its own buffer holds every rank's words of
   * the same tiles and writes y.  Receive buffer layout: [world][N / 16][M][8] words of
   * 8 bytes (sender outermost).  ar_recv: host array of ar_world device pointers, rank r's
   * buffer at [r] (the peers' mapped through CUDA IPC), each ar_recv_bytes long;
   * ar_epochs: this rank's uint32 call counts per 16-row tile [N / 16], zero before the
   * first call and updated by the launch.  Every rank makes the same sequence of calls on a
   * buffer; two calls in a row use different buffers (and epoch arrays), so a rank never
   * overwrites words a peer is still reading.  Runs on the streaming-warp kernel.  A wait
   * that runs out sets bit 5 of li4_device_errors and the launch finishes with what it read. */
  void* const* ar_recv;
  size_t ar_recv_bytes;
  unsigned* ar_epochs;
  int ar_world, ar_rank;
} li4_fusion;

/* li4_int4_linear with a fused prologue / epilogue (`fusion` NULL = plain).
 * Uses the streaming-warp or tile kernel (group_size >= 128).  The workspace
 * rule is li4_int4_linear's.  Replaces, inside one launch: RMSNorm.forward
 * (llama/model.py:61-75), apply_rotary_emb and the cache writes of
 * Attention.forward (:126-152, :251-262), F.silu(w1(x)) * w3(x) (:315) and the
 * residual adds of TransformerBlock.forward (:358-362). */
int li4_int4_linear_fused(const void* x, const void* packed, const void* scale, const void* zero, void* y,
                          int64_t M, int64_t N, int64_t K, int64_t group_size,
                          int64_t stride_xm, int64_t stride_pn, int64_t stride_sn, int64_t stride_ym,
                          const li4_fusion* fusion, void* workspace, size_t workspace_bytes, void* stream);

/* Decode attention for one new token per sequence at position *pos:
 *   out[b, h] = softmax(q[b, h] . K[b, 0..pos, h / rep]^T / sqrt(head_dim)) V[b, 0..pos, h / rep]
 * with rep = n_heads / n_kv_heads (grouped-query attention without the
 * repeat_kv copies).  Scores are rounded to fp16 (the reference's fp16
 * matmul), the softmax is fp32, the probabilities are rounded to fp16 and
 * P.V accumulates in fp32 (llama/model.py:266-275).  q: fp16 [batch, n_heads *
 * head_dim] (row stride stride_qb); cache_k / cache_v: fp16 [batch, seq,
 * n_kv_heads, head_dim] with element strides cache_stride_b / cache_stride_s;
 * out: fp16 [batch, n_heads * head_dim] (row stride stride_ob).  head_dim 32, 64 or 128;
 * *pos < max_seq (the kernel clamps to max_seq - 1).  Launched with programmatic
 * dependent launch: q and cache row *pos may come from the preceding kernel on the
 * stream, but the rows before *pos are read while that kernel may still run, so
 * they must have been written before it (as a decode step's earlier positions are).
 * Replaces: Attention.forward's repeat_kv, two matmuls and softmax
 * (llama/model.py:262-275) at seqlen 1. */
int li4_decode_attention(const void* q, int64_t stride_qb, const void* cache_k, const void* cache_v,
                         int64_t cache_stride_b, int64_t cache_stride_s, void* out, int64_t stride_ob,
                         int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                         const int64_t* pos, int64_t max_seq, void* stream);

/* out[r * out_stride] = argmax of row r of logits [rows, cols] (dtype LI4_F16 or
 * LI4_F32, row stride `stride` elements): the first index of the row's maximum,
 * a NaN counting as the maximum, as torch.argmax.  One cluster of 8 CTAs per row.
 * Replaces: the greedy logits[:, -1].argmax(-1) of the decode loop
 * (bench.py:154-161, llama/generation.py:59-60). */
int li4_argmax_rows(const void* logits, int dtype, int64_t rows, int64_t cols, int64_t stride,
                    int64_t* out, int64_t out_stride, void* stream);

/* The row winners of li4_argmax_rows as keys for a vocabulary split over ranks:
 * keys[r * keys_stride] = a signed 64-bit key of the winner of row r at global index
 * index_offset + its column, ordered as torch.argmax orders candidates (larger value, NaN
 * above all, then the smaller index).  The largest key over the ranks' shards (an int64 MAX
 * all-reduce) is the winner over the whole row; its index is 0xFFFFFFFF - (key & 0xFFFFFFFF).
 * Replaces: the all-gather of the vocabulary-sharded logits and the argmax over the
 * gathered row at tensor-parallel decode (greedy step of llama/generation.py:59-60). */
int li4_argmax_rows_keys(const void* logits, int dtype, int64_t rows, int64_t cols, int64_t stride,
                         int64_t index_offset, int64_t* keys, int64_t keys_stride, void* stream);

/* The greedy step of a vocabulary-sharded lm_head under tensor parallelism, in one launch:
 * every rank finds the winner of its shard (columns index_offset .. index_offset + cols - 1 of
 * the full vocabulary) as li4_argmax_rows_keys does, stores its key into every rank's receive
 * buffer over NVLink as two 8-byte words that carry the call's epoch, waits (bounded) for every
 * rank's key of the row in its own buffer, and writes out[r * out_stride] = the global index of
 * the largest key -- torch.argmax over the gathered logits.  Receive buffer layout:
 * [2][world][rows][2] words of 8 bytes (the epoch's parity picks the half); recv: host array of
 * world device pointers, rank r's buffer at [r] (the peers' through CUDA IPC), each recv_bytes
 * long; epochs: this rank's uint32 call counts per row, zero before the first call.  Every rank
 * makes the same calls with the same rows.  A wait that runs out sets bit 6 of
 * li4_device_errors.  Replaces: the reference's greedy logits[:, -1].argmax(-1) (bench.py:154-161)
 * over logits that tensor parallelism would all-gather first. */
int li4_argmax_rows_allreduce(const void* logits, int dtype, int64_t rows, int64_t cols, int64_t stride,
                              int64_t index_offset, void* const* recv, size_t recv_bytes, unsigned* epochs,
                              int world, int rank, int64_t* out, int64_t out_stride, void* stream);

/* out[r, :] = table[ids[r], :] for r < rows: fp16 rows of `cols` values (cols % 8 == 0,
 * 16-byte aligned rows; rows <= 65535).  An id outside [0, table_rows) is clamped and
 * sets bit 3 of li4_device_errors.  The ids may come from the preceding kernel on the
 * stream (programmatic dependent launch: they are read after its completion).
 * Replaces: the token embedding lookup of the decode step (llama/model.py:440). */
int li4_gather_rows(const void* table, int64_t table_rows, int64_t cols, int64_t stride_t, const int64_t* ids,
                    int64_t rows, void* out, int64_t stride_o, void* stream);

/* Device-side error flags of the current device (bit 0: a bounded pipeline wait
 * inside a GEMV kernel ran out; bit 1: a bounded wait for a peer's flag in
 * li4_allreduce_add ran out; bit 2: a decode program's wait for another op
 * ran out; bit 3: a gather (li4_gather_rows or a program gather) met an id
 * outside its table; bit 4: a bounded wait inside li4_int4_gemm ran out; bit 5: an
 * LI4_EPI_ALLREDUCE_RESIDUAL epilogue's wait for a peer's words ran out; bit 6: a wait of
 * li4_argmax_rows_allreduce for a peer's key ran out -- the kernel
 * carried on and its outputs are not valid).  Synchronising: copies the flags to the host; reset != 0 clears them.
 * A diagnostic for tests and health checks, not for the decode loop. */
int li4_device_errors(unsigned* flags, int reset);

/* Test hook for the bounded device waits: the poll limit of li4_allreduce_add's
 * peer-flag waits, of the LI4_EPI_ALLREDUCE_RESIDUAL epilogue's waits for the
 * peers' words and of li4_argmax_rows_allreduce's waits for the peers' keys
 * (allreduce_polls), the poll limit of the decode program's
 * op-counter waits (program_polls) -- 0 restores each default (about a second
 * of polling) -- and, when program_wait_extra > 0, a target no program counter
 * wait can meet.  With a short limit a test can make a wait run out without a
 * fault: the kernel sets its bit in li4_device_errors and returns.  Applies to
 * the current device; synchronous.  No counterpart in the reference (it has no
 * device waits). */
int li4_debug_set_wait_limits(unsigned allreduce_polls, unsigned program_polls, unsigned program_wait_extra);

/* ---------------------------------------------------------------------------
 * Tensor-parallel all-reduce over NVLink peer memory (one GPU per process).
 * Every rank allocates one communication buffer (li4_comm_alloc), exports it
 * (li4_ipc_get_handle), exchanges the handles with the other ranks through the
 * host, and maps the peers' buffers (li4_ipc_open_handle).  Each buffer holds
 * two partial-sum slots and a flag array of ctas x world uint32, zeroed at
 * allocation; each rank also keeps ctas uint32 call counts, zeroed.
 * --------------------------------------------------------------------------- */
#define LI4_IPC_HANDLE_BYTES 64

/* cudaMalloc + zero fill of a buffer that other processes can map. */
int li4_comm_alloc(size_t bytes, void** dev_ptr);
int li4_comm_free(void* dev_ptr);
/* The IPC handle (LI4_IPC_HANDLE_BYTES bytes, host memory) of a li4_comm_alloc buffer. */
int li4_ipc_get_handle(void* dev_ptr, void* handle);
/* Map a peer's buffer from its handle (peer access enabled on first use). */
int li4_ipc_open_handle(const void* handle, void** dev_ptr);
int li4_ipc_close(void* dev_ptr);

/* out[0..n) = fp16(residual + fp16(sum over ranks of slots[r][0..n))), the sum in
 * fp32 in rank order; slots[r] is this call's slot (fp16, 16-byte aligned) in rank
 * r's buffer, written by this rank's preceding kernel for r == rank.  flags[r]
 * is rank r's flag array, counts this rank's call counts.  Every rank must make
 * the same sequence of calls, alternating the two slots, with the same ctas.
 * The kernel waits for all peers' flags (bounded); ranks run on separate GPUs.
 * slots and flags are host arrays of device pointers (world entries, <= 8).
 * Replaces: the NCCL all-reduce after each row-parallel linear and the residual
 * add that follows it (llama/model.py:276-277, 358-362 under tensor parallelism). */
int li4_allreduce_add(const void* const* slots, void* const* flags, void* counts, int ctas, int world, int rank,
                      int64_t n, const void* residual, void* out, void* stream);

/* w16[N, K] (fp16, row stride stride_wn elements) = dequantized weights,
 * bit-identical to the reference's fp32 (q - zero) * scale rounded to fp16.
 * Replaces: QuantizedLinear.dequantize_packed (llama/quantize.py:78-104) and
 * the bit-identical dequantize_packed_v2 (llama/quantize.py:107-126). */
int li4_dequantize(const void* packed, const void* scale, const void* zero, void* w16,
                   int64_t N, int64_t K, int64_t group_size,
                   int64_t stride_pn, int64_t stride_sn, int64_t stride_wn, void* stream);

/* Quantize w[N, K] (dtype li4_dtype, row stride stride_wn elements) to the
 * packed INT4 format: per-group min/max in fp32, scale = (max-min)/15 (0 -> 1),
 * zero = clamp(round(-min/scale), 0, 15), q = clamp(round(w/scale + zero), 0, 15),
 * round-half-to-even, IEEE fp32 division; scale and zero stored as fp16.
 * Bit-identical to the reference (packed bytes, scale and zero bits).
 * Outputs are contiguous: packed [N, K/2], scale/zero [N, K/group].
 * Replaces: QuantizedLinear.quantize_tensor (llama/quantize.py:44-75). */
int li4_quantize(const void* w, int w_dtype, void* packed, void* scale, void* zero,
                 int64_t N, int64_t K, int64_t group_size, int64_t stride_wn, void* stream);

/* ---------------------------------------------------------------------------
 * Decode program: a list of ops run by ONE persistent launch (one CTA per SM).
 *
 * Each CTA has a producer warp that streams the weight tiles of every linear op
 * of the program, in program order, into a ring of shared-memory stages with
 * bulk copies -- it never waits for activations, so the weights of the next ops
 * are already on chip while the current op waits for its inputs.  The consumer
 * warps run the ops in order; an op with wait = j first waits (bounded) until
 * every CTA has finished op j, and reads its inputs after that.  Ops without a
 * wait run as soon as their weights arrive.  An op reads and writes its buffers
 * only after its wait completes, so a write-after-read hazard needs a wait too.
 *
 * Replaces: the per-token sequence of launches of the reference's decode step
 * (Llama.forward at seqlen 1, llama/model.py:222-277, 310-315, 358-362, 440-455,
 * and the greedy argmax of llama/generation.py:59-60) by one launch; each op
 * computes what the per-launch entry points above compute (li4_int4_linear_fused,
 * li4_decode_attention, li4_argmax_rows).
 *
 * Build once (outside CUDA graph capture: finalize allocates device memory),
 * then launch any number of times (a launch is capturable).  Every pointer an
 * op was given is read at each launch; its contents may change between
 * launches.  Launches of one program must not overlap (one stream).
 * --------------------------------------------------------------------------- */
typedef struct li4_program li4_program;

#define LI4_NO_WAIT (-1)

int li4_program_create(li4_program** prog);
int li4_program_destroy(li4_program* prog);

/* An INT4 linear with an optional fusion (as li4_int4_linear_fused; fusion may be
 * NULL).  Program linears take group 128, N >= 16, K % 128 == 0 with
 * K <= 2048 or K % 2048 == 0, 16-byte aligned x rows and packed / scale / zero
 * rows (stride_pn % 16 == 0; stride_sn % 8 == 0 unless the rows are contiguous).
 * *op receives the op index. */
int li4_program_add_linear(li4_program* prog, const void* x, const void* packed, const void* scale,
                           const void* zero, void* y, int64_t M, int64_t N, int64_t K, int64_t group_size,
                           int64_t stride_xm, int64_t stride_pn, int64_t stride_sn, int64_t stride_ym,
                           const li4_fusion* fusion, int wait, int* op);

/* Decode attention as li4_decode_attention (n_heads / n_kv_heads in {1, 2, 4, 8},
 * head_dim 32, 64 or 128, (n_heads / n_kv_heads) * head_dim <= 512).  One CTA per
 * (sequence, KV head); max_seq is bounded by the CTA's shared memory
 * (LI4_ERR_UNSUPPORTED beyond it). */
int li4_program_add_attention(li4_program* prog, const void* q, int64_t stride_qb, const void* cache_k,
                              const void* cache_v, int64_t cache_stride_b, int64_t cache_stride_s, void* out,
                              int64_t stride_ob, int64_t batch, int64_t n_heads, int64_t n_kv_heads,
                              int64_t head_dim, const int64_t* pos, int64_t max_seq, int wait, int* op);

/* out[r, :] = table[ids[r], :] for r < rows (fp16 rows of `cols` values; an id
 * outside [0, table_rows) is clamped and sets bit 3 of li4_device_errors).
 * Replaces: the token embedding lookup (llama/model.py:440). */
int li4_program_add_gather(li4_program* prog, const void* table, int64_t table_rows, int64_t cols,
                           int64_t stride_t, const int64_t* ids, int64_t rows, void* out, int64_t stride_o,
                           int wait, int* op);

/* out[r * out_stride] = torch.argmax(logits[r, :cols]) for fp32 logits (first
 * index on ties, NaN above all), as li4_argmax_rows. */
int li4_program_add_argmax(li4_program* prog, const float* logits, int64_t rows, int64_t cols, int64_t stride,
                           int64_t* out, int64_t out_stride, int wait, int* op);

/* *value += 1 once every op of the launch has finished (the decode position). */
int li4_program_add_increment(li4_program* prog, int64_t* value);

/* Plan the launch on the current device, allocate the program's device state
 * (op table, completion counters, split-K scratch) and upload it. */
int li4_program_finalize(li4_program* prog);

/* Launch the whole program on `stream`. */
int li4_program_launch(li4_program* prog, void* stream);

/* Per-op timeline of the following launches (NULL turns it off): stamps[(op * ctas + cta) * 4 + i]
 * = %globaltimer (ns) when the CTA started op `op` (i = 0), its input wait ended (1), its x was
 * staged (2, linear ops) and its units were done (3); ops a CTA has no units of are not stamped.
 * capacity >= ops * ctas * 4 int64 values (after finalize). */
int li4_program_set_trace(li4_program* prog, int64_t* stamps, int64_t capacity);

/* CTAs, ring stages per CTA and dynamic shared memory of the launch (after finalize). */
int li4_program_info(const li4_program* prog, int* ctas, int* stages, size_t* smem_bytes);

#ifdef __cplusplus
}
#endif

#endif /* LLAMA_INT4_B200_H */
