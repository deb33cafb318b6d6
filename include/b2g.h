/*
 * b2g.h — C ABI of the B200 GEMM engine for Chroma Radiance and its T5-XXL encoder.
 *
 * Every entry point takes plain device pointers, sizes and an optional CUDA stream
 * (passed as `void*`, NULL = legacy default stream 0, which is what every call in the
 * reference uses).  Nothing here allocates per call: a workspace for F32->bf16
 * activation casts is created on first need and reused (it only grows).
 *
 * Layout convention (row-major, the reference's convention):
 *     X  [M, K]  activations, row stride lda (elements)
 *     W  [N, K]  weights,     row stride ldb (elements)   -> D = X . W^T
 *     D  [M, N]  output,      row stride ldd (elements)
 *
 * Errors: every call returns a b2g_status; b2g_last_error() gives the message.  The
 * reference instead prints and calls exit(1) (cublas_ops.cuh:73-79, :496-499); the C++
 * drop-in header (chroma-radiance_b200/dropin/cublas_ops.cuh) maps a non-OK status back
 * to that behaviour.
 *
 * Thread safety: none, like the reference (single host thread, global state).
 */
#ifndef B2G_H
#define B2G_H

#include <stddef.h>
#include <stdint.h>
#include <library_types.h> /* cudaDataType_t: plain C enum from the CUDA toolkit */

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  B2G_OK = 0,
  B2G_ERR_INVALID = 1,       /* bad argument (null pointer, negative size, shape mismatch) */
  B2G_ERR_UNSUPPORTED = 2,   /* dtype combination or epilogue the engine does not implement */
  B2G_ERR_CUDA = 3,          /* a CUDA runtime/driver call failed */
  B2G_ERR_NO_DEVICE = 4,     /* no sm_100 device, or the library was built without it */
  B2G_ERR_DEVICE_TIMEOUT = 5 /* a kernel gave up waiting on a pipeline barrier (see below) */
} b2g_status;

typedef enum {
  B2G_F32 = 0,
  B2G_F16 = 1,
  B2G_BF16 = 2,
  B2G_E4M3 = 3
} b2g_dtype;

typedef enum {
  B2G_EPI_NONE = 0,           /* D = acc (+ bias)                                   */
  B2G_EPI_GELU = 1,           /* D = gelu_tanh(acc (+ bias))                        */
  B2G_EPI_GATED_RESIDUAL = 2, /* D[m,n] (F32, read-modify-write) += gate[n] * (acc (+ bias)) */
  B2G_EPI_SILU = 3            /* D = silu(acc (+ bias)) = v / (1 + e^-v): the approximator's
                                 in_layer -> silu_cuda (chroma.cuh:201-203, kernels.cu:346) */
} b2g_epilogue;

/* One GEMM with a fused epilogue.  a/b dtypes: (BF16,BF16), (F16,F16) run on the
 * tcgen05 tensor-core path; (F32,BF16) and (F32,F16) cast X first (as the reference's
 * linear() does, cublas_ops.cuh:484-495); (F32,F32) runs an exact-fp32 path.  */
typedef struct {
  int64_t M, N, K;
  const void* a; b2g_dtype a_dtype; int64_t lda;   /* X [M,K] */
  const void* b; b2g_dtype b_dtype; int64_t ldb;   /* W [N,K] */
  const void* bias; b2g_dtype bias_dtype;          /* [N] (F32 or BF16) or NULL */
  void* d; b2g_dtype d_dtype; int64_t ldd;         /* D [M,N]: F32, BF16 or F16 */
  b2g_epilogue epilogue;
  const float* gate;                               /* [N], B2G_EPI_GATED_RESIDUAL only */
} b2g_gemm_desc;

/* Library setup.  Replaces init_cublas() (cublas_ops.cuh:152-159): selects nothing,
 * queries the current device, checks it is sm_100, sets kernel attributes. Idempotent. */
b2g_status b2g_init(void);
/* Frees the cast workspace.  The reference never frees its handles; this is extra. */
b2g_status b2g_shutdown(void);
/* Message for the last non-OK status returned on this host thread's library state. */
const char* b2g_last_error(void);
/* Engine version string. */
const char* b2g_version(void);

/* General fused GEMM.  New entry point (no reference counterpart beyond linear_lt). */
b2g_status b2g_gemm(const b2g_gemm_desc* desc, void* stream);

/* `count` independent b2g_gemm problems in stream order.  When two to four of them share N,
 * K, dtypes, bias presence and epilogue (the txt and img streams of one double-block layer:
 * chroma.cuh:826-839 qkv, :888-892 proj, :923-927 / :958-962 MLP, each run by the reference
 * as a separate linear() per stream; with classifier-free guidance also each stream's
 * conditional and unconditional rows) they run as one persistent tensor-core launch whose
 * tiles fill the SMs together; otherwise one after the other.  Problems that read the same
 * F32 activations against 16-bit weights (the T5 layer's q, k, v: t5.cuh:233-275) share one
 * cast of them.  New entry point. */
b2g_status b2g_gemm_group(const b2g_gemm_desc* descs, int count, void* stream);

/* out[M,N] (F32) = x[M,K] . w[N,K]^T + bias[N] (F32, may be NULL).
 * Same arguments, meaning and dtype rules as the reference's
 *   static void linear_lt(int64_t M, int64_t K, int64_t N, const void* x_data,
 *       cudaDataType_t x_type, const void* w_data, cudaDataType_t w_type,
 *       const void* bias_data, void* out_data)          cublas_ops.cuh:214-288
 * x_type == w_type in {CUDA_R_16BF, CUDA_R_16F, CUDA_R_32F}; runs on stream 0. */
b2g_status b2g_linear_lt(int64_t M, int64_t K, int64_t N,
                         const void* x_data, cudaDataType_t x_type,
                         const void* w_data, cudaDataType_t w_type,
                         const void* bias_data, void* out_data);

/* Same as b2g_linear_lt on an explicit stream. */
b2g_status b2g_linear_lt_stream(int64_t M, int64_t K, int64_t N,
                                const void* x_data, cudaDataType_t x_type,
                                const void* w_data, cudaDataType_t w_type,
                                const void* bias_data, void* out_data, void* stream);

/* residual[M,N_out] (F32, in place) += gate[N_out] * (x[M,K] . w[N_out,K]^T + bias).
 * Replaces the BF16 branch of
 *   static void linear_gated_residual(const Tensor& x, const Tensor& W, const Tensor* bias,
 *       float* residual_inout, const float* gate, int64_t M, int64_t N_out)
 *                                                        cublas_ops.cuh:684-723
 * which runs linear() into a temporary and then gated_residual_cuda (kernels.cu:942-968);
 * here it is one kernel.  x dtype: F32 (cast to w's dtype first, as linear() does), BF16
 * or F16; w: BF16 or F16; bias: F32 or NULL.  Stream 0. */
b2g_status b2g_linear_gated_residual(const void* x, cudaDataType_t x_type,
                                     const void* w, cudaDataType_t w_type,
                                     const float* bias, float* residual_inout,
                                     const float* gate, int64_t M, int64_t K, int64_t N_out);

/* C[b] = A[b] . B[b]^T for b in [0,batch); A [batch,M,K], B [batch,N,K], C [batch,M,N],
 * all F32, densely packed.  Replaces
 *   static void batched_matmul_Bt(const Tensor& A, const Tensor& B, Tensor& C)
 *                                                        cublas_ops.cuh:558-585
 * The reference asks cuBLAS for CUBLAS_COMPUTE_32F_FAST_16BF, which on B200 runs as TF32
 * products of round-to-nearest TF32 operands with fp32 accumulation (checked against the
 * reference's own outputs); this engine does the same on kind::tf32 tensor cores.  Stream 0. */
b2g_status b2g_batched_matmul_Bt(const float* A, const float* B, float* C,
                                 int64_t batch, int64_t M, int64_t K, int64_t N);
/* The same on an explicit stream (the NeRF decoder's GLU products inside a captured step). */
b2g_status b2g_batched_matmul_Bt_stream(const float* A, const float* B, float* C, int64_t batch, int64_t M, int64_t K,
                                        int64_t N, void* stream);

/* out[L, n_head*d_head] (F32) = softmax(rope(Q) rope(K)^T / sqrt(d_head) + mask) V per head.
 * Q, K, V: F32 [L, n_head, d_head] (Q and K already RMS-normed), pe: F32 [L, d_head/2, 4]
 * (cos, -sin, sin, cos per rotation pair), attn_mask: F32 [L] key bias (0 or -inf) or NULL.
 * Replaces
 *   static Tensor attention_with_rope(const Tensor& Q, const Tensor& K, const Tensor& V,
 *       const Tensor& pe, int n_head, int d_head, const float* attn_mask)  attention.cuh:23-28
 * i.e. cudnn_attention_with_rope (cudnn_attention.cuh:449-476): RoPE + bf16 operands, fp32
 * softmax, bf16 probabilities.  Here a prologue kernel rotates Q and K and writes bf16 Q, K, V
 * into a library workspace (3*L*n_head*d_head*2 bytes), then one fused tcgen05 attention
 * kernel keeps scores and probabilities on chip (no [n_head, L, L] matrix).  d_head 64 or 128;
 * Q, K, V and pe 16-byte aligned. */
b2g_status b2g_attention_with_rope(const float* Q, const float* K, const float* V, const float* pe, int n_head,
                                   int d_head, int64_t L, const float* attn_mask, float* out, void* stream);

/* The fused form the engine's block path uses: Q, K, V are column ranges of one F32 qkv
 * buffer (row strides ldq/ldk/ldv, e.g. 3*n_head*d_head); q_norm/k_norm (F32 [d_head], may be
 * NULL) apply the per-head RMSNorm of qk_norm (chroma.cuh:513-515, rms_norm eps) inside the
 * RoPE producer, with q_norm2/k_norm2 for rows >= norm_split (the double block's img rows;
 * pass -1 for one set); the output is written as F32 or BF16 with row stride ldo, e.g.
 * straight into the bf16 [L, 3072 + 12288] concat buffer that feeds linear2.  New entry point. */
b2g_status b2g_attention_qknorm_rope(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                                     int64_t ldv, const float* q_norm, const float* k_norm, const float* q_norm2,
                                     const float* k_norm2, int64_t norm_split, float eps, const float* pe,
                                     const float* attn_mask, void* out, b2g_dtype out_dtype, int64_t ldo, int64_t L,
                                     int n_head, int d_head, void* stream);

/* b2g_gemm that allocates nothing (no reference counterpart).  For callers that cannot let a
 * library allocate device memory: engines that hand all of HBM to their own arena up front
 * (the reference's tensor.cuh pool does), and loops that cannot take the device-wide sync that
 * b2g_gemm's workspace growth (cudaMalloc, cudaFree) brings.  F32 activations with 16-bit
 * weights are cast into an 8 MiB array compiled into the library, so M*round_up(K,8)*2 must be
 * <= 8388608 bytes (else B2G_ERR_INVALID, nothing launched); K is never split.  Otherwise the
 * same arguments and rules as b2g_gemm, and the same results up to fp32 accumulation order
 * (b2g_gemm may split K).  The array is shared per device: calls whose kernels can overlap
 * race on it.  The first call on a device must come before any stream capture on it (it looks
 * up the array's device address); after a device reset, call b2g_shutdown first so the
 * address is looked up again.  Loading the library reserves the 8 MiB on every device it
 * runs on, whether or not this entry point is called. */
b2g_status b2g_gemm_noalloc(const b2g_gemm_desc* desc, void* stream);

/* T5 attention.  Same arguments and meaning as the reference's
 *   static Tensor t5_attention(const Tensor& Q, const Tensor& K, const Tensor& V,
 *       const float* rel_bias, int n_head, int d_head, float scale, const float* attn_mask)
 *                                                             attention.cuh:34-91
 * Q, K, V F32 [L, n_head, d_head]; rel_bias F32 [n_head, L, L] or NULL; attn_mask F32 [L]
 * (0 / -inf on keys) or NULL; out F32 [L, n_head*d_head].  softmax(scale Q K^T + rel_bias +
 * mask) V on the tensor cores: the scores with fp32-level accuracy from TF32 hi/lo operand
 * splits (the reference runs exact fp32 SGEMMs), P.V in TF32.  L and d_head multiples of 4. */
b2g_status b2g_t5_attention(const float* Q, const float* K, const float* V, const float* rel_bias, int n_head,
                            int d_head, int64_t L, float scale, const float* attn_mask, float* out, void* stream);

/* FP8 E4M3 quantisation of the rows of a matrix (no reference counterpart; the reference's
 * quantised path is INT8, quantize_act / linear_prequant in cublas_ops.cuh:294-791).  For each
 * row r of src [rows, cols] (F32, BF16 or F16, row stride ld): scales[r] = absmax_r / 448 (1
 * for an all-zero row) and dst[r, c] = E4M3(src[r, c] * 448 / absmax_r), round to nearest
 * even, saturating at +-448 (row stride dst_ld bytes).  Used once at load time on a weight
 * [N, K] (one scale per output channel: the FP8 variant of load_weight, chroma.cuh:97-134)
 * and per call on activations (one scale per token).  cols % 8 == 0, 16-byte source rows. */
b2g_status b2g_quantize_e4m3(const void* src, b2g_dtype src_dtype, int64_t rows, int64_t cols, int64_t ld,
                             uint8_t* dst, int64_t dst_ld, float* scales, void* stream);

/* FP8 linear (no reference counterpart): D = epilogue((A . W^T) * a_scale[m] * b_scale[n] +
 * bias) with W = desc->b an E4M3 [N, K] weight from b2g_quantize_e4m3 and b_scale its scales.
 * desc->a is either E4M3 with per-row scales a_scale, or BF16 / F16 / F32 activations, which
 * are quantised per token first (a_scale ignored).  Products exact, fp32 accumulation; the
 * same epilogues and output types as b2g_gemm.  K % 16 == 0 (16-byte rows). */
b2g_status b2g_gemm_fp8(const b2g_gemm_desc* desc, const float* a_scale, const float* b_scale, void* stream);

/* `count` (up to 4) b2g_gemm_fp8 problems on E4M3 activations (already quantised per row)
 * and E4M3 weights, a_scales[i] / b_scales[i] their scales.  Problems that share N, K, bias
 * presence, output dtype and epilogue run as one tensor-core launch (the FP8 form of
 * b2g_gemm_group: the txt and img streams of a double-block layer, and with guidance both
 * halves of each); otherwise one after the other.  No reference counterpart (the reference's
 * quantised linears are INT8, cublas_ops.cuh:294-791). */
b2g_status b2g_gemm_fp8_group(const b2g_gemm_desc* descs, const float* const* a_scales,
                              const float* const* b_scales, int count, void* stream);

/* residual[m, n] (F32, row stride ldr) += gate[n] * (y[m, n] + bias[n]) for the tensor-parallel
 * path: the reference's gated_residual (kernels.cu:942-968) with the linear's bias folded in,
 * applied once after the all-reduce of the row-split layer's partial sums (which carry no
 * bias).  y BF16 or F32 (row stride ldy); bias may be NULL.  N % 8 == 0, 16-byte rows,
 * 16-byte aligned bias and gate. */
b2g_status b2g_bias_gated_residual(const void* y, b2g_dtype y_dtype, int64_t ldy, const float* bias,
                                   const float* gate, float* residual, int64_t ldr, int64_t M, int64_t N,
                                   void* stream);

/* Tensor-parallel row-split layer with its all-reduce fused into the GEMM (no reference
 * counterpart; replaces GEMM -> ncclAllReduce -> gated_residual, kernels.cu:942-968, on the
 * path the north star adds to chroma.cuh for large images).  Every rank calls it with its
 * K-slice: descs[i] = {M, N, K of the slice, a = this rank's activations, b = this rank's weight
 * columns, bias = the full bias (F32, may be NULL), gate = the full gate}; d is ignored.  Each
 * output tile's bf16 partial goes to this rank's part_ptrs[rank]; the last rank to finish a
 * tile (arrival counted on rank 0's counters) sums all ranks' partials in rank order and
 * writes residual + gate * (sum + bias) into every rank's res_ptrs[q] rows row0[i].. .
 * part_ptrs / res_ptrs are device arrays of peer-mapped (NVLink) buffers; counters start at
 * zero and are never reset (arrivals are counted modulo world).  The caller runs a cross-rank
 * barrier after the call before anything reads a residual copy or reuses the partial buffer. */
typedef struct {
  int world, rank;
  void* const* part_ptrs;    /* device array [world] of bf16 [rows, ld_part] buffers */
  float* const* res_ptrs;    /* device array [world] of F32 [rows, ld_res] residual copies */
  int64_t ld_part, ld_res;
  int* counters;             /* rank 0's counter array (peer-mapped), counter_slots ints */
  int64_t counter_slots;
} b2g_tp_reduce_desc;
b2g_status b2g_gemm_tp_reduce(const b2g_gemm_desc* descs, const int64_t* row0, int count,
                              const b2g_tp_reduce_desc* tp, void* stream);

/* Cross-rank barrier for the fused tensor-parallel layers (no reference counterpart): rank
 * `rank` stores `epoch` into slot `rank` of every rank's flag array (flag_ptrs: device array
 * [world] of peer-mapped int[world] arrays, own_flags = this rank's) and waits until all slots
 * of its own array reach `epoch`.  Call with the same increasing epoch on every rank.  The wait
 * is bounded (2 s): on timeout the device error word gets bit 8 (b2g_check_device_error). */
b2g_status b2g_tp_barrier(int* const* flag_ptrs, int* own_flags, int world, int rank, int epoch, void* stream);
/* The same barrier with the epoch kept in device memory: epoch_counter (this rank's own int,
 * zero before the first call, not peer-mapped) holds the last epoch; the kernel waits on
 * *epoch_counter + 1 and stores it back.  Because the host passes no epoch, a CUDA graph that
 * captured the call replays with a fresh epoch each time (b2g_tp_barrier bakes its argument
 * into the graph).  Every rank makes the same sequence of calls; do not mix the two forms on
 * one flag array. */
b2g_status b2g_tp_barrier_next(int* const* flag_ptrs, int* own_flags, int* epoch_counter, int world, int rank,
                               void* stream);

/* Two-phase all-reduce of a row-split layer's bf16 partial over NVLink peer memory, with the
 * residual update folded in (no reference counterpart: it replaces the ncclAllReduce +
 * gated_residual (kernels.cu:942-968) of the tensor-parallel path).  Rows [0, rows) are split
 * into world shards of ceil(rows / world); rank q owns shard q.
 *   b2g_tp_reduce_shard: sums, in rank order, the world partials [rows, N] (part_ptrs: device
 *     array [world] of peer-mapped bf16 buffers, row stride ld) over this rank's shard, rounds
 *     to bf16 and stores it at the same rows of `sum` (this rank's peer-mapped buffer).
 *   b2g_tp_gather_residual: for every row m of each segment, residual[m - row0] += gate *
 *     (sums[owner(m)][m] + bias) (sum_ptrs: device array [world] of the ranks' sum buffers).
 * A cross-rank barrier (b2g_tp_barrier) must precede each call: the partials, then the sums,
 * must be complete on every rank.  world <= 8, N % 8 == 0, 16-byte aligned rows, gate, bias. */
typedef struct {
  int64_t row0, rows;        /* rows [row0, row0 + rows) of the sum buffers */
  const float* bias;         /* [N] or NULL */
  const float* gate;         /* [N] */
  float* residual;           /* F32 [rows, ldr], this rank's replicated residual */
  int64_t ldr;
} b2g_tp_residual_seg;
b2g_status b2g_tp_reduce_shard(const void* const* part_ptrs, void* sum, int64_t ld, int64_t rows, int64_t N,
                               int world, int rank, void* stream);
b2g_status b2g_tp_gather_residual(const void* const* sum_ptrs, int64_t ld, int64_t rows, int64_t N, int world,
                                  const b2g_tp_residual_seg* segs, int nsegs, void* stream);

/* The push form of the same all-reduce (no reference counterpart): every transfer over NVLink
 * is a copy-engine copy of whole rows (cudaMemcpyAsync on `stream`), none an SM load.  Rows
 * [0, rows) are split into world shards of ceil(rows / world) as above; peer addresses are
 * HOST arrays here.
 *   b2g_tp_push_rows: this rank's bf16 partial [rows, N] (local, row stride N) goes, shard by
 *     shard, into the owning rank's receive buffer, slot `rank` (recv_ptrs: host array [world] of
 *     peer-mapped bf16 [world][shard][N] buffers).
 *   b2g_tp_reduce_slots: sums the world slots of this rank's receive buffer (local reads) in rank
 *     order into its rows of `sum` [rows, N] (bf16).
 *   b2g_tp_push_sums: this rank's rows of the sums go into every other rank's sum buffer
 *     (sum_ptrs: host array [world]); each rank then applies b2g_bias_gated_residual from its
 *     own, now complete, sum buffer.
 * A b2g_tp_barrier goes before b2g_tp_reduce_slots and after b2g_tp_push_sums. */
b2g_status b2g_tp_push_rows(const void* part, void* const* recv_ptrs, int64_t rows, int64_t N, int world, int rank,
                            void* stream);
b2g_status b2g_tp_push_sums(void* const* sum_ptrs, int64_t rows, int64_t N, int world, int rank, void* stream);
b2g_status b2g_tp_reduce_slots(const void* recv, void* sum, int64_t rows, int64_t N, int world, int rank,
                               void* stream);

/* The store form of the same all-reduce (no reference counterpart): every transfer over NVLink
 * is an SM store of 16 bytes a thread, none a load and none a copy-engine copy.  Shards as above;
 * peer addresses are DEVICE arrays [world] here.
 *   b2g_tp_scatter_rows: row m of this rank's bf16 partial [rows, N] (local, row stride N) goes to
 *     its owner q = m / shard, slot `rank`, row m - q * shard of q's receive buffer (recv_ptrs:
 *     the ranks' peer-mapped bf16 [world][shard][N] buffers).
 *   b2g_tp_reduce_slots_bcast: sums this rank's receive slots in rank order (local reads), rounds
 *     to bf16 and stores each of its rows into every rank's sum buffer (sum_ptrs: the ranks'
 *     peer-mapped bf16 [rows, N] buffers, row stride N), its own included.
 * A b2g_tp_barrier goes after each; each rank then applies b2g_bias_gated_residual from its own
 * sum buffer.  world <= 8, N % 8 == 0, 16-byte aligned buffers. */
b2g_status b2g_tp_scatter_rows(const void* part, void* const* recv_ptrs, int64_t rows, int64_t N, int world,
                               int rank, void* stream);
b2g_status b2g_tp_reduce_slots_bcast(const void* recv, void* const* sum_ptrs, int64_t rows, int64_t N, int world,
                                     int rank, void* stream);

/* Attention input projection with qk_norm and RoPE fused into the GEMM epilogue.  The
 * reference runs these as three linears into F32 q, k, v, then qk_norm (rms_norm per head with
 * a learned scale) on q and k (chroma.cuh:822-842 double block, chroma.cuh:1108-1116 single
 * block), then RoPE + bf16 inside attention_with_rope (apply_rope_fused_bf16,
 * cudnn_attention.cuh:449-476).  descs[i]: bf16/fp16 x [M,K] . w[N,K]^T + bias (F32), or on
 * E4M3 x and w with rope[i].a_scale / b_scale (the FP8 variant: acc * a_scale[m] * b_scale[n]
 * before the bias), with
 * N = 3 * n_head * 128 ([q | k | v] weight rows, as the reference's fused qkv weight stores
 * them), epilogue B2G_EPI_NONE, bf16 output d [M, ldd] (16-byte aligned rows).  In the output
 * the q and k heads are RMSNorm'd with rope[i].q_norm / k_norm ([128] F32 each, NULL: no norm;
 * x * rsqrt(mean(x^2) + eps) * scale) and rotated by the pe table rows rope[i].pe (F32
 * [M][64][4], the rows of problem i's tokens in the attention sequence); v is the plain
 * product.  count 1 to 4 (the txt and img streams, and with classifier-free guidance their
 * conditional and unconditional rows: one launch).
 * GELU tail (the single block's linear1, whose weight rows are [q | k | v | mlp],
 * chroma.cuh:1109-1113): with gelu_out set (count 1), N may exceed 3 * n_head * 128; columns
 * past it get bias + tanh-GELU and are written bf16 to gelu_out [M, gelu_ld] (e.g. the
 * linear2 concat buffer at column 3072, chroma.cuh:1150-1153), d holding only the
 * 3 * n_head * 128 [q | k | v] columns (ldd >= that). */
typedef struct {
  const float* pe;       /* RoPE rows of this problem's first token, 16-byte aligned */
  const float* q_norm;   /* [128] or NULL */
  const float* k_norm;   /* [128] or NULL */
  void* gelu_out;        /* NULL, or the GELU tail's bf16 output (16-byte aligned rows) */
  int64_t gelu_ld;       /* its row stride in elements */
  int64_t pe_period;     /* 0, or P > 0: row m rotates by pe row m % P (several sequences of
                            P tokens stacked in one problem, e.g. the conditional and
                            unconditional halves of a guidance batch; pe then holds P rows) */
  const float* a_scale;  /* E4M3 operands only: per-row activation scales [M] */
  const float* b_scale;  /* E4M3 operands only: per-output-channel weight scales [N] */
  int64_t pe_compact;    /* 0: pe rows are the reference's [64][4] (c0, c1, c2, c3) per pair;
                            1: [64][2] (cos, sin) per pair for tables of the rotation form
                            (cos, -sin, sin, cos), which every RoPE table is: the same values
                            from half the table bytes */
} b2g_qkv_rope_desc;
b2g_status b2g_gemm_qkv_rope(const b2g_gemm_desc* descs, const b2g_qkv_rope_desc* rope, int count, int n_head,
                             float eps, void* stream);

/* The fused attention on bf16 operands that are already normed and rotated, e.g. the three
 * sections of a b2g_gemm_qkv_rope output: q = d, k = d + H*D, v = d + 2*H*D, all with row
 * stride ldd.  softmax(Q K^T / sqrt(d_head) + key_bias[key]) V per head (key_bias [L] F32 or
 * NULL), out [L, ldo] F32 or BF16 with head h at columns h*d_head.  Replaces the cuDNN SDPA
 * call of cudnn_attention_with_rope (cudnn_attention.cuh:408-443, 466-471), whose operands are
 * bf16 at that point.  Q/K/V bases 16-byte aligned, row strides multiples of 8 elements. */
b2g_status b2g_attention_bf16(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                              int64_t L, int n_head, int d_head, const float* key_bias, void* out,
                              b2g_dtype out_dtype, int64_t ldo, void* stream);

/* b2g_attention_bf16 over `batch` sequences of L rows stored one after another in q, k, v and
 * out (sequence b at rows [b*L, (b+1)*L), each attending only within itself), in one launch;
 * sequence b's key bias starts at key_bias + b * bias_stride (bias_stride 0: one bias for all).
 * The guidance halves of forward_cfg (chroma.cuh:1540-1563), which the reference runs as one
 * cuDNN SDPA call per half after gathering each half's [txt; img] rows (chroma.cuh:851-876,
 * 1118-1136), stored here half-major.  batch <= 65535, batch * L < 2^30. */
b2g_status b2g_attention_bf16_batched(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                      int64_t ldv, int64_t L, int64_t batch, int n_head, int d_head,
                                      const float* key_bias, int64_t bias_stride, void* out, b2g_dtype out_dtype,
                                      int64_t ldo, void* stream);

/* The block GEMMs' A-operand producer.  Same arguments and meaning as the reference's
 *   void modulate_to_bf16_cuda(const float* x, const float* shift, const float* scale,
 *                              __nv_bfloat16* out, int64_t M, int64_t C, float eps)
 *                                                       kernels.cu:592-599 (kernel :552-590)
 * called before every block GEMM group (chroma.cuh:824, 835, 920, ...): out[m, c] =
 * bf16((x[m, c] - mean_m) * rsqrt(var_m + eps) * (1 + scale[c]) + shift[c]), mean and variance
 * of row m over its C values (variance about the mean, two passes).  x, shift, scale 16-byte
 * aligned, out 8-byte aligned, C % 4 == 0 and C <= 4096 (else B2G_ERR_UNSUPPORTED). */
b2g_status b2g_modulate_to_bf16(const float* x, const float* shift, const float* scale, void* out, int64_t M,
                                int64_t C, float eps, void* stream);

/* The same modulated values quantised per row to E4M3 for b2g_gemm_fp8's activations (no
 * reference counterpart: the reference's quantised producers are INT8,
 * kernels.cu:1988-2125): row_scale[m] = absmax_m / 448 (1 for an all-zero row), out = E4M3 of
 * the fp32 modulated values times 448 / absmax_m, round to nearest even, saturating. */
b2g_status b2g_modulate_to_e4m3(const float* x, const float* shift, const float* scale, uint8_t* out,
                                float* row_scale, int64_t M, int64_t C, float eps, void* stream);

/* Both streams of a double block modulated in one launch.  The reference modulates each
 * stream with its own vectors (modulate_to_bf16_cuda on txt and on img, chroma.cuh:824, 835,
 * 920, 955; with guidance each stream holds both halves' rows).  Here x [M, C] is the F32 stream
 * in the half-major layout: whole sequences of `seq` rows, the first txt_rows of each being
 * text tokens (txt_shift / txt_scale) and the rest image tokens (img_shift / img_scale).  out
 * bf16 (out_dtype B2G_BF16, row_scale NULL) or per-row E4M3 (B2G_E4M3, row_scale [M]), each row
 * as b2g_modulate_to_bf16 / b2g_modulate_to_e4m3 writes it.  M % seq == 0. */
b2g_status b2g_modulate_streams(const float* x, const float* txt_shift, const float* txt_scale,
                                const float* img_shift, const float* img_scale, int64_t seq, int64_t txt_rows,
                                void* out, b2g_dtype out_dtype, float* row_scale, int64_t M, int64_t C, float eps,
                                void* stream);

/* ---- The rest of the denoising step (ChromaRadiance::forward_cfg, chroma.cuh:1499-1584) ----
 * The operand producers and element-wise steps around the embedder, approximator and NeRF
 * GEMMs; all stream-ordered on `stream`, no allocation. */

/* im2col of conv2d_img_in (chroma.cuh:1311-1327, patchify_kernel kernels.cu:975-1019) fused
 * with linear()'s F32 -> bf16 activation cast: x F32 [C, H, W] -> out bf16 [(H/p)(W/p), ldo],
 * column c*p*p + py*p + px of patch (ph, pw) = x[c, ph*p + py, pw*p + px].  p even, H and W
 * multiples of p, x 8-byte and out 4-byte aligned. */
b2g_status b2g_patchify_bf16(const float* x, int C, int H, int W, int p, void* out, int64_t ldo, void* stream);

/* The approximator's input of compute_modulation (chroma.cuh:467-505): rows i < rows of
 * [timestep_embedding(*timestep, 16) | timestep_embedding(guidance, 16) |
 *  timestep_embedding(i, 32)] with time factor 1000 and period 10000 (kernels.cu:608-631,
 * evaluated with the same fast-math functions), F32 [rows, 64].  The timestep is read from
 * device memory, so a captured step can be replayed at another timestep. */
b2g_status b2g_timestep_vec(const float* timestep, float guidance, float* out, int rows, void* stream);

/* rms_norm_cuda (kernels.cu:174-212): out[r, c] = x[r, c] * rsqrt(mean_c(x[r]^2) + eps) *
 * scale[c], rows of C values (row strides ldx / ldo), F32 or BF16 out (the bf16 form is the
 * approximator's norm followed by linear()'s cast).  C a multiple of 4, 16-byte aligned x and
 * scale; C <= 256 and a multiple of 64 takes one warp per row. */
b2g_status b2g_rms_norm(const float* x, int64_t ldx, const float* scale, void* out, b2g_dtype out_dtype, int64_t ldo,
                        int64_t rows, int64_t C, float eps, void* stream);

/* NeRF decoder input (nerf_decode steps 1-3, chroma.cuh:1170-1200): row patch*256 + pix =
 * [x[0..2] at the pixel | dct[pix, 0..63] | zeros], bf16 [P*256, ldo], ldo >= 67 and a
 * multiple of 8 (72 pads the embedder's K = 67 to 16-byte rows; its weight is padded with
 * zero columns to match, which changes no product).  x F32 [3, H, W], dct F32 [256, 64]. */
b2g_status b2g_nerf_input_bf16(const float* x, const float* dct, int H, int W, void* out, int64_t ldo, void* stream);

/* The per-patch weights of one NeRF GLU block from its param_generator output params [P, ldp]
 * (slice_transpose x3 + l2_norm x3, chroma.cuh:1264-1281): gate, value F32 [P, 256, 64] (the
 * [64, 256] slices 0 and 1 transposed, rows L2-normalised), fc2 F32 [P, 64, 256] (slice 2
 * [256, 64] transposed, rows L2-normalised), norms floored at 1e-12. */
b2g_status b2g_nerf_glu_weights(const float* params, int64_t ldp, int64_t patches, float* gate, float* value,
                                float* fc2, void* stream);

/* dst[r, c] = round-to-nearest bf16 / fp16 of src[r, c] (f32_to_bf16_cuda / f32_to_fp16_cuda,
 * kernels.cu:40-92, the activation cast inside linear()), rows x cols with row strides lds/ldd. */
b2g_status b2g_convert_f32(const float* src, int64_t lds, int64_t rows, int64_t cols, void* dst, b2g_dtype dst_dtype,
                           int64_t ldd, void* stream);

/* One whole NeRF GLU block (NerfGLUBlock::forward, chroma.cuh:1253-1306) for `patches` patches in
 * one persistent tcgen05 kernel: from each patch's param_generator output row params[p] (ldp >=
 * 49152 floats) the L2-normalised gate / value / fc2 weights, rms_norm of the state x[p]
 * [256, 64] (norm_scale [64], eps 1e-6), the three TF32 products with silu * mul between them,
 * and x[p] += the result, in place.  Replaces b2g_nerf_glu_weights + b2g_rms_norm + three
 * b2g_batched_matmul_Bt + b2g_silu_mul + b2g_add_inplace with no intermediate in HBM.  x
 * 16-byte aligned; each kernel wait is bounded (b2g_check_device_error). */
b2g_status b2g_nerf_glu_block(const float* params, int64_t ldp, const float* norm_scale, float* x, int64_t patches,
                              void* stream);

/* a = silu(a) * b (silu_mul_cuda) and x += y (add_cuda), F32, n % 4 == 0, 16-byte aligned. */
b2g_status b2g_silu_mul(float* a, const float* b, int64_t n, void* stream);
b2g_status b2g_add_inplace(float* x, const float* y, int64_t n, void* stream);

/* The NeRF final layer and the guidance blend (chroma.cuh:1225-1250, 1581): each half's decoder
 * state feat [P, 256, 64] is un-patchified, RMS-normed over its 64 channels at every pixel
 * (scale norm_scale, eps 1e-6) and convolved 3x3 (conv_w [3, 64, 3, 3], conv_b [3], zero
 * padding); out F32 [3, H, W] = uncond + cfg_scale * (cond - uncond), or the conditional
 * result alone when feat_uncond is NULL.  One kernel: the normed state never leaves shared
 * memory.  feat_cond, feat_uncond and norm_scale 16-byte aligned; H and W multiples of 16. */
b2g_status b2g_nerf_final(const float* feat_cond, const float* feat_uncond, const float* norm_scale,
                          const float* conv_w, const float* conv_b, float cfg_scale, int H, int W, float* out,
                          void* stream);

/* Reads and clears the device-side error word that the tensor-core kernels set when a
 * pipeline wait exceeds its time limit (they then drain and return instead of hanging).
 * Synchronises the device.  Returns B2G_OK or B2G_ERR_DEVICE_TIMEOUT; *code gets the
 * raw word (which role gave up), may be NULL. */
b2g_status b2g_check_device_error(int* code);

/* Number of this library's kernels launched since load (host-side counter). */
uint64_t b2g_launch_count(void);

/* Tensor-core kernel selection for tests and tuning (no reference counterpart):
 * variant -1 automatic (default), 0 = one CTA per 128x128 tile, 1 = one CTA per 128x256
 * tile, 2 = a 2-CTA cluster per 256x256 tile; splits 0 automatic, > 0 the split-K factor of
 * every tile, < 0 (-S) whole tiles for the full waves and the last, partial wave's tiles split
 * S ways (partials reduced in a fixed order by the last split).  Affects later calls. */
b2g_status b2g_set_gemm_variant(int variant, int splits);

/* Fused-attention key splits for tests and tuning (no reference counterpart): 0 automatic
 * (a launch that fills under half of the SMs, e.g. a tensor-parallel rank's few heads, splits
 * its key blocks into slices run by separate CTAs and merged by a second kernel), -1 never,
 * > 0 that many slices (at most one per 4 key blocks).  Sequences of over 64K keys always
 * split (a CTA covers at most 512 key blocks).  Affects later calls. */
b2g_status b2g_set_attention_splits(int splits);

#ifdef __cplusplus
}
#endif
#endif /* B2G_H */
