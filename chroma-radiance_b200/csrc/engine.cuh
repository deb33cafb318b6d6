// engine.cuh — internal declarations shared by the engine's translation units.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <string>
#include <utility>
#include "../../include/b2g.h"

namespace b2g {

// Most problems one tensor-core launch computes together (tc_gemm_launch_group).
constexpr int kMaxGemmGroups = 4;

// Normalised problem handed from the C ABI to a kernel launcher.  All pointers are device
// pointers; strides are in elements.  A GEMM with batch > 1 uses the *_bstride fields.
struct GemmProblem {
  int64_t M = 0, N = 0, K = 0, batch = 1;
  const void* a = nullptr; b2g_dtype a_dtype = B2G_BF16; int64_t lda = 0, a_bstride = 0;
  const void* b = nullptr; b2g_dtype b_dtype = B2G_BF16; int64_t ldb = 0, b_bstride = 0;
  const void* bias = nullptr; b2g_dtype bias_dtype = B2G_F32;
  void* d = nullptr; b2g_dtype d_dtype = B2G_F32; int64_t ldd = 0, d_bstride = 0;
  b2g_epilogue epilogue = B2G_EPI_NONE;
  const float* gate = nullptr;
  bool allow_tf32 = false;  // F32 x F32 may run as TF32 products (batched_matmul_Bt only)
  bool round_tf32 = false;  // TF32 operands still plain fp32: the kernel rounds each shared-memory
                            // stage to nearest TF32 before the MMAs read it (1-CTA kernels)
  float alpha = 1.0f;       // D = epilogue(alpha * A.B^T + bias); internal (attention scores)
  bool allow_split = true;  // false: never split K (split-K needs workspace; b2g_gemm_noalloc)
  // E4M3 operands: D = (sum_k A.B) * a_scale[m] * b_scale[n] + bias, before the epilogue.
  const float* a_scale = nullptr;
  const float* b_scale = nullptr;
  // Tensor-parallel row-split layer (epilogue kEpiTpReduce): this rank's partial product is
  // summed with the other ranks' over NVLink inside the GEMM, see TpReduce.
  const struct TpReduce* tp = nullptr;
  int64_t tp_row0 = 0;      // first row of this problem in the partial / residual buffers
  // Attention input projection (epilogue kEpiQkvRope), see QkvRope.
  const struct QkvRope* rope = nullptr;
};

// Internal epilogue: D = [q | k | v] (N = 3 * heads * 128, bf16 out) with per-head RMSNorm
// (when scales are given) and RoPE applied to the q and k heads inside the GEMM.
constexpr int kEpiQkvRope = 17;
struct QkvRope {
  int64_t heads = 0;                // H; head_dim is 128
  float eps = 1e-6f;
  const float* pe = nullptr;        // RoPE table rows of this problem's first token [M][64][4]
  const float* q_norm = nullptr;    // RMSNorm scales [128] of the q heads (NULL: no norm)
  const float* k_norm = nullptr;    // and of the k heads
  void* gelu_out = nullptr;         // optional: columns past 3 * heads * 128 -> bias + GELU, bf16 here
  int64_t gelu_ld = 0;
  int64_t pe_period = 0;            // rows per sequence when one problem stacks several (0: M)
  bool pe_compact = false;          // pe rows [64][2] (cos, sin) instead of [64][4]
};

// Internal epilogue: bf16 partial -> all-rank sum (fixed rank order) -> residual += gate *
// (sum + bias), the residual updated in every rank's copy.  All buffers are peer-mapped.
constexpr int kEpiTpReduce = 16;
struct TpReduce {
  int world, rank;
  void* const* part_ptrs;   // device array [world]: each rank's bf16 partial buffer [rows, ld_part]
  float* const* res_ptrs;   // device array [world]: each rank's F32 residual copy [rows, ld_res]
  int64_t ld_part, ld_res;
  int* counters;            // rank 0's arrival counters (one per output tile slot), peer-mapped
  int64_t counter_slots;    // capacity of `counters`
};

// The checks of b2g_gemm on one descriptor (`who` names the entry point in error messages);
// fills *p, and sets *empty for an M == 0 or N == 0 problem (nothing to do).
b2g_status desc_to_problem(const b2g_gemm_desc* d, const char* who, GemmProblem* p, bool* empty);
// Forgets b2g_gemm_noalloc's cached per-device scratch addresses (b2g_shutdown).
void noalloc_forget();

// Records a message for b2g_last_error() and returns `st`.
b2g_status set_error(b2g_status st, const std::string& msg);
b2g_status check_cuda(cudaError_t e, const char* what);

// Per-device state resolved on first use of a device.
struct DeviceInfo {
  int device = -1;
  int num_sms = 0;
  int cc_major = 0, cc_minor = 0;
  int* err_word = nullptr;  // device address of the kernels' error word
};
b2g_status device_info(DeviceInfo** out);

// Counts launches of this library's kernels (reported by b2g_launch_count).
void note_launch(uint64_t n = 1);

// Programmatic dependent launch for the hot kernels (B2G_PDL=0 in the environment turns it
// off): a kernel launched this way may start while the previous kernel on the stream is
// still finishing, so it runs its set-up (barriers, TMEM, descriptor prefetch) early and then
// executes griddep_wait() in every CTA before it reads or writes any memory that an earlier
// kernel may still use.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
b2g_status launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, const char* what,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  b2g_status s = check_cuda(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), what);
  if (s == B2G_OK) note_launch();
  return s;
}

// Workspaces (device memory owned by the library, grown on demand, never shrunk), one per
// purpose so that one call can use several.  kWsCounters is zero-filled when (re)allocated
// and kernels leave it zero.
enum WorkspaceSlot { kWsOperands = 0, kWsSplitK = 1, kWsCounters = 2, kWsAttention = 3, kWsAttnSplit = 4, kWsSlots = 5 };
b2g_status workspace_get(size_t bytes, void** ptr, int slot = kWsOperands);
void workspace_release();

// True if the tensor-core path can run this problem (dtypes, strides, alignment).
// 3-D TMA map over a K-major bf16/fp16/fp32 operand: dims {K, rows, batch}, row stride ld,
// batch stride bstride (elements); box = 128 bytes of K x box_rows, 128-byte swizzle, zero
// fill outside the tensor.  (CUtensorMap from <cuda.h>.)
b2g_status make_operand_map(CUtensorMap* map, const void* base, b2g_dtype dt, int64_t K, int64_t rows, int64_t ld,
                            int64_t batch, int64_t bstride, uint32_t box_rows);

// Per-row E4M3 quantisation (fp8.cu): scales[r] = absmax_r / 448 (1 for a zero row),
// dst[r, c] = E4M3(src[r, c] * 448 / absmax_r), round to nearest even, saturating.
b2g_status quantize_rows_e4m3(const void* src, b2g_dtype src_dtype, int64_t rows, int64_t cols, int64_t ld,
                              uint8_t* dst, int64_t dst_ld, float* scales, cudaStream_t st);

// residual[m, n] += gate[n] * (y[m, n] + bias[n]) after a tensor-parallel all-reduce
// (elementwise.cu); y BF16 or F32, bias may be NULL.
b2g_status bias_gated_residual(const void* y, b2g_dtype y_dtype, int64_t ldy, const float* bias, const float* gate,
                               float* residual, int64_t ldr, int64_t M, int64_t N, cudaStream_t st);

// Cross-rank barrier over peer-mapped flag arrays (tp_comm.cu), bounded wait.
b2g_status tp_barrier(int* const* flag_ptrs, int* own_flags, int world, int rank, int epoch, int* epoch_ctr,
                      cudaStream_t st);
b2g_status tp_reduce_shard(const void* const* part_ptrs, void* sum, int64_t ld, int64_t rows, int64_t N, int world,
                           int rank, cudaStream_t st);
b2g_status tp_gather_residual(const void* const* sum_ptrs, int64_t ld, int64_t rows, int64_t N, int world,
                              const b2g_tp_residual_seg* segs, int nsegs, cudaStream_t st);
b2g_status tp_reduce_slots(const void* recv, void* sum, int64_t rows, int64_t N, int world, int rank,
                           cudaStream_t st);
b2g_status tp_push_rows(const void* part, void* const* recv_ptrs, int64_t rows, int64_t N, int world, int rank,
                        cudaStream_t st);
b2g_status tp_push_sums(void* const* sum_ptrs, int64_t rows, int64_t N, int world, int rank, cudaStream_t st);
b2g_status tp_scatter_rows(const void* part, void* const* recv_ptrs, int64_t rows, int64_t N, int world, int rank,
                           cudaStream_t st);
b2g_status tp_reduce_slots_bcast(const void* recv, void* const* sum_ptrs, int64_t rows, int64_t N, int world,
                                 int rank, cudaStream_t st);

// T5 attention (t5_attention.cu): Q, K, V [L, H, D] F32, rel_bias [H, L, L] or NULL, key mask
// [L] or NULL, out [L, H*D] F32.
b2g_status t5_attention(const float* Q, const float* K, const float* V, const float* rel_bias, int n_head,
                        int d_head, int64_t L, float scale, const float* attn_mask, float* out, cudaStream_t st);

bool tc_gemm_supported(const GemmProblem& p, std::string* why);
b2g_status tc_gemm_launch(const GemmProblem& p, cudaStream_t st);
// One launch over `count` (<= 2) problems that tc_gemm_groupable() accepts pairwise; their
// tiles share the persistent grid (fills the SMs where each problem alone would not).
bool tc_gemm_groupable(const GemmProblem& a, const GemmProblem& b);
b2g_status tc_gemm_launch_group(const GemmProblem* ps, int count, cudaStream_t st);
// Kernel variant override for tests/tuning: -1 automatic, 0 = 1-CTA 128x128 tiles,
// 1 = 1-CTA 128x256 tiles, 2 = 2-CTA 256x256 tiles.
void tc_gemm_set_variant(int force_variant, int allow_pair, int force_splits);
extern int g_attn_splits;  // fused attention key splits: 0 automatic, -1 never, > 0 forced

// Attention with RoPE (attention.cu).  q, k, v F32 rows of H*D (row strides ldq/ldk/ldv);
// q_norm/k_norm: optional per-head RMSNorm scales [D] (eps) fused into the Q/K producer;
// pe [L, D/2, 4]; key_bias [L] (0 / -inf) or null; out [L, H*D] F32 or BF16 (row stride ldo).
struct AttnArgs {
  const float *q = nullptr, *k = nullptr, *v = nullptr;
  int64_t ldq = 0, ldk = 0, ldv = 0;
  const float *q_norm = nullptr, *k_norm = nullptr;    // rows [0, norm_split)
  const float *q_norm2 = nullptr, *k_norm2 = nullptr;  // rows [norm_split, L) (null: same)
  int64_t norm_split = -1;                             // -1: one set of scales for all rows
  float eps = 1e-6f;
  const float* pe = nullptr;
  const float* key_bias = nullptr;
  void* out = nullptr;
  b2g_dtype out_dtype = B2G_F32;
  int64_t ldo = 0;
  int64_t L = 0, H = 0, D = 0;
};
b2g_status attention_rope_ex(const AttnArgs& a, cudaStream_t st);
// The fused attention kernel alone, on bf16 operands already normed and rotated: Q, K, V
// [L, ld] with head h at columns [h*D, (h+1)*D) (e.g. the three sections of one [L, 3*H*D]
// buffer written by the kEpiQkvRope GEMM epilogue).
struct AttnBf16Args {
  const __nv_bfloat16 *q = nullptr, *k = nullptr, *v = nullptr;
  int64_t ldq = 0, ldk = 0, ldv = 0;
  const float* key_bias = nullptr;  // [L] additive, NULL: none
  void* out = nullptr;
  b2g_dtype out_dtype = B2G_F32;
  int64_t ldo = 0;
  int64_t L = 0, H = 0, D = 0;
  int64_t batch = 1;        // sequences of L rows stored one after another, each attending within itself
  int64_t bias_stride = 0;  // floats between consecutive sequences' key biases (0: shared)
};
b2g_status attention_bf16(const AttnBf16Args& a, cudaStream_t st);

// out = LN(x) * (1 + scale) + shift per row of x [M, C] F32 (no-affine LayerNorm, two-pass
// statistics), written as bf16 or as per-row E4M3 with row_scale[M] (absmax / 448).  With
// period > 0, rows r with r % period >= split use (shift2, scale2) instead.
b2g_status modulate_rows(const float* x, const float* shift, const float* scale, void* out, b2g_dtype out_dtype,
                         float* row_scale, int64_t M, int64_t C, float eps, cudaStream_t st,
                         const float* shift2 = nullptr, const float* scale2 = nullptr, int64_t period = 0,
                         int64_t split = 0);
// Contiguous F32 [L, H*D] form of the above (no norm), the reference's attention_with_rope.
b2g_status attention_rope(const float* q, const float* k, const float* v, const float* pe, const float* key_bias,
                          float* out, int64_t L, int64_t H, int64_t D, cudaStream_t st);

// Exact-fp32 CUDA-core path for everything the tensor-core path does not take.
b2g_status simt_gemm_launch(const GemmProblem& p, cudaStream_t st);

// Elementwise F32 -> bf16/fp16 conversion of `batch` row blocks (strides in elements).
// dst_dtype B2G_F32 rounds to TF32 precision (round to nearest even, 10 mantissa bits)
// and keeps fp32 storage.
b2g_status cast_f32_to_16(const float* src, void* dst, b2g_dtype dst_dtype, int64_t batch, int64_t rows,
                          int64_t cols, int64_t src_ld, int64_t src_bs, int64_t dst_ld, int64_t dst_bs,
                          cudaStream_t st);

}  // namespace b2g
