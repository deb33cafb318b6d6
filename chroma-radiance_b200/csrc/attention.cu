// attention.cu — the Chroma transformer's attention as two tensor-core batched GEMMs.
//
// Replaces cudnn_attention_with_rope (cudnn_attention.cuh:449-476): RoPE + bf16 on Q and K
// (apply_rope_fused_bf16, rope.cuh:180-221), V to bf16, softmax(Q K^T / sqrt(D) + key_bias) V
// (cuDNN SDPA, cudnn_attention.cuh:408-443), output F32 [L, H*D].
//
//   1. qknorm_rope_bf16  Q, K F32 rows [L, H*D] -> optional per-head RMSNorm (qk_norm) ->
//                        RoPE -> bf16 [L, H*D].  The layout is kept: the GEMMs below read
//                        head h through TMA batch strides (row stride H*D, batch stride D),
//                        so no permute pass.
//   2. v_to_bf16_t       V F32 [L, H*D] -> bf16 [H, D, L] (the PV GEMM's K-major B operand).
//   3. S = alpha Q K^T + key_bias     batched GEMM, batch = H, M = N = L, K = D, F32 out;
//                        the key mask (0 / -inf) is the GEMM's per-column bias.
//   4. softmax_rows      S -> P bf16 (rows normalised; masked keys get exactly 0).
//   5. O = P V           batched GEMM, batch = H, M = L, N = D, K = L, written straight into
//                        the F32 [L, H*D] output (row stride H*D, batch stride D).
#include <cuda_bf16.h>
#include <cstdint>
#include "engine.cuh"

namespace b2g {

namespace {

// Fused Q/K producer: per (token, head) row of D values, RMSNorm with a learned scale
// (rms_norm, kernels.cu:174-207, as qk_norm applies it, chroma.cuh:513-515), then RoPE,
// then bf16.  One warp per row; lane i handles rotation pairs i, i+32, ...
// Rows l >= norm_split use norm2 (the double block's txt and img streams have their own
// scales); pe row l holds D/2 groups of (cos, -sin, sin, cos), the table gen_pe builds
// (rope.cuh:84) and apply_rope_fused_bf16 applies (rope.cuh:180-221).
__global__ void qknorm_rope_bf16_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ norm1,
                                        const float* __restrict__ norm2, int norm_split, float eps,
                                        const float* __restrict__ pe, __nv_bfloat16* __restrict__ out, long long ldo,
                                        int L, int H, int D) {
  const long long row = blockIdx.x * static_cast<long long>(blockDim.y) + threadIdx.y;
  if (row >= static_cast<long long>(L) * H) return;
  const int l = static_cast<int>(row / H), h = static_cast<int>(row % H);
  const float* norm = l < norm_split ? norm1 : norm2;
  const float* xr = x + l * ldx + h * D;
  const int half = D / 2;
  float ss = 0.f;
  for (int j = threadIdx.x; j < half; j += 32) {
    const float2 v = *reinterpret_cast<const float2*>(xr + 2 * j);
    ss += v.x * v.x + v.y * v.y;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = norm ? rsqrtf(ss / static_cast<float>(D) + eps) : 1.f;
  for (int j = threadIdx.x; j < half; j += 32) {
    float2 v = *reinterpret_cast<const float2*>(xr + 2 * j);
    if (norm) {
      v.x = v.x * inv * norm[2 * j];
      v.y = v.y * inv * norm[2 * j + 1];
    }
    const float4 p = *reinterpret_cast<const float4*>(pe + (static_cast<long long>(l) * half + j) * 4);
    *reinterpret_cast<__nv_bfloat162*>(out + l * ldo + h * D + 2 * j) =
        __floats2bfloat162_rn(v.x * p.x + v.y * p.y, v.x * p.z + v.y * p.w);
  }
}

// V [L, H*D] F32 -> Vt [H, D, L] bf16 through 32x32 shared-memory tiles.
__global__ void v_to_bf16_t_kernel(const float* __restrict__ v, long long ldv, __nv_bfloat16* __restrict__ vt, int L,
                                   int HD) {
  __shared__ float tile[32][33];
  const int l0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int l = l0 + r, c = c0 + threadIdx.x;
    tile[r][threadIdx.x] = (l < L && c < HD) ? v[l * ldv + c] : 0.f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int c = c0 + r, l = l0 + threadIdx.x;
    if (c < HD && l < L) vt[static_cast<long long>(c) * L + l] = __float2bfloat16(tile[threadIdx.x][r]);
  }
}

// One warp per row: max, sum of exp(s - max), then P = exp(s - max) / sum as bf16.
// A row whose entries are all -inf gives zeros (cannot occur with image tokens present).
__global__ void softmax_rows_bf16_kernel(const float* __restrict__ S, __nv_bfloat16* __restrict__ P, long long rows,
                                         int cols) {
  const long long row = blockIdx.x * static_cast<long long>(blockDim.y) + threadIdx.y;
  if (row >= rows) return;
  const float* s = S + row * cols;
  const int lane = threadIdx.x;
  float m = -INFINITY, l = 0.f;
  for (int c = lane * 4; c < cols; c += 128) {
    const float4 v = *reinterpret_cast<const float4*>(s + c);
    const float vm = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
    const float nm = fmaxf(m, vm);
    if (nm != -INFINITY) {
      l = l * __expf(m - nm) + __expf(v.x - nm) + __expf(v.y - nm) + __expf(v.z - nm) + __expf(v.w - nm);
      m = nm;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float ol = __shfl_xor_sync(0xffffffffu, l, o);
    const float nm = fmaxf(m, om);
    if (nm != -INFINITY) {
      l = l * __expf(m - nm) + ol * __expf(om - nm);
      m = nm;
    }
  }
  const float inv = (l > 0.f) ? 1.f / l : 0.f;
  __nv_bfloat16* p = P + row * cols;
  for (int c = lane * 4; c < cols; c += 128) {
    const float4 v = *reinterpret_cast<const float4*>(s + c);
    const float a = m == -INFINITY ? 0.f : __expf(v.x - m) * inv;
    const float b = m == -INFINITY ? 0.f : __expf(v.y - m) * inv;
    const float cc = m == -INFINITY ? 0.f : __expf(v.z - m) * inv;
    const float d = m == -INFINITY ? 0.f : __expf(v.w - m) * inv;
    reinterpret_cast<__nv_bfloat162*>(p + c)[0] = __floats2bfloat162_rn(a, b);
    reinterpret_cast<__nv_bfloat162*>(p + c)[1] = __floats2bfloat162_rn(cc, d);
  }
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace

b2g_status attention_rope_ex(const AttnArgs& a, cudaStream_t st) {
  const int64_t L = a.L, H = a.H, D = a.D;
  if (L <= 0 || H <= 0) return B2G_OK;
  // 16-byte TMA row strides for the bf16 operands (P and Vt rows are L long).
  if (D % 8 != 0 || L % 8 != 0)
    return set_error(B2G_ERR_UNSUPPORTED, "attention: head dim and sequence length must be multiples of 8");
  if (a.out_dtype != B2G_F32 && a.out_dtype != B2G_BF16)
    return set_error(B2G_ERR_UNSUPPORTED, "attention: output must be F32 or BF16");
  const int64_t HD = H * D;
  const size_t qk_bytes = static_cast<size_t>(round_up(L * HD * 2, 256));
  const size_t vt_bytes = static_cast<size_t>(round_up(HD * L * 2, 256));
  const size_t s_bytes = static_cast<size_t>(round_up(H * L * L * 4, 256));
  const size_t p_bytes = static_cast<size_t>(round_up(H * L * L * 2, 256));
  void* ws = nullptr;
  b2g_status s = workspace_get(2 * qk_bytes + vt_bytes + s_bytes + p_bytes, &ws, kWsAttention);
  if (s != B2G_OK) return s;
  char* base = static_cast<char*>(ws);
  __nv_bfloat16* qb = reinterpret_cast<__nv_bfloat16*>(base);
  __nv_bfloat16* kb = reinterpret_cast<__nv_bfloat16*>(base + qk_bytes);
  __nv_bfloat16* vt = reinterpret_cast<__nv_bfloat16*>(base + 2 * qk_bytes);
  float* S = reinterpret_cast<float*>(base + 2 * qk_bytes + vt_bytes);
  __nv_bfloat16* P = reinterpret_cast<__nv_bfloat16*>(base + 2 * qk_bytes + vt_bytes + s_bytes);

  const dim3 nb(32, 8);
  const unsigned nrows = static_cast<unsigned>((L * H + 7) / 8);
  const int split = a.norm_split >= 0 && a.norm_split < L ? static_cast<int>(a.norm_split) : static_cast<int>(L);
  qknorm_rope_bf16_kernel<<<nrows, nb, 0, st>>>(a.q, a.ldq, a.q_norm, a.q_norm2 ? a.q_norm2 : a.q_norm, split, a.eps,
                                                a.pe, qb, HD, static_cast<int>(L), static_cast<int>(H),
                                                static_cast<int>(D));
  qknorm_rope_bf16_kernel<<<nrows, nb, 0, st>>>(a.k, a.ldk, a.k_norm, a.k_norm2 ? a.k_norm2 : a.k_norm, split, a.eps,
                                                a.pe, kb, HD, static_cast<int>(L), static_cast<int>(H),
                                                static_cast<int>(D));
  v_to_bf16_t_kernel<<<dim3(static_cast<unsigned>((L + 31) / 32), static_cast<unsigned>((HD + 31) / 32)), dim3(32, 8),
                       0, st>>>(a.v, a.ldv, vt, static_cast<int>(L), static_cast<int>(HD));
  note_launch(3);
  if ((s = check_cuda(cudaGetLastError(), "attention prologue kernels")) != B2G_OK) return s;

  // S[h] = (1/sqrt(D)) Q_h K_h^T + key_bias
  GemmProblem g;
  g.M = L; g.N = L; g.K = D; g.batch = H;
  g.a = qb; g.a_dtype = B2G_BF16; g.lda = HD; g.a_bstride = D;
  g.b = kb; g.b_dtype = B2G_BF16; g.ldb = HD; g.b_bstride = D;
  g.bias = a.key_bias; g.bias_dtype = B2G_F32;
  g.d = S; g.d_dtype = B2G_F32; g.ldd = L; g.d_bstride = L * L;
  g.alpha = 1.0f / sqrtf(static_cast<float>(D));
  if ((s = tc_gemm_launch(g, st)) != B2G_OK) return s;

  const long long rows = H * L;
  softmax_rows_bf16_kernel<<<static_cast<unsigned>((rows + 7) / 8), nb, 0, st>>>(S, P, rows, static_cast<int>(L));
  note_launch();
  if ((s = check_cuda(cudaGetLastError(), "softmax kernel")) != B2G_OK) return s;

  // O[:, h*D:(h+1)*D] = P_h V_h, written in the caller's layout and dtype
  GemmProblem o;
  o.M = L; o.N = D; o.K = L; o.batch = H;
  o.a = P; o.a_dtype = B2G_BF16; o.lda = L; o.a_bstride = L * L;
  o.b = vt; o.b_dtype = B2G_BF16; o.ldb = L; o.b_bstride = D * L;
  o.d = a.out; o.d_dtype = a.out_dtype; o.ldd = a.ldo; o.d_bstride = D;
  return tc_gemm_launch(o, st);
}

b2g_status attention_rope(const float* q, const float* k, const float* v, const float* pe, const float* key_bias,
                          float* out, int64_t L, int64_t H, int64_t D, cudaStream_t st) {
  AttnArgs a;
  a.q = q; a.k = k; a.v = v;
  a.ldq = a.ldk = a.ldv = H * D;
  a.pe = pe; a.key_bias = key_bias;
  a.out = out; a.out_dtype = B2G_F32; a.ldo = H * D;
  a.L = L; a.H = H; a.D = D;
  return attention_rope_ex(a, st);
}

}  // namespace b2g
