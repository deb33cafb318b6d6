// t5_attention.cu — the T5 encoder's attention on the tensor cores with fp32-level accuracy.
//
// Replaces t5_attention (attention.cuh:34-91): scores = scale * Q K^T per head (the reference:
// cublasGemmStridedBatchedEx, CUBLAS_COMPUTE_32F under CUBLAS_DEFAULT_MATH, i.e. exact fp32),
// + relative position bias [H, L, L] + key mask [L], row softmax (softmax_with_mask,
// kernels.cu:1144-1201), then P V per head written as [L, H*D] (the reference's strided V
// layout).  T5 does not scale its logits, so they are large and a plain TF32 product would move
// the probabilities by percents.  The engine therefore splits each fp32 operand into two TF32
// parts, x = hi + lo (hi = tf32(x), lo = tf32(x - hi)), and runs one kind::tf32 GEMM over a
// K axis three times as long:
//     [Q_hi | Q_hi | Q_lo] . [K_hi | K_lo | K_hi]^T = Q_hi K_hi + Q_hi K_lo + Q_lo K_hi
// which drops only lo*lo (relative 2^-22): fp32-level scores from the tensor cores.  P . V
// (P in [0, 1]) runs as plain TF32 (relative error ~2^-11 per product, averaged over L keys).
//
//   1. t5_split_qk      Q, K [L, H, D] -> [H, L, 3D] TF32 parts in the two patterns above.
//   2. t5_vt            V [L, H*D] -> Vt [H, D, L] rounded to TF32 (K-major operand of P.V).
//   3. GEMM (kind::tf32, batch H)   S = scale * Qs Ks^T, F32 [H, L, L].
//   4. t5_softmax       S + rel_bias + mask -> softmax per row, P rounded to TF32, in place.
//   5. GEMM (kind::tf32, batch H)   out[:, h*D:(h+1)*D] = P_h Vt_h^T.
#include <cstdint>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

namespace {


// x [L, H, D] (row stride H*D) -> dst [H, L, 3D]: pattern 0 = [hi | hi | lo], 1 = [hi | lo | hi].
__global__ void t5_split_qk_kernel(const float* __restrict__ x, float* __restrict__ dst, int L, int H, int D,
                                   int pattern) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long n = static_cast<long long>(L) * H * D;
  if (i >= n) return;
  const int d = static_cast<int>(i % D);
  const long long lh = i / D;
  const int h = static_cast<int>(lh % H), l = static_cast<int>(lh / H);
  const float v = x[i];
  const float hi = round_tf32(v), lo = round_tf32(v - hi);
  float* o = dst + (static_cast<long long>(h) * L + l) * (3 * D);
  o[d] = hi;
  o[D + d] = pattern == 0 ? hi : lo;
  o[2 * D + d] = pattern == 0 ? lo : hi;
}

// V [L, H*D] -> Vt [H*D, L] rounded to TF32, through 32x33 shared-memory tiles.
__global__ void t5_vt_kernel(const float* __restrict__ v, float* __restrict__ vt, int L, int HD) {
  __shared__ float tile[32][33];
  const int l0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int l = l0 + r, c = c0 + threadIdx.x;
    tile[r][threadIdx.x] = (l < L && c < HD) ? v[static_cast<long long>(l) * HD + c] : 0.f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int c = c0 + r, l = l0 + threadIdx.x;
    if (c < HD && l < L) vt[static_cast<long long>(c) * L + l] = round_tf32(tile[threadIdx.x][r]);
  }
}

// One warp per row of S [H*L, L]: s + rel_bias + mask, softmax (max-subtracted, expf), P
// rounded to TF32 written back in place.  A row whose keys are all masked gives zeros.
__global__ void t5_softmax_kernel(float* __restrict__ S, const float* __restrict__ rel_bias,
                                  const float* __restrict__ mask, long long rows, int L) {
  const long long row = blockIdx.x * static_cast<long long>(blockDim.y) + threadIdx.y;
  if (row >= rows) return;
  float* s = S + row * L;
  const float* rb = rel_bias ? rel_bias + row * L : nullptr;
  const int lane = threadIdx.x;
  float m = -INFINITY;
  for (int c = lane * 4; c < L; c += 128) {
    float4 v = *reinterpret_cast<const float4*>(s + c);
    if (rb) {
      const float4 b = *reinterpret_cast<const float4*>(rb + c);
      v.x += b.x; v.y += b.y; v.z += b.z; v.w += b.w;
    }
    if (mask) {
      const float4 k = *reinterpret_cast<const float4*>(mask + c);
      v.x += k.x; v.y += k.y; v.z += k.z; v.w += k.w;
    }
    *reinterpret_cast<float4*>(s + c) = v;
    m = fmaxf(m, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float sum = 0.f;
  for (int c = lane * 4; c < L; c += 128) {
    float4 v = *reinterpret_cast<const float4*>(s + c);
    v.x = m == -INFINITY ? 0.f : expf(v.x - m);
    v.y = m == -INFINITY ? 0.f : expf(v.y - m);
    v.z = m == -INFINITY ? 0.f : expf(v.z - m);
    v.w = m == -INFINITY ? 0.f : expf(v.w - m);
    *reinterpret_cast<float4*>(s + c) = v;
    sum += (v.x + v.y) + (v.z + v.w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = sum > 0.f ? 1.f / sum : 0.f;
  for (int c = lane * 4; c < L; c += 128) {
    float4 v = *reinterpret_cast<const float4*>(s + c);
    *reinterpret_cast<float4*>(s + c) =
        make_float4(round_tf32(v.x * inv), round_tf32(v.y * inv), round_tf32(v.z * inv), round_tf32(v.w * inv));
  }
}

int64_t round_up_t5(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace

b2g_status t5_attention(const float* Q, const float* K, const float* V, const float* rel_bias, int n_head,
                        int d_head, int64_t L, float scale, const float* attn_mask, float* out, cudaStream_t st) {
  const int64_t H = n_head, D = d_head;
  if (L < 0 || H <= 0 || D <= 0) return set_error(B2G_ERR_INVALID, "t5_attention: sizes");
  if (L == 0) return B2G_OK;
  if (!Q || !K || !V || !out) return set_error(B2G_ERR_INVALID, "t5_attention: null operand");
  // 16-byte rows for the TF32 GEMM operands (3D and L floats) and the softmax's float4 access.
  if (L % 4 != 0 || D % 4 != 0 || L > (1ll << 30) || H * L > (1ll << 31))
    return set_error(B2G_ERR_UNSUPPORTED, "t5_attention: L and d_head must be multiples of 4");
  const uintptr_t bits = reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(rel_bias) |
                         reinterpret_cast<uintptr_t>(attn_mask);
  if (bits & 15u) return set_error(B2G_ERR_UNSUPPORTED, "t5_attention: 16-byte aligned out, rel_bias and mask");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const int64_t HD = H * D;
  const size_t qk_bytes = static_cast<size_t>(round_up_t5(H * L * 3 * D * 4, 256));
  const size_t s_bytes = static_cast<size_t>(round_up_t5(H * L * L * 4, 256));
  const size_t vt_bytes = static_cast<size_t>(round_up_t5(HD * L * 4, 256));
  void* ws = nullptr;
  if ((s = workspace_get(2 * qk_bytes + s_bytes + vt_bytes, &ws, kWsAttention)) != B2G_OK) return s;
  char* base = static_cast<char*>(ws);
  float* qs = reinterpret_cast<float*>(base);
  float* ks = reinterpret_cast<float*>(base + qk_bytes);
  float* S = reinterpret_cast<float*>(base + 2 * qk_bytes);
  float* vt = reinterpret_cast<float*>(base + 2 * qk_bytes + s_bytes);

  const long long n = L * HD;
  const unsigned nb = static_cast<unsigned>((n + 255) / 256);
  t5_split_qk_kernel<<<nb, 256, 0, st>>>(Q, qs, static_cast<int>(L), n_head, d_head, 0);
  t5_split_qk_kernel<<<nb, 256, 0, st>>>(K, ks, static_cast<int>(L), n_head, d_head, 1);
  t5_vt_kernel<<<dim3(static_cast<unsigned>((L + 31) / 32), static_cast<unsigned>((HD + 31) / 32)), dim3(32, 8), 0,
                 st>>>(V, vt, static_cast<int>(L), static_cast<int>(HD));
  note_launch(3);
  if ((s = check_cuda(cudaGetLastError(), "t5_attention operand kernels")) != B2G_OK) return s;

  // S[h] = scale * [Q_hi|Q_hi|Q_lo] . [K_hi|K_lo|K_hi]^T
  GemmProblem g;
  g.M = L; g.N = L; g.K = 3 * D; g.batch = H;
  g.a = qs; g.a_dtype = B2G_F32; g.lda = 3 * D; g.a_bstride = L * 3 * D;
  g.b = ks; g.b_dtype = B2G_F32; g.ldb = 3 * D; g.b_bstride = L * 3 * D;
  g.d = S; g.d_dtype = B2G_F32; g.ldd = L; g.d_bstride = L * L;
  g.allow_tf32 = true;
  g.alpha = scale;
  if (!tc_gemm_supported(g, nullptr)) return set_error(B2G_ERR_UNSUPPORTED, "t5_attention: scores GEMM");
  if ((s = tc_gemm_launch(g, st)) != B2G_OK) return s;

  const long long rows = H * L;
  t5_softmax_kernel<<<static_cast<unsigned>((rows + 7) / 8), dim3(32, 8), 0, st>>>(S, rel_bias, attn_mask, rows,
                                                                                 static_cast<int>(L));
  note_launch();
  if ((s = check_cuda(cudaGetLastError(), "t5_softmax launch")) != B2G_OK) return s;

  // out[:, h*D:(h+1)*D] = P_h . Vt_h^T
  GemmProblem o;
  o.M = L; o.N = D; o.K = L; o.batch = H;
  o.a = S; o.a_dtype = B2G_F32; o.lda = L; o.a_bstride = L * L;
  o.b = vt; o.b_dtype = B2G_F32; o.ldb = L; o.b_bstride = D * L;
  o.d = out; o.d_dtype = B2G_F32; o.ldd = HD; o.d_bstride = D;
  o.allow_tf32 = true;
  if (!tc_gemm_supported(o, nullptr)) return set_error(B2G_ERR_UNSUPPORTED, "t5_attention: output GEMM");
  return tc_gemm_launch(o, st);
}

}  // namespace b2g
