// elementwise.cu — the one elementwise step the tensor-parallel path needs after its
// all-reduce: residual[m, n] += gate[n] * (y[m, n] + bias[n]).
//
// In the single-GPU path bias and gated residual are GEMM epilogues.  With row-split (K-split)
// layers each rank's GEMM produces a partial sum without bias; the partials are all-reduced
// and only then may bias and gate be applied, once.  This is the reference's gated_residual
// (kernels.cu:942-968, x + gate * y) with the linear's bias (added in linear_lt's cuBLASLt
// epilogue, cublas_ops.cuh:214-288) folded in.  y is bf16 (the all-reduced partials) or F32.
#include <cuda_bf16.h>
#include <cstdint>
#include "engine.cuh"

namespace b2g {

namespace {

template <bool BF16>
__global__ void __launch_bounds__(256) bias_gated_residual_kernel(const void* __restrict__ y, long long ldy,
                                                                  const float* __restrict__ bias,
                                                                  const float* __restrict__ gate,
                                                                  float* __restrict__ res, long long ldr, int M,
                                                                  int N) {
  const int groups = N / 8;  // 8 columns per thread
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<long long>(M) * groups) return;
  const int m = static_cast<int>(idx / groups), n = static_cast<int>(idx % groups) * 8;
  float v[8];
  if constexpr (BF16) {
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(y) + m * ldy + n);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(y) + m * ldy + n);
    const float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  float4* r = reinterpret_cast<float4*>(res + m * ldr + n);
  float4 r0 = r[0], r1 = r[1];
  float b[8], g[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    b[i] = bias ? __ldg(bias + n + i) : 0.f;
    g[i] = __ldg(gate + n + i);
  }
  r0.x += g[0] * (v[0] + b[0]); r0.y += g[1] * (v[1] + b[1]); r0.z += g[2] * (v[2] + b[2]); r0.w += g[3] * (v[3] + b[3]);
  r1.x += g[4] * (v[4] + b[4]); r1.y += g[5] * (v[5] + b[5]); r1.z += g[6] * (v[6] + b[6]); r1.w += g[7] * (v[7] + b[7]);
  r[0] = r0;
  r[1] = r1;
}

}  // namespace

b2g_status bias_gated_residual(const void* y, b2g_dtype y_dtype, int64_t ldy, const float* bias, const float* gate,
                               float* residual, int64_t ldr, int64_t M, int64_t N, cudaStream_t st) {
  if (M < 0 || N < 0) return set_error(B2G_ERR_INVALID, "bias_gated_residual: negative size");
  if (M == 0 || N == 0) return B2G_OK;
  if (!y || !gate || !residual) return set_error(B2G_ERR_INVALID, "bias_gated_residual: null pointer");
  if (y_dtype != B2G_BF16 && y_dtype != B2G_F32)
    return set_error(B2G_ERR_UNSUPPORTED, "bias_gated_residual: y must be BF16 or F32");
  if (ldy < N || ldr < N) return set_error(B2G_ERR_INVALID, "bias_gated_residual: ld < N");
  const int64_t esz = y_dtype == B2G_BF16 ? 2 : 4;
  if (N % 8 != 0 || (ldy * esz) % 16 != 0 || (ldr * 4) % 16 != 0 || (reinterpret_cast<uintptr_t>(y) & 15u) ||
      (reinterpret_cast<uintptr_t>(residual) & 15u))
    return set_error(B2G_ERR_UNSUPPORTED, "bias_gated_residual: N % 8 and 16-byte aligned rows required");
  if (M * (N / 8) > (1ll << 40)) return set_error(B2G_ERR_UNSUPPORTED, "bias_gated_residual: size");
  const long long threads = M * (N / 8);
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  if (y_dtype == B2G_BF16)
    bias_gated_residual_kernel<true><<<blocks, 256, 0, st>>>(y, ldy, bias, gate, residual, ldr, static_cast<int>(M),
                                                             static_cast<int>(N));
  else
    bias_gated_residual_kernel<false><<<blocks, 256, 0, st>>>(y, ldy, bias, gate, residual, ldr, static_cast<int>(M),
                                                              static_cast<int>(N));
  note_launch();
  return check_cuda(cudaGetLastError(), "bias_gated_residual launch");
}

}  // namespace b2g
