// elementwise.cu — the one elementwise step the tensor-parallel path needs after its
// all-reduce: residual[m, n] += gate[n] * (y[m, n] + bias[n]).
//
// In the single-GPU path bias and gated residual are GEMM epilogues.  With row-split (K-split)
// layers each rank's GEMM produces a partial sum without bias; the partials are all-reduced
// and only then may bias and gate be applied, once.  This is the reference's gated_residual
// (kernels.cu:942-968, x + gate * y) with the linear's bias (added in linear_lt's cuBLASLt
// epilogue, cublas_ops.cuh:214-288) folded in.  y is bf16 (the all-reduced partials) or F32.
//
// Also the A-operand producer of the block GEMMs, modulate_to_bf16 (kernels.cu:552-599):
// out = bf16(LN(x) * (1 + scale[c]) + shift[c]), LayerNorm without affine, eps 1e-6, its mean
// and variance in two passes as the reference takes them; and the same values quantised per
// token to E4M3 for the FP8 linears (scale absmax/448, the quantize_rows_e4m3 recipe of fp8.cu).
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

namespace {

// res[m][n] += gate[n] * (y[m][n] + bias[n]).  A thread owns 8 columns (one 16-byte bf16 or
// two float4 loads of y, two float4 of the residual) of kBgrRows consecutive rows: the bias and
// gate are loaded once (as float4s) for all of them, and every row's loads are issued before
// any is used.
constexpr int kBgrRows = 4;

template <bool BF16>
__global__ void __launch_bounds__(256) bias_gated_residual_kernel(const void* __restrict__ y, long long ldy,
                                                                  const float* __restrict__ bias,
                                                                  const float* __restrict__ gate,
                                                                  float* __restrict__ res, long long ldr, int M,
                                                                  int N) {
  const int groups = N / 8;  // 8 columns per thread
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long row_groups = (M + kBgrRows - 1) / kBgrRows;
  if (idx >= row_groups * groups) return;
  const int m0 = static_cast<int>(idx / groups) * kBgrRows, n = static_cast<int>(idx % groups) * 8;
  float b[8], g[8];
  {
    const float4 g0 = __ldg(reinterpret_cast<const float4*>(gate + n)), g1 = __ldg(reinterpret_cast<const float4*>(gate + n) + 1);
    g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w; g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
    float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
    if (bias) {
      b0 = __ldg(reinterpret_cast<const float4*>(bias + n));
      b1 = __ldg(reinterpret_cast<const float4*>(bias + n) + 1);
    }
    b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
  }
  float v[kBgrRows][8];
  float4 r[kBgrRows][2];
#pragma unroll
  for (int k = 0; k < kBgrRows; ++k) {
    const int m = m0 + k;
    if (m >= M) break;
    if constexpr (BF16) {
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(y) + m * ldy + n));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[k][2 * i] = f.x;
        v[k][2 * i + 1] = f.y;
      }
    } else {
      const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(y) + m * ldy + n);
      const float4 a = __ldcs(p), c = __ldcs(p + 1);
      v[k][0] = a.x; v[k][1] = a.y; v[k][2] = a.z; v[k][3] = a.w;
      v[k][4] = c.x; v[k][5] = c.y; v[k][6] = c.z; v[k][7] = c.w;
    }
    const float4* rp = reinterpret_cast<const float4*>(res + m * ldr + n);
    r[k][0] = rp[0];
    r[k][1] = rp[1];
  }
#pragma unroll
  for (int k = 0; k < kBgrRows; ++k) {
    const int m = m0 + k;
    if (m >= M) break;
    float4 r0 = r[k][0], r1 = r[k][1];
    r0.x += g[0] * (v[k][0] + b[0]); r0.y += g[1] * (v[k][1] + b[1]);
    r0.z += g[2] * (v[k][2] + b[2]); r0.w += g[3] * (v[k][3] + b[3]);
    r1.x += g[4] * (v[k][4] + b[4]); r1.y += g[5] * (v[k][5] + b[5]);
    r1.z += g[6] * (v[k][6] + b[6]); r1.w += g[7] * (v[k][7] + b[7]);
    float4* rp = reinterpret_cast<float4*>(res + m * ldr + n);
    rp[0] = r0;
    rp[1] = r1;
  }
}

// One 128-thread block per row of x [M, C] (16-byte aligned rows, C % 4 == 0,
// C <= 128 * 4 * NV): the row is read from memory once into registers (NV float4 per thread),
// then mean, variance about the mean and the modulated output; the block sums go through
// four warp shuffles and a 4-entry shared array.  OUT 0: bf16; 1: E4M3 with a per-row scale.
// With period > 0, rows whose index modulo `period` is >= `split` take (shift2, scale2): the
// img rows of a half-major [txt | img] stream (period = T + I, split = T), so one launch
// modulates both streams of a double block for every guidance half.
constexpr int kModThreads = 128;

__device__ __forceinline__ float block_sum4(float v, float* red, int warp, int lane) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const float t = (red[0] + red[1]) + (red[2] + red[3]);
  __syncthreads();  // red is reused by the next reduction
  return t;
}

template <int NV, int OUT>
__global__ void __launch_bounds__(kModThreads) modulate_rows_kernel(const float* __restrict__ x,
                                                                    const float* __restrict__ shift,
                                                                    const float* __restrict__ scale,
                                                                    const float* __restrict__ shift2,
                                                                    const float* __restrict__ scale2, int period,
                                                                    int split, void* __restrict__ out,
                                                                    float* __restrict__ row_scale, int M, int C,
                                                                    float eps) {
  __shared__ float red[4];
  griddep_wait();
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = blockIdx.x;
  if (period > 0 && static_cast<int>(row % period) >= split) {
    shift = shift2;
    scale = scale2;
  }
  const float4* xr = reinterpret_cast<const float4*>(x + row * C);
  const int nv4 = C >> 2;
  float4 v[NV];
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = k * kModThreads + threadIdx.x;
    v[k] = i < nv4 ? __ldcs(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);  // streamed: read once
    sum += (v[k].x + v[k].y) + (v[k].z + v[k].w);
  }
  const float mean = block_sum4(sum, red, warp, lane) / static_cast<float>(C);
  float var = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (k * kModThreads + static_cast<int>(threadIdx.x) < nv4) {
      const float a = v[k].x - mean, b = v[k].y - mean, c = v[k].z - mean, d = v[k].w - mean;
      var += (a * a + b * b) + (c * c + d * d);
    }
  }
  const float inv_std = rsqrtf(block_sum4(var, red, warp, lane) / static_cast<float>(C) + eps);
  const float4* sc = reinterpret_cast<const float4*>(scale);
  const float4* sh = reinterpret_cast<const float4*>(shift);
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = k * kModThreads + threadIdx.x;
    if (i < nv4) {
      const float4 a = __ldg(sc + i), b = __ldg(sh + i);
      v[k].x = (v[k].x - mean) * inv_std * (1.0f + a.x) + b.x;
      v[k].y = (v[k].y - mean) * inv_std * (1.0f + a.y) + b.y;
      v[k].z = (v[k].z - mean) * inv_std * (1.0f + a.z) + b.z;
      v[k].w = (v[k].w - mean) * inv_std * (1.0f + a.w) + b.w;
      if constexpr (OUT == 0) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(v[k].x, v[k].y), hi = __floats2bfloat162_rn(v[k].z, v[k].w);
        reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + row * C)[i] =
            make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
      } else {
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
      }
    }
  }
  if constexpr (OUT == 1) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[warp] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float inv = amax > 0.f ? 448.0f / amax : 1.0f;
    if (threadIdx.x == 0) row_scale[row] = amax > 0.f ? amax / 448.0f : 1.0f;
    uint32_t* orow = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(out) + row * C);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = k * kModThreads + threadIdx.x;
      if (i < nv4) {
        const __nv_fp8x2_storage_t lo =
            __nv_cvt_float2_to_fp8x2(make_float2(v[k].x * inv, v[k].y * inv), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t hi =
            __nv_cvt_float2_to_fp8x2(make_float2(v[k].z * inv, v[k].w * inv), __NV_SATFINITE, __NV_E4M3);
        orow[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
      }
    }
  }
}

template <int OUT>
b2g_status launch_modulate(const float* x, const float* shift, const float* scale, const float* shift2,
                           const float* scale2, int period, int split, void* out, float* row_scale, int64_t M,
                           int64_t C, float eps, cudaStream_t st) {
  const unsigned grid = static_cast<unsigned>(M);
  const int nv = static_cast<int>((C / 4 + kModThreads - 1) / kModThreads);
  const int m = static_cast<int>(M), c = static_cast<int>(C);
  auto kern = nv <= 2 ? modulate_rows_kernel<2, OUT>
              : nv <= 4 ? modulate_rows_kernel<4, OUT>
              : nv <= 6 ? modulate_rows_kernel<6, OUT> : modulate_rows_kernel<8, OUT>;
  return launch_pdl(kern, dim3(grid), dim3(kModThreads), 0, st, "modulate launch", x, shift, scale, shift2, scale2,
                    period, split, out, row_scale, m, c, eps);
}

}  // namespace

b2g_status modulate_rows(const float* x, const float* shift, const float* scale, void* out, b2g_dtype out_dtype,
                         float* row_scale, int64_t M, int64_t C, float eps, cudaStream_t st, const float* shift2,
                         const float* scale2, int64_t period, int64_t split) {
  if (M < 0 || C < 0) return set_error(B2G_ERR_INVALID, "modulate: negative size");
  if (M == 0 || C == 0) return B2G_OK;
  if (!x || !shift || !scale || !out) return set_error(B2G_ERR_INVALID, "modulate: null pointer");
  if (period < 0 || period > (1ll << 30) || (period > 0 && (split < 0 || split > period || !shift2 || !scale2)))
    return set_error(B2G_ERR_INVALID, "modulate: second parameter set needs 0 <= split <= period and its vectors");
  if (period == 0) shift2 = shift, scale2 = scale;
  if (out_dtype != B2G_BF16 && out_dtype != B2G_E4M3) return set_error(B2G_ERR_UNSUPPORTED, "modulate: bf16 or E4M3 out");
  if (out_dtype == B2G_E4M3 && !row_scale) return set_error(B2G_ERR_INVALID, "modulate: E4M3 needs row scales");
  if (C % 4 != 0 || C > 4096 || M > (1ll << 31) - 1)
    return set_error(B2G_ERR_UNSUPPORTED, "modulate: C must be a multiple of 4 and at most 4096");
  const uintptr_t bits = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(shift) |
                         reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(shift2) |
                         reinterpret_cast<uintptr_t>(scale2);
  const uintptr_t obits = reinterpret_cast<uintptr_t>(out);
  if ((bits & 15u) || (obits & (out_dtype == B2G_BF16 ? 7u : 3u)))
    return set_error(B2G_ERR_UNSUPPORTED, "modulate: x, shift, scale 16-byte and out 8/4-byte aligned");
  const int per = static_cast<int>(period), spl = static_cast<int>(split);
  if (out_dtype == B2G_BF16)
    return launch_modulate<0>(x, shift, scale, shift2, scale2, per, spl, out, nullptr, M, C, eps, st);
  return launch_modulate<1>(x, shift, scale, shift2, scale2, per, spl, out, row_scale, M, C, eps, st);
}

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
  if ((reinterpret_cast<uintptr_t>(gate) & 15u) || (bias && (reinterpret_cast<uintptr_t>(bias) & 15u)))
    return set_error(B2G_ERR_UNSUPPORTED, "bias_gated_residual: bias and gate must be 16-byte aligned");
  const long long threads = (M + kBgrRows - 1) / kBgrRows * (N / 8);
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
