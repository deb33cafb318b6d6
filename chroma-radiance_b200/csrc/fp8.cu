// fp8.cu — the FP8 E4M3 variant of the engine's linear layers.
//
// The reference has no FP8 path (its quantised path is INT8: quantize_act / linear_prequant in
// cublas_ops.cuh:294-791).  The north star's FP8 variant is: transformer weights stored as E4M3
// with one fp32 scale per output channel (absmax / 448), made once at load time, the transform
// that load_weight (chroma.cuh:97-134) applies when the weight arena is filled; activations
// quantised per token to E4M3 the same way; the GEMM runs tcgen05.mma kind::f8f6f4 with fp32
// accumulation and applies both scales in the epilogue before bias / GELU / gated residual.
//
//   quantize_rows_e4m3   per row r: s_r = absmax_r / 448 (1 for an all-zero row);
//                        q = E4M3(x * (448 / absmax_r)), round to nearest even, saturating
//                        at +-448.  One CTA per row; rows of up to 16384 values are read
//                        from memory once, into registers.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

namespace {

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_e4m3_kernel(const T* __restrict__ src, long long ld, int cols,
                                                                 uint8_t* __restrict__ dst, long long dst_ld,
                                                                 float* __restrict__ scales) {
  __shared__ float red[8];
  const long long row = blockIdx.x;
  const T* s = src + row * ld;
  float amax = 0.f;
  for (int c = threadIdx.x * 8; c < cols; c += blockDim.x * 8) {
    float v[8];
    load8<T>(s + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  const float inv = amax > 0.f ? 448.0f / amax : 1.0f;
  if (threadIdx.x == 0) scales[row] = amax > 0.f ? amax / 448.0f : 1.0f;
  uint8_t* d = dst + row * dst_ld;
  for (int c = threadIdx.x * 8; c < cols; c += blockDim.x * 8) {
    float v[8];
    load8<T>(s + c, v);
    uint32_t w[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const __nv_fp8x2_storage_t lo =
          __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i] * inv, v[4 * i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi =
          __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i + 2] * inv, v[4 * i + 3] * inv), __NV_SATFINITE, __NV_E4M3);
      w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    *reinterpret_cast<uint2*>(d + c) = make_uint2(w[0], w[1]);
  }
}

// The same quantisation with the row held in registers (NV groups of 8 values per thread,
// rows of up to 256 * 8 * NV values): one read of the row instead of two, and a programmatic
// dependent launch like the engine's other producers.
template <typename T, int NV>
__global__ void __launch_bounds__(256) quantize_rows_e4m3_reg_kernel(const T* __restrict__ src, long long ld,
                                                                     int cols, uint8_t* __restrict__ dst,
                                                                     long long dst_ld, float* __restrict__ scales) {
  __shared__ float red[8];
  griddep_wait();
  griddep_launch_dependents();
  const long long row = blockIdx.x;
  const T* s = src + row * ld;
  float v[NV][8];
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int c = (k * 256 + static_cast<int>(threadIdx.x)) * 8;
    if (c < cols) {
      load8<T>(s + c, v[k]);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[k][i]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  const float inv = amax > 0.f ? 448.0f / amax : 1.0f;
  if (threadIdx.x == 0) scales[row] = amax > 0.f ? amax / 448.0f : 1.0f;
  uint8_t* d = dst + row * dst_ld;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int c = (k * 256 + static_cast<int>(threadIdx.x)) * 8;
    if (c < cols) {
      uint32_t w[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
            make_float2(v[k][4 * i] * inv, v[k][4 * i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
            make_float2(v[k][4 * i + 2] * inv, v[k][4 * i + 3] * inv), __NV_SATFINITE, __NV_E4M3);
        w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
      }
      *reinterpret_cast<uint2*>(d + c) = make_uint2(w[0], w[1]);
    }
  }
}

template <typename T>
b2g_status launch_quantize(const T* src, int64_t rows, int64_t cols, int64_t ld, uint8_t* dst, int64_t dst_ld,
                           float* scales, cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>(rows)), block(256);
  const int c = static_cast<int>(cols);
  const int nv = static_cast<int>((cols + 2047) / 2048);
  if (nv <= 2) return launch_pdl(quantize_rows_e4m3_reg_kernel<T, 2>, grid, block, 0, st, "quantize_e4m3 launch", src,
                                 static_cast<long long>(ld), c, dst, static_cast<long long>(dst_ld), scales);
  if (nv <= 4) return launch_pdl(quantize_rows_e4m3_reg_kernel<T, 4>, grid, block, 0, st, "quantize_e4m3 launch", src,
                                 static_cast<long long>(ld), c, dst, static_cast<long long>(dst_ld), scales);
  if (nv <= 8) return launch_pdl(quantize_rows_e4m3_reg_kernel<T, 8>, grid, block, 0, st, "quantize_e4m3 launch", src,
                                 static_cast<long long>(ld), c, dst, static_cast<long long>(dst_ld), scales);
  quantize_rows_e4m3_kernel<T><<<grid, block, 0, st>>>(src, ld, c, dst, dst_ld, scales);
  note_launch();
  return check_cuda(cudaGetLastError(), "quantize_e4m3 launch");
}

}  // namespace

b2g_status quantize_rows_e4m3(const void* src, b2g_dtype src_dtype, int64_t rows, int64_t cols, int64_t ld,
                              uint8_t* dst, int64_t dst_ld, float* scales, cudaStream_t st) {
  if (rows < 0 || cols < 0) return set_error(B2G_ERR_INVALID, "quantize_e4m3: negative size");
  if (rows == 0 || cols == 0) return B2G_OK;
  if (!src || !dst || !scales) return set_error(B2G_ERR_INVALID, "quantize_e4m3: null pointer");
  if (ld < cols || dst_ld < cols) return set_error(B2G_ERR_INVALID, "quantize_e4m3: ld < cols");
  if (rows > 0x7fffffff) return set_error(B2G_ERR_UNSUPPORTED, "quantize_e4m3: too many rows");
  if (src_dtype != B2G_F32 && src_dtype != B2G_BF16 && src_dtype != B2G_F16)
    return set_error(B2G_ERR_UNSUPPORTED, "quantize_e4m3: source must be F32, BF16 or F16");
  const int64_t esz = src_dtype == B2G_F32 ? 4 : 2;
  // 8 elements per vector access: 16-byte source rows, 8-byte destination rows.
  if (cols % 8 != 0 || (ld * esz) % 16 != 0 || dst_ld % 8 != 0 || (reinterpret_cast<uintptr_t>(src) & 15u) ||
      (reinterpret_cast<uintptr_t>(dst) & 7u))
    return set_error(B2G_ERR_UNSUPPORTED, "quantize_e4m3: cols % 8, 16-byte source rows and 8-byte destination "
                                          "rows required");
  if (src_dtype == B2G_BF16)
    return launch_quantize(static_cast<const __nv_bfloat16*>(src), rows, cols, ld, dst, dst_ld, scales, st);
  if (src_dtype == B2G_F16) return launch_quantize(static_cast<const __half*>(src), rows, cols, ld, dst, dst_ld, scales, st);
  return launch_quantize(static_cast<const float*>(src), rows, cols, ld, dst, dst_ld, scales, st);
}

}  // namespace b2g
