// gemm_simt.cu — CUDA-core GEMM for the cases the tensor-core path does not take, and the
// elementwise conversion kernels that feed it.
//
// The SIMT GEMM serves (F32 x F32) with exact fp32 products, as the reference's linear_lt
// does for CUDA_R_32F operands (cublas_ops.cuh:479-480, CUBLAS_COMPUTE_32F), and any
// operand whose stride or base alignment a TMA descriptor cannot express (e.g. the NeRF
// embedder's K=67 rows, chroma.cuh:1199).  It is a correctness path, not a fast path.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <type_traits>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

namespace {

constexpr int kTile = 64;
constexpr int kTileK = 16;

struct SimtParams {
  int M, N, K, batch;
  const void* a; int a_dtype; long long lda, a_bstride;
  const void* b; int b_dtype; long long ldb, b_bstride;
  const void* bias; int bias_kind;  // 0 none, 1 f32, 2 bf16
  void* d; int d_dtype; long long ldd, d_bstride;
  int epilogue;
  const float* gate;
  float alpha;
};

__device__ __forceinline__ float load_elem(const void* base, int dt, long long idx) {
  if (dt == B2G_F32) return static_cast<const float*>(base)[idx];
  if (dt == B2G_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
  return __half2float(static_cast<const __half*>(base)[idx]);
}

__device__ __forceinline__ float gelu_tanh(float v) {
  const float inner = 0.7978845608f * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner));
}

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// 64x64 output tile per 256-thread block, 4x4 outputs per thread, K staged 16 at a time.
__global__ void __launch_bounds__(256) simt_gemm_kernel(const SimtParams p) {
  __shared__ float As[kTileK][kTile + 4];
  __shared__ float Bs[kTileK][kTile + 4];
  const int bz = blockIdx.z;
  const int m0 = blockIdx.y * kTile, n0 = blockIdx.x * kTile;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const long long abase = static_cast<long long>(bz) * p.a_bstride;
  const long long bbase = static_cast<long long>(bz) * p.b_bstride;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < p.K; k0 += kTileK) {
    for (int i = threadIdx.x; i < kTile * kTileK; i += 256) {
      const int r = i / kTileK, kk = i % kTileK;
      const int gm = m0 + r, gn = n0 + r, gk = k0 + kk;
      As[kk][r] = (gm < p.M && gk < p.K) ? load_elem(p.a, p.a_dtype, abase + gm * p.lda + gk) : 0.f;
      Bs[kk][r] = (gn < p.N && gk < p.K) ? load_elem(p.b, p.b_dtype, bbase + gn * p.ldb + gk) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kTileK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  const long long dbase = static_cast<long long>(bz) * p.d_bstride;
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= p.M) continue;
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= p.N) continue;
      float v = p.alpha * acc[i][j];
      if (p.bias_kind == 1) v += static_cast<const float*>(p.bias)[n];
      else if (p.bias_kind == 2) v += __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[n]);
      const long long o = dbase + static_cast<long long>(m) * p.ldd + n;
      if (p.epilogue == B2G_EPI_GELU) v = gelu_tanh(v);
      if (p.epilogue == B2G_EPI_SILU) v = silu(v);
      if (p.epilogue == B2G_EPI_GATED_RESIDUAL) {
        float* dp = static_cast<float*>(p.d);
        dp[o] = dp[o] + p.gate[n] * v;
      } else if (p.d_dtype == B2G_F32) {
        static_cast<float*>(p.d)[o] = v;
      } else if (p.d_dtype == B2G_BF16) {
        static_cast<__nv_bfloat16*>(p.d)[o] = __float2bfloat16(v);
      } else {
        static_cast<__half*>(p.d)[o] = __float2half(v);
      }
    }
  }
}

// F32 -> bf16/fp16 copy with round-to-nearest-even, as f32_to_bf16_kernel /
// f32_to_fp16_kernel do (kernels.cu:40-60); here batched and strided on both sides.
template <typename T>
__global__ void cast_rows_kernel(const float* __restrict__ src, T* __restrict__ dst, long long batch, long long rows,
                                 long long cols, long long src_ld, long long src_bs, long long dst_ld,
                                 long long dst_bs) {
  const long long per = rows * cols, total = batch * per;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long b = i / per, rc = i - b * per;
    const long long r = rc / cols, c = rc - r * cols;
    const float v = src[b * src_bs + r * src_ld + c];
    if constexpr (std::is_same<T, __nv_bfloat16>::value) dst[b * dst_bs + r * dst_ld + c] = __float2bfloat16(v);
    else if constexpr (std::is_same<T, float>::value) dst[b * dst_bs + r * dst_ld + c] = round_tf32(v);
    else dst[b * dst_bs + r * dst_ld + c] = __float2half(v);
  }
}

// Dense fast path: 4 elements per thread with 16-byte loads.
template <typename T>
__global__ void cast_dense4_kernel(const float4* __restrict__ src, T* __restrict__ dst, long long n4) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 v = src[i];
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
      reinterpret_cast<__nv_bfloat162*>(dst)[2 * i] = lo;
      reinterpret_cast<__nv_bfloat162*>(dst)[2 * i + 1] = hi;
    } else if constexpr (std::is_same<T, float>::value) {
      reinterpret_cast<float4*>(dst)[i] = make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
    } else {
      __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
      reinterpret_cast<__half2*>(dst)[2 * i] = lo;
      reinterpret_cast<__half2*>(dst)[2 * i + 1] = hi;
    }
  }
}

}  // namespace

b2g_status simt_gemm_launch(const GemmProblem& p, cudaStream_t st) {
  if (p.M == 0 || p.N == 0) return B2G_OK;
  SimtParams s{};
  s.M = static_cast<int>(p.M);
  s.N = static_cast<int>(p.N);
  s.K = static_cast<int>(p.K);
  s.batch = static_cast<int>(p.batch);
  s.a = p.a; s.a_dtype = p.a_dtype; s.lda = p.lda; s.a_bstride = p.a_bstride;
  s.b = p.b; s.b_dtype = p.b_dtype; s.ldb = p.ldb; s.b_bstride = p.b_bstride;
  s.bias = p.bias; s.bias_kind = p.bias ? (p.bias_dtype == B2G_F32 ? 1 : 2) : 0;
  s.d = p.d; s.d_dtype = p.d_dtype; s.ldd = p.ldd; s.d_bstride = p.d_bstride;
  s.epilogue = p.epilogue;
  s.gate = p.gate;
  s.alpha = p.alpha;
  if (p.batch > 65535 || (p.M + kTile - 1) / kTile > 65535)
    return set_error(B2G_ERR_UNSUPPORTED, "SIMT GEMM: grid too large");
  dim3 grid(static_cast<unsigned>((p.N + kTile - 1) / kTile), static_cast<unsigned>((p.M + kTile - 1) / kTile),
            static_cast<unsigned>(p.batch));
  simt_gemm_kernel<<<grid, 256, 0, st>>>(s);
  note_launch();
  return check_cuda(cudaGetLastError(), "simt_gemm launch");
}

b2g_status cast_f32_to_16(const float* src, void* dst, b2g_dtype dst_dtype, int64_t batch, int64_t rows,
                          int64_t cols, int64_t src_ld, int64_t src_bs, int64_t dst_ld, int64_t dst_bs,
                          cudaStream_t st) {
  const long long total = batch * rows * cols;
  if (total == 0) return B2G_OK;
  const int threads = 256;
  const long long cap = 148LL * 16;
  const bool dense = (src_ld == cols) && (dst_ld == cols) && (batch == 1 || (src_bs == rows * cols && dst_bs == rows * cols)) &&
                     ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) &&
                     (total % 4 == 0);
  if (dense) {
    const long long n4 = total / 4;
    const int blocks = static_cast<int>((n4 + threads - 1) / threads < cap ? (n4 + threads - 1) / threads : cap);
    if (dst_dtype == B2G_BF16)
      cast_dense4_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(reinterpret_cast<const float4*>(src),
                                                                    static_cast<__nv_bfloat16*>(dst), n4);
    else if (dst_dtype == B2G_F32)
      cast_dense4_kernel<float><<<blocks, threads, 0, st>>>(reinterpret_cast<const float4*>(src),
                                                            static_cast<float*>(dst), n4);
    else
      cast_dense4_kernel<__half><<<blocks, threads, 0, st>>>(reinterpret_cast<const float4*>(src),
                                                             static_cast<__half*>(dst), n4);
  } else {
    const int blocks = static_cast<int>((total + threads - 1) / threads < cap ? (total + threads - 1) / threads : cap);
    if (dst_dtype == B2G_BF16)
      cast_rows_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(src, static_cast<__nv_bfloat16*>(dst), batch, rows,
                                                                  cols, src_ld, src_bs, dst_ld, dst_bs);
    else if (dst_dtype == B2G_F32)
      cast_rows_kernel<float><<<blocks, threads, 0, st>>>(src, static_cast<float*>(dst), batch, rows, cols, src_ld,
                                                          src_bs, dst_ld, dst_bs);
    else
      cast_rows_kernel<__half><<<blocks, threads, 0, st>>>(src, static_cast<__half*>(dst), batch, rows, cols, src_ld,
                                                           src_bs, dst_ld, dst_bs);
  }
  note_launch();
  return check_cuda(cudaGetLastError(), "cast kernel launch");
}

}  // namespace b2g
