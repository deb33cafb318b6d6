// cublas_ops.cuh — drop-in replacement for the reference's GEMM layer header.
//
// Integration: in the reference tree, rename its original
// cublas_ops.cuh to cublas_ops_cublaslt.cuh, put this file in its place, add the engine's
// include/ directory to the include path and link libb2g.so.  chroma.cuh, t5.cuh,
// attention.cuh and main.cu then compile unchanged: every function, global and macro the
// original header provided still exists under the same name and signature.
//
// Routing:
//   linear / linear_lt / linear_gated_residual / batched_matmul_Bt  -> libb2g.so
//     (BF16, FP16 and F32 operands: the whole non-quantised model path)
//   INT8 weights, calibration mode, and every INT8 helper (quantize_act*, linear_prequant*,
//     linear_int8_gemm, ...)  -> the original cuBLASLt code, renamed below (out of scope for
//     the engine)
//   g_cublas / g_cublaslt / CHECK_CUBLAS stay defined: attention.cuh (T5 attention) uses them.
// Errors keep the reference's behaviour: print and exit(1).
#pragma once
#include "tensor.cuh"
#include "b2g.h"

// The original header, with its four GEMM entry points and init renamed so that the
// b2g-backed versions below can take their names.  Its internal calls (e.g. the INT8
// per-group path calling linear_lt) are renamed consistently and stay on cuBLASLt.
#define linear ref_cublaslt_linear
#define linear_lt ref_cublaslt_linear_lt
#define linear_gated_residual ref_cublaslt_linear_gated_residual
#define batched_matmul_Bt ref_cublaslt_batched_matmul_Bt
#define init_cublas ref_cublaslt_init_cublas
#include "cublas_ops_cublaslt.cuh"
#undef linear
#undef linear_lt
#undef linear_gated_residual
#undef batched_matmul_Bt
#undef init_cublas

#define B2G_CHECK(call)                                                                         \
  do {                                                                                          \
    b2g_status b2g_st_ = (call);                                                                \
    if (b2g_st_ != B2G_OK) {                                                                    \
      fprintf(stderr, "b2g error at %s:%d: %d (%s)\n", __FILE__, __LINE__, (int)b2g_st_,         \
              b2g_last_error());                                                                \
      exit(1);                                                                                  \
    }                                                                                           \
  } while (0)

static inline b2g_dtype b2g_dtype_of(DType t) {
  switch (t) {
    case DType::F32: return B2G_F32;
    case DType::FP16: return B2G_F16;
    case DType::BF16: return B2G_BF16;
    default: return B2G_E4M3;  // not reachable for the routed dtypes
  }
}
static inline cudaDataType_t b2g_cuda_type_of(DType t) {
  return t == DType::F32 ? CUDA_R_32F : (t == DType::FP16 ? CUDA_R_16F : CUDA_R_16BF);
}

// init_cublas (cublas_ops.cuh:152): the cuBLAS handles stay (INT8 path, T5 attention); the
// engine checks the device.
static void init_cublas() {
  ref_cublaslt_init_cublas();
  B2G_CHECK(b2g_init());
}

// linear_lt (cublas_ops.cuh:214): same arguments; F32 output; F32 bias or null; stream 0.
static void linear_lt(int64_t M, int64_t K, int64_t N, const void* x_data, cudaDataType_t x_type,
                      const void* w_data, cudaDataType_t w_type, const void* bias_data, void* out_data) {
  B2G_CHECK(b2g_linear_lt(M, K, N, x_data, x_type, w_data, w_type, bias_data, out_data));
}

// linear (cublas_ops.cuh:359): output (F32) = x . W^T + bias.  Same asserts, same rule that
// only an F32 GPU bias is used, same F32-activation cast (done inside the engine).
static void linear(const Tensor& x, const Tensor& W, const Tensor* bias, Tensor& output) {
  if (W.dtype == DType::INT8 || g_calib.active) {
    ref_cublaslt_linear(x, W, bias, output);
    return;
  }
  assert(x.on_gpu && W.on_gpu && output.on_gpu);
  assert(x.ndim >= 1 && W.ndim == 2);
  const int64_t K = x.shape[x.ndim - 1];
  const int64_t M = x.numel() / K;
  const int64_t N = W.shape[0];
  assert(W.shape[1] == K);
  assert(output.numel() == M * N);
  const bool x_ok = x.dtype == W.dtype || (x.dtype == DType::F32 && W.dtype != DType::F32);
  if (!x_ok) {
    fprintf(stderr, "Unsupported dtype combo in linear: x=%s W=%s\n", dtype_name(x.dtype), dtype_name(W.dtype));
    exit(1);
  }
  b2g_gemm_desc d{};
  d.M = M;
  d.N = N;
  d.K = K;
  d.a = x.data;
  d.a_dtype = b2g_dtype_of(x.dtype);
  d.lda = K;
  d.b = W.data;
  d.b_dtype = b2g_dtype_of(W.dtype);
  d.ldb = K;
  d.bias = (bias && bias->on_gpu && bias->dtype == DType::F32) ? bias->data : nullptr;
  d.bias_dtype = B2G_F32;
  d.d = output.data;
  d.d_dtype = B2G_F32;
  d.ldd = N;
  d.epilogue = B2G_EPI_NONE;
  B2G_CHECK(b2g_gemm(&d, nullptr));
}

// linear_gated_residual (cublas_ops.cuh:684): residual += gate * (x . W^T + bias), fused.
static void linear_gated_residual(const Tensor& x, const Tensor& W, const Tensor* bias, float* residual_inout,
                                  const float* gate, int64_t M, int64_t N_out) {
  if (W.dtype == DType::INT8) {
    ref_cublaslt_linear_gated_residual(x, W, bias, residual_inout, gate, M, N_out);
    return;
  }
  const int64_t K = x.shape[x.ndim - 1];
  const float* b = (bias && bias->on_gpu && bias->dtype == DType::F32) ? bias->f32() : nullptr;
  B2G_CHECK(b2g_linear_gated_residual(x.data, b2g_cuda_type_of(x.dtype), W.data, b2g_cuda_type_of(W.dtype), b,
                                      residual_inout, gate, M, K, N_out));
}

// batched_matmul_Bt (cublas_ops.cuh:558): C[b] = A[b] . B[b]^T, all F32.
static void batched_matmul_Bt(const Tensor& A, const Tensor& B, Tensor& C) {
  assert(A.on_gpu && B.on_gpu && C.on_gpu);
  assert(A.dtype == DType::F32 && B.dtype == DType::F32 && C.dtype == DType::F32);
  assert(A.ndim == 3 && B.ndim == 3 && C.ndim == 3);
  const int64_t batch = A.shape[0], M = A.shape[1], K = A.shape[2], N = B.shape[1];
  assert(B.shape[0] == batch && B.shape[2] == K);
  assert(C.shape[0] == batch && C.shape[1] == M && C.shape[2] == N);
  B2G_CHECK(b2g_batched_matmul_Bt(A.f32(), B.f32(), C.f32(), batch, M, K, N));
}
