// ref_attn_shim.cu — TEST INFRASTRUCTURE ONLY.  The reference's attention path, unchanged,
// compiled from its sources (attention.cuh -> cudnn_attention.cuh, rope.cuh, kernels.cu)
// behind extern "C" functions: cuDNN-frontend flash SDPA with RoPE, exactly as the Chroma
// blocks call it (chroma.cuh:721, 1092).
#include <functional>
#include "tensor.cuh"
#include "cublas_ops.cuh"
#include "kernels.cu"
#include "attention.cuh"

extern "C" {

int ref_attn_init(void) {
  init_cublas();
  init_cudnn();
  return 0;
}

// Q, K, V: F32 [L, n_head, d_head]; pe F32 [L, d_head/2*4]; mask F32 [L] or null;
// out F32 [L, n_head*d_head].
int ref_attention_with_rope(const float* Q, const float* K, const float* V, const float* pe, int n_head, int d_head,
                            int64_t L, const float* mask, float* out) {
  Tensor tq = Tensor::wrap_gpu(const_cast<float*>(Q), {L, (int64_t)n_head, (int64_t)d_head}, DType::F32);
  Tensor tk = Tensor::wrap_gpu(const_cast<float*>(K), {L, (int64_t)n_head, (int64_t)d_head}, DType::F32);
  Tensor tv = Tensor::wrap_gpu(const_cast<float*>(V), {L, (int64_t)n_head, (int64_t)d_head}, DType::F32);
  Tensor tp = Tensor::wrap_gpu(const_cast<float*>(pe), {L, (int64_t)d_head / 2 * 4}, DType::F32);
  Tensor o = attention_with_rope(tq, tk, tv, tp, n_head, d_head, mask);
  CHECK_CUDA(cudaMemcpy(out, o.data, o.nbytes(), cudaMemcpyDeviceToDevice));
  return 0;
}

// Times attention_with_rope with CUDA events (device buffers given by the caller).
int ref_bench_attention(const float* Q, const float* K, const float* V, const float* pe, int n_head, int d_head,
                        int64_t L, const float* mask, int iters, int warmup, double* ms_total) {
  Tensor tq = Tensor::wrap_gpu(const_cast<float*>(Q), {L, (int64_t)n_head, (int64_t)d_head}, DType::F32);
  Tensor tk = Tensor::wrap_gpu(const_cast<float*>(K), {L, (int64_t)n_head, (int64_t)d_head}, DType::F32);
  Tensor tv = Tensor::wrap_gpu(const_cast<float*>(V), {L, (int64_t)n_head, (int64_t)d_head}, DType::F32);
  Tensor tp = Tensor::wrap_gpu(const_cast<float*>(pe), {L, (int64_t)d_head / 2 * 4}, DType::F32);
  for (int i = 0; i < warmup; ++i) {
    Tensor o = attention_with_rope(tq, tk, tv, tp, n_head, d_head, mask);
  }
  CHECK_CUDA(cudaDeviceSynchronize());
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  double total = 0;
  for (int i = 0; i < iters; ++i) {
    cudaEventRecord(e0, 0);
    Tensor o = attention_with_rope(tq, tk, tv, tp, n_head, d_head, mask);
    cudaEventRecord(e1, 0);
    cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    total += ms;
  }
  *ms_total = total;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return 0;
}

}  // extern "C"
