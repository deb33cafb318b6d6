// cudnn_attention.cuh — drop-in replacement for the reference's attention header
// (cudnn_attention.cuh).
//
// Integration: in the reference tree, rename its original cudnn_attention.cuh to
// cudnn_attention_cudnn.cuh and put this file in its place (as with the drop-in
// cublas_ops.cuh).  attention.cuh and chroma.cuh then compile unchanged.
//
// Routing:
//   cudnn_attention_with_rope (cudnn_attention.cuh:449-476: RoPE + permute to bf16, cuDNN
//     flash SDPA, un-permute to F32)  -> b2g_attention_with_rope: the RoPE producer and the
//     engine's tcgen05 attention kernel, F32 [L, n_head*d_head] out, same key-bias mask
//   everything else (init_cudnn, build_sdpa_graph, cudnn_sdpa_forward and the INT8 attention
//     helpers the INT8 block path calls directly) -> the original code, renamed below
// Errors keep the reference's behaviour: print and exit(1).
#pragma once
#include "tensor.cuh"
#include "b2g.h"

#define cudnn_attention_with_rope ref_cudnn_attention_with_rope
#include "cudnn_attention_cudnn.cuh"
#undef cudnn_attention_with_rope

#ifndef B2G_CHECK
#define B2G_CHECK(call)                                                                         \
  do {                                                                                          \
    b2g_status b2g_st_ = (call);                                                                \
    if (b2g_st_ != B2G_OK) {                                                                    \
      fprintf(stderr, "b2g error at %s:%d: %d (%s)\n", __FILE__, __LINE__, (int)b2g_st_,         \
              b2g_last_error());                                                                \
      exit(1);                                                                                  \
    }                                                                                           \
  } while (0)
#endif

// cudnn_attention_with_rope (cudnn_attention.cuh:449): Q, K, V F32 [L, n_head, d_head], pe F32
// [L, d_head/2*4], attn_mask F32 [L] (0 / -inf) or null; returns F32 [L, n_head*d_head].
static Tensor cudnn_attention_with_rope(const Tensor& Q, const Tensor& K, const Tensor& V, const Tensor& pe,
                                         int n_head, int d_head, const float* attn_mask = nullptr) {
  assert(Q.on_gpu && K.on_gpu && V.on_gpu && pe.on_gpu);
  assert(Q.dtype == DType::F32 && K.dtype == DType::F32 && V.dtype == DType::F32 && pe.dtype == DType::F32);
  const int64_t L = Q.shape[0];
  Tensor output = Tensor::alloc({L, (int64_t)(n_head * d_head)}, DType::F32, true);
  B2G_CHECK(b2g_attention_with_rope(Q.f32(), K.f32(), V.f32(), pe.f32(), n_head, d_head, L, attn_mask,
                                    output.f32(), nullptr));
  return output;
}
