// attention.cuh — drop-in replacement for the reference's attention.cuh.
//
// Integration: in the reference tree, rename its original attention.cuh to
// attention_cublas.cuh and put this file in its place.  chroma.cuh and t5.cuh then compile
// unchanged.
//
// Routing:
//   t5_attention (attention.cuh:34-91: permute, fp32 cuBLAS QK^T, relative bias, masked
//     softmax, fp32 cuBLAS P.V)  -> b2g_t5_attention: the same computation on the tensor cores
//     (scores at fp32-level accuracy from TF32 hi/lo operand splits), F32 [L, n_head*d_head]
//   attention_with_rope (attention.cuh:23-28) -> unchanged: it calls cudnn_attention_with_rope,
//     which the drop-in cudnn_attention.cuh routes to the engine
// Errors keep the reference's behaviour: print and exit(1).
#pragma once
#include "tensor.cuh"
#include "b2g.h"

#define t5_attention ref_cublas_t5_attention
#include "attention_cublas.cuh"
#undef t5_attention

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

// t5_attention (attention.cuh:34): Q, K, V F32 [L, n_head, d_head]; rel_bias [n_head, L, L]
// or null; scores scaled by `scale`; attn_mask [L] (0 / -inf on keys) or null.
static Tensor t5_attention(const Tensor& Q, const Tensor& K, const Tensor& V, const float* rel_bias, int n_head,
                           int d_head, float scale, const float* attn_mask = nullptr) {
  assert(Q.on_gpu && K.on_gpu && V.on_gpu);
  const int64_t L = Q.shape[0];
  Tensor output = Tensor::alloc({L, (int64_t)(n_head * d_head)}, DType::F32, true);
  B2G_CHECK(b2g_t5_attention(Q.f32(), K.f32(), V.f32(), rel_bias, n_head, d_head, L, scale, attn_mask,
                             output.f32(), nullptr));
  return output;
}
