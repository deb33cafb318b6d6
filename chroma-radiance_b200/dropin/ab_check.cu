// ab_check.cu — compiled inside the reference tree by build_reference_with_b2g.sh.  It
// includes the reference's model headers unchanged (through the drop-in cublas_ops.cuh,
// cudnn_attention.cuh and attention.cuh), then runs each routed entry point twice on the
// same device buffers: once through the engine (the names the model code calls) and once
// through the original code (renamed ref_cublaslt_*, ref_cudnn_attention_with_rope,
// ref_cublas_t5_attention), and prints max|diff|/max|ref| per entry point.
#include <functional>
#include "tensor.cuh"
#include "cublas_ops.cuh"
#include "kernels.cu"
#include "t5.cuh"
#include "chroma.cuh"
#include "sampler.cuh"
#include <vector>

static double rel_diff(const Tensor& a, const Tensor& b) {
  std::vector<float> ha(a.numel()), hb(b.numel());
  CHECK_CUDA(cudaMemcpy(ha.data(), a.data, a.nbytes(), cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(hb.data(), b.data, b.nbytes(), cudaMemcpyDeviceToHost));
  double md = 0, mr = 0;
  for (size_t i = 0; i < ha.size(); ++i) {
    md = fmax(md, fabs((double)ha[i] - hb[i]));
    mr = fmax(mr, fabs((double)hb[i]));
  }
  return mr > 0 ? md / mr : md;
}

static Tensor randn(std::initializer_list<int64_t> dims, DType dt, float scale, unsigned long long seed) {
  Tensor f = Tensor::alloc(dims, DType::F32, true);
  rand_normal_cuda(f.f32(), f.numel(), seed);
  scale_cuda(f.f32(), scale, f.numel());
  if (dt == DType::F32) return f;
  Tensor t = Tensor::alloc(dims, dt, true);
  if (dt == DType::BF16) f32_to_bf16_cuda(f.f32(), t.bf16(), f.numel());
  else f32_to_fp16_cuda(f.f32(), t.fp16(), f.numel());
  return t;
}

int main() {
  init_cublas();
  int fails = 0;
  auto report = [&](const char* name, double d, double tol) {
    printf("{\"entry\": \"%s\", \"rel_diff\": %.3e, \"tol\": %.1e}\n", name, d, tol);
    if (!(d <= tol)) ++fails;
  };
  // linear, bf16 activations (single-block linear1 at 512^2)
  {
    Tensor x = randn({1536, 3072}, DType::BF16, 1.0f, 1);
    Tensor w = randn({21504, 3072}, DType::BF16, 0.02f, 2);
    Tensor b = randn({21504}, DType::F32, 0.02f, 3);
    Tensor o1 = Tensor::alloc({1536, 21504}, DType::F32, true), o2 = Tensor::alloc({1536, 21504}, DType::F32, true);
    linear(x, w, &b, o1);
    ref_cublaslt_linear(x, w, &b, o2);
    report("linear bf16", rel_diff(o1, o2), 2e-3);
  }
  // linear, F32 activations with fp16 weights (T5 wi_0 shape)
  {
    Tensor x = randn({512, 4096}, DType::F32, 1.0f, 4);
    Tensor w = randn({10240, 4096}, DType::FP16, 0.02f, 5);
    Tensor o1 = Tensor::alloc({512, 10240}, DType::F32, true), o2 = Tensor::alloc({512, 10240}, DType::F32, true);
    linear(x, w, nullptr, o1);
    ref_cublaslt_linear(x, w, nullptr, o2);
    report("linear f32x fp16w", rel_diff(o1, o2), 2e-3);
  }
  // linear_gated_residual (double-block proj, F32 attention output)
  {
    Tensor x = randn({1024, 3072}, DType::F32, 1.0f, 6);
    Tensor w = randn({3072, 3072}, DType::BF16, 0.02f, 7);
    Tensor b = randn({3072}, DType::F32, 0.02f, 8);
    Tensor g = randn({3072}, DType::F32, 1.0f, 9);
    Tensor r1 = randn({1024, 3072}, DType::F32, 1.0f, 10), r2 = randn({1024, 3072}, DType::F32, 1.0f, 10);
    linear_gated_residual(x, w, &b, r1.f32(), g.f32(), 1024, 3072);
    ref_cublaslt_linear_gated_residual(x, w, &b, r2.f32(), g.f32(), 1024, 3072);
    report("linear_gated_residual", rel_diff(r1, r2), 2e-3);
  }
  // cudnn_attention_with_rope (the double block's attention at 512^2, F32 Q/K/V, RoPE table
  // and a key mask): engine kernel against the original cuDNN SDPA path
  {
    const int L = 1536, H = 24, D = 128;
    Tensor q = randn({L, H, D}, DType::F32, 1.0f, 13), k = randn({L, H, D}, DType::F32, 1.0f, 14);
    Tensor v = randn({L, H, D}, DType::F32, 1.0f, 15);
    std::vector<int> axes = {16, 56, 56};
    std::vector<float> pe_h = RoPE::gen_pe(512, 512, 16, 512, 10000, axes);
    Tensor pe = Tensor::alloc({L, D / 2 * 4}, DType::F32, true);
    CHECK_CUDA(cudaMemcpy(pe.data, pe_h.data(), pe_h.size() * 4, cudaMemcpyHostToDevice));
    std::vector<float> mask_h(L, 0.f);
    for (int i = 112; i < 512; ++i) mask_h[i] = -INFINITY;
    Tensor mask = Tensor::alloc({L}, DType::F32, true);
    CHECK_CUDA(cudaMemcpy(mask.data, mask_h.data(), L * 4, cudaMemcpyHostToDevice));
    init_cudnn();
    Tensor o1 = cudnn_attention_with_rope(q, k, v, pe, H, D, mask.f32());
    Tensor o2 = ref_cudnn_attention_with_rope(q, k, v, pe, H, D, mask.f32());
    report("cudnn_attention_with_rope", rel_diff(o1, o2), 1e-2);
  }
  // t5_attention (one T5-XXL layer: 512 tokens, 64 heads x 64, relative bias, scale 1)
  {
    const int L = 512, H = 64, D = 64;
    Tensor q = randn({L, H, D}, DType::F32, 1.0f, 16), k = randn({L, H, D}, DType::F32, 1.0f, 17);
    Tensor v = randn({L, H, D}, DType::F32, 1.0f, 18);
    Tensor bias = randn({H, L, L}, DType::F32, 1.0f, 19);
    Tensor o1 = t5_attention(q, k, v, bias.f32(), H, D, 1.0f, nullptr);
    Tensor o2 = ref_cublas_t5_attention(q, k, v, bias.f32(), H, D, 1.0f, nullptr);
    report("t5_attention", rel_diff(o1, o2), 2e-3);
  }
  // batched_matmul_Bt (NeRF GLU shape)
  {
    Tensor a = randn({64, 256, 64}, DType::F32, 1.0f, 11);
    Tensor bb = randn({64, 256, 64}, DType::F32, 1.0f, 12);
    Tensor c1 = Tensor::alloc({64, 256, 256}, DType::F32, true), c2 = Tensor::alloc({64, 256, 256}, DType::F32, true);
    batched_matmul_Bt(a, bb, c1);
    ref_cublaslt_batched_matmul_Bt(a, bb, c2);
    report("batched_matmul_Bt", rel_diff(c1, c2), 2e-3);
  }
  CHECK_CUDA(cudaDeviceSynchronize());
  printf("{\"fails\": %d}\n", fails);
  return fails ? 1 : 0;
}
