// forward_cfg_harness.cu — runs the reference's own ChromaRadiance::forward_cfg
// (chroma.cuh:1499-1584: img_in conv, txt_in, approximator, 19 double + 38 single blocks under
// classifier-free guidance, two NeRF decodes, cfg_blend) on seeded random-init weights.
//
// Built twice from the reference's sources, which are never modified:
//   stock    with the reference's own cublas_ops.cuh / cudnn_attention.cuh / attention.cuh
//            (cuBLASLt, cuDNN SDPA, cuBLAS): the reference arm of the benchmark;
//   drop-in  through build_reference_with_b2g.sh --shared, with this directory's drop-in
//            headers in place of those three: the same model code with every GEMM and every
//            attention in libb2g.so (what a maintainer gets by swapping the headers).
// The weights are the reference's own Tensor fields (bypassing load(), which needs the 19 GB
// checkpoint), filled with the reference's Philox generator (rand_normal_cuda, kernels.cu), so
// the two builds hold bit-identical weights for the same seed.  Every weight and input is
// exported by its checkpoint name (fc_tensor), so a caller can run another implementation on
// the very same device buffers.
#include <functional>
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>
#include "tensor.cuh"
#include "cublas_ops.cuh"
#include "kernels.cu"
#include "rope.cuh"
#include "attention.cuh"
#include "chroma.cuh"

void scale_cuda(float* x, float scale, int64_t n);
void add_scalar_cuda(float* x, float val, int64_t n);

namespace {

ChromaRadiance* g_model = nullptr;
std::unordered_map<std::string, Tensor*> g_named;
std::vector<std::string> g_names;
unsigned long long g_seed = 0;
int g_H = 0, g_W = 0, g_T = 0;

// Inputs of forward_cfg (main.cu:379-471 builds the same ones from the prompt and noise).
Tensor g_x, g_ctx_c, g_ctx_u, g_pe, g_dct, g_mask_c, g_mask_u, g_vel, g_mod;
float* g_host_in = nullptr;   // pinned: x, ctx_c, ctx_u (the per-step inputs)
float* g_host_out = nullptr;  // pinned: velocity

void name(const std::string& n, Tensor& t) {
  g_named[n] = &t;
  g_names.push_back(n);
}

// t = shift + scale * N(0, 1) from the reference's Philox generator, stored as t.dtype.
void fill(Tensor& t, float scale, float shift) {
  const int64_t n = t.numel();
  Tensor f = Tensor::alloc({n}, DType::F32, true);
  rand_normal_cuda(f.f32(), n, ++g_seed);
  scale_cuda(f.f32(), scale, n);
  if (shift != 0.f) add_scalar_cuda(f.f32(), shift, n);
  if (t.dtype == DType::F32) {
    CHECK_CUDA(cudaMemcpy(t.data, f.data, n * 4, cudaMemcpyDeviceToDevice));
  } else {
    f32_to_bf16_cuda(f.f32(), t.bf16(), n);
  }
  CHECK_CUDA(cudaDeviceSynchronize());
}

Tensor weight(std::initializer_list<int64_t> dims) {  // bf16 linear weights ~ N(0, 0.02)
  Tensor t = Tensor::alloc(dims, DType::BF16, true);
  fill(t, 0.02f, 0.f);
  return t;
}
Tensor bias(int64_t n) {  // F32 biases ~ N(0, 0.02)
  Tensor t = Tensor::alloc({n}, DType::F32, true);
  fill(t, 0.02f, 0.f);
  return t;
}
Tensor norm_scale(int64_t n) {  // F32 RMSNorm scales ~ 1 + N(0, 0.1)
  Tensor t = Tensor::alloc({n}, DType::F32, true);
  fill(t, 0.1f, 1.f);
  return t;
}

// The DCT position features of the NeRF decoder (main.cu:22-65), [256, 64].
std::vector<float> dct_features(int patch, int freqs) {
  const float PI = 3.14159265358979323846f;
  std::vector<float> out(static_cast<size_t>(patch * patch * freqs * freqs));
  for (int p = 0; p < patch * patch; ++p) {
    const float px = static_cast<float>(p % patch) / static_cast<float>(patch - 1);
    const float py = static_cast<float>(p / patch) / static_cast<float>(patch - 1);
    for (int fx = 0; fx < freqs; ++fx) {
      const float cx = cosf(px * static_cast<float>(fx) * PI);
      for (int fy = 0; fy < freqs; ++fy) {
        const float cy = cosf(py * static_cast<float>(fy) * PI);
        out[p * freqs * freqs + fx * freqs + fy] = cx * cy * (1.0f / (1.0f + static_cast<float>(fx) * fy));
      }
    }
  }
  return out;
}

// Key bias of one guidance half (main.cu:413-430): the first real_tokens + 1 text tokens and
// every image token attend, the rest of the text tokens are -inf.
std::vector<float> key_mask(int T, int L, int real_tokens) {
  std::vector<float> m(L, 0.f);
  for (int i = std::min(real_tokens + 1, T); i < T; ++i) m[i] = -HUGE_VALF;
  return m;
}

template <typename V>
void upload(Tensor& t, const V& host) {
  CHECK_CUDA(cudaMemcpy(t.data, host.data(), host.size() * sizeof(host[0]), cudaMemcpyHostToDevice));
}

}  // namespace

extern "C" {

// Builds the model with random weights (seed) for an H x W image and 512 text tokens, and the
// forward_cfg inputs: noise x ~ N(0,1) [1,3,H,W], the two T5 contexts ~ N(0,1) [512,4096], the
// RoPE table (RoPE::gen_pe, as main.cu builds it), the DCT features and the two key masks
// (real_cond / real_uncond prompt tokens).  Returns 0 or a CUDA error code.
int fc_setup(unsigned long long seed, int H, int W, int real_cond, int real_uncond) {
  if (g_model) return 0;
  init_cublas();
  init_cudnn();
  g_seed = seed * 1000003ull;
  g_H = H;
  g_W = W;
  g_T = 512;
  ChromaRadiance& m = *(g_model = new ChromaRadiance());
  const int64_t D = ChromaRadiance::hidden_size, MLP = ChromaRadiance::mlp_hidden;
  m.img_in_patch_w = weight({D, 3, 16, 16});
  m.img_in_patch_b = bias(D);
  m.txt_in_w = weight({D, 4096});
  m.txt_in_b = bias(D);
  name("img_in_patch.weight", m.img_in_patch_w);
  name("img_in_patch.bias", m.img_in_patch_b);
  name("txt_in.weight", m.txt_in_w);
  name("txt_in.bias", m.txt_in_b);
  m.nerf_small.embedder_w = weight({64, 67});
  m.nerf_small.embedder_b = bias(64);
  m.nerf_small.final_norm_scale = norm_scale(64);
  m.nerf_small.final_conv_w = Tensor::alloc({3, 64, 3, 3}, DType::F32, true);
  fill(m.nerf_small.final_conv_w, 0.02f, 0.f);
  m.nerf_small.final_conv_b = bias(3);
  name("nerf_image_embedder.embedder.0.weight", m.nerf_small.embedder_w);
  name("nerf_image_embedder.embedder.0.bias", m.nerf_small.embedder_b);
  name("nerf_final_layer_conv.norm.scale", m.nerf_small.final_norm_scale);
  name("nerf_final_layer_conv.conv.weight", m.nerf_small.final_conv_w);
  name("nerf_final_layer_conv.conv.bias", m.nerf_small.final_conv_b);
  auto& a = m.approx;
  const std::string ap = "distilled_guidance_layer.";
  a.in_proj_w = weight({5120, 64});
  a.in_proj_b = bias(5120);
  a.out_proj_w = weight({D, 5120});
  a.out_proj_b = bias(D);
  name(ap + "in_proj.weight", a.in_proj_w);
  name(ap + "in_proj.bias", a.in_proj_b);
  name(ap + "out_proj.weight", a.out_proj_w);
  name(ap + "out_proj.bias", a.out_proj_b);
  for (int i = 0; i < 5; ++i) {
    auto& l = a.layers[i];
    l.norm_scale = norm_scale(5120);
    l.in_w = weight({5120, 5120});
    l.in_b = bias(5120);
    l.out_w = weight({5120, 5120});
    l.out_b = bias(5120);
    const std::string lp = ap + "layers." + std::to_string(i) + ".";
    name(ap + "norms." + std::to_string(i) + ".scale", l.norm_scale);
    name(lp + "in_layer.weight", l.in_w);
    name(lp + "in_layer.bias", l.in_b);
    name(lp + "out_layer.weight", l.out_w);
    name(lp + "out_layer.bias", l.out_b);
  }
  m.double_block_weights.resize(ChromaRadiance::depth);
  for (int i = 0; i < ChromaRadiance::depth; ++i) {
    auto& w = m.double_block_weights[i];
    const std::string p = "double_blocks." + std::to_string(i) + ".";
    struct S { const char* s; Tensor *qkv_w, *qkv_b, *qn, *kn, *proj_w, *proj_b, *m0w, *m0b, *m2w, *m2b; };
    S streams[2] = {{"img", &w.img_qkv_w, &w.img_qkv_b, &w.img_q_norm, &w.img_k_norm, &w.img_proj_w, &w.img_proj_b,
                     &w.img_mlp_0_w, &w.img_mlp_0_b, &w.img_mlp_2_w, &w.img_mlp_2_b},
                    {"txt", &w.txt_qkv_w, &w.txt_qkv_b, &w.txt_q_norm, &w.txt_k_norm, &w.txt_proj_w, &w.txt_proj_b,
                     &w.txt_mlp_0_w, &w.txt_mlp_0_b, &w.txt_mlp_2_w, &w.txt_mlp_2_b}};
    for (auto& s : streams) {
      const std::string sp = p + s.s;
      *s.qkv_w = weight({3 * D, D});
      *s.qkv_b = bias(3 * D);
      *s.qn = norm_scale(128);
      *s.kn = norm_scale(128);
      *s.proj_w = weight({D, D});
      *s.proj_b = bias(D);
      *s.m0w = weight({MLP, D});
      *s.m0b = bias(MLP);
      *s.m2w = weight({D, MLP});
      *s.m2b = bias(D);
      name(sp + "_attn.qkv.weight", *s.qkv_w);
      name(sp + "_attn.qkv.bias", *s.qkv_b);
      name(sp + "_attn.norm.query_norm.scale", *s.qn);
      name(sp + "_attn.norm.key_norm.scale", *s.kn);
      name(sp + "_attn.proj.weight", *s.proj_w);
      name(sp + "_attn.proj.bias", *s.proj_b);
      name(sp + "_mlp.0.weight", *s.m0w);
      name(sp + "_mlp.0.bias", *s.m0b);
      name(sp + "_mlp.2.weight", *s.m2w);
      name(sp + "_mlp.2.bias", *s.m2b);
    }
  }
  m.single_block_weights.resize(ChromaRadiance::depth_single);
  for (int i = 0; i < ChromaRadiance::depth_single; ++i) {
    auto& w = m.single_block_weights[i];
    const std::string p = "single_blocks." + std::to_string(i) + ".";
    w.linear1_w = weight({3 * D + MLP, D});
    w.linear1_b = bias(3 * D + MLP);
    w.linear2_w = weight({D, D + MLP});
    w.linear2_b = bias(D);
    w.q_norm = norm_scale(128);
    w.k_norm = norm_scale(128);
    name(p + "linear1.weight", w.linear1_w);
    name(p + "linear1.bias", w.linear1_b);
    name(p + "linear2.weight", w.linear2_w);
    name(p + "linear2.bias", w.linear2_b);
    name(p + "norm.query_norm.scale", w.q_norm);
    name(p + "norm.key_norm.scale", w.k_norm);
  }
  m.nerf_block_weights.resize(ChromaRadiance::nerf_depth);
  for (int i = 0; i < ChromaRadiance::nerf_depth; ++i) {
    auto& w = m.nerf_block_weights[i];
    const std::string p = "nerf_blocks." + std::to_string(i) + ".";
    w.param_gen_w = weight({3 * 64 * 256, D});
    w.param_gen_b = bias(3 * 64 * 256);
    w.norm_scale = norm_scale(64);
    name(p + "param_generator.weight", w.param_gen_w);
    name(p + "param_generator.bias", w.param_gen_b);
    name(p + "norm.scale", w.norm_scale);
  }

  // forward_cfg inputs
  const int L = g_T + (H / 16) * (W / 16);
  g_x = Tensor::alloc({1, 3, H, W}, DType::F32, true);
  fill(g_x, 1.f, 0.f);
  g_ctx_c = Tensor::alloc({g_T, 4096}, DType::F32, true);
  fill(g_ctx_c, 1.f, 0.f);
  g_ctx_u = Tensor::alloc({g_T, 4096}, DType::F32, true);
  fill(g_ctx_u, 1.f, 0.f);
  std::vector<int> axes = {16, 56, 56};
  const std::vector<float> pe = RoPE::gen_pe(H, W, 16, g_T, 10000, axes);
  g_pe = Tensor::alloc({L, 256}, DType::F32, true);
  upload(g_pe, pe);
  g_dct = Tensor::alloc({256, 64}, DType::F32, true);
  upload(g_dct, dct_features(16, 8));
  g_mask_c = Tensor::alloc({L}, DType::F32, true);
  upload(g_mask_c, key_mask(g_T, L, real_cond));
  g_mask_u = Tensor::alloc({L}, DType::F32, true);
  upload(g_mask_u, key_mask(g_T, L, real_uncond));
  g_vel = Tensor::alloc({1, 3, H, W}, DType::F32, true);
  g_mod = Tensor::alloc({ChromaRadiance::mod_index_length, D}, DType::F32, true);
  name("x", g_x);
  name("context_cond", g_ctx_c);
  name("context_uncond", g_ctx_u);
  name("pe", g_pe);
  name("dct", g_dct);
  name("mask_cond", g_mask_c);
  name("mask_uncond", g_mask_u);
  name("velocity", g_vel);
  name("mod", g_mod);
  const size_t in_floats = static_cast<size_t>(3 * H * W + 2 * g_T * 4096);
  CHECK_CUDA(cudaMallocHost(&g_host_in, in_floats * 4));
  CHECK_CUDA(cudaMallocHost(&g_host_out, static_cast<size_t>(3 * H * W) * 4));
  CHECK_CUDA(cudaMemcpy(g_host_in, g_x.data, g_x.nbytes(), cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(g_host_in + 3 * H * W, g_ctx_c.data, g_ctx_c.nbytes(), cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(g_host_in + 3 * H * W + g_T * 4096, g_ctx_u.data, g_ctx_u.nbytes(), cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaDeviceSynchronize());
  return static_cast<int>(cudaGetLastError());
}

// Device pointer, dtype (0 F32, 1 FP16, 2 BF16) and element count of a weight or input by its
// checkpoint name (e.g. "double_blocks.3.img_attn.qkv.weight") or input name ("x",
// "context_cond", "context_uncond", "pe", "dct", "mask_cond", "mask_uncond", "velocity", "mod").
int fc_tensor(const char* n, void** ptr, int* dtype, int64_t* numel) {
  auto it = g_named.find(n);
  if (it == g_named.end()) return 1;
  *ptr = it->second->data;
  *dtype = static_cast<int>(it->second->dtype);
  *numel = it->second->numel();
  return 0;
}

int fc_num_tensors(void) { return static_cast<int>(g_names.size()); }
const char* fc_tensor_name(int i) { return i >= 0 && i < static_cast<int>(g_names.size()) ? g_names[i].c_str() : ""; }

// One forward_cfg on the current inputs; the velocity [1,3,H,W] lands in "velocity".
int fc_forward(float timestep, float cfg_scale) {
  Tensor v = g_model->forward_cfg(g_x, g_ctx_c, g_ctx_u, timestep, g_pe, g_dct, g_mask_c.f32(), g_mask_u.f32(),
                                  cfg_scale);
  CHECK_CUDA(cudaMemcpyAsync(g_vel.data, v.data, g_vel.nbytes(), cudaMemcpyDeviceToDevice, 0));
  CHECK_CUDA(cudaDeviceSynchronize());
  return static_cast<int>(cudaGetLastError());
}

// The approximator's modulation vectors for `timestep` (compute_modulation, guidance 0 as
// forward_cfg calls it) into "mod" [344, 3072].
int fc_modulation(float timestep) {
  Tensor m = g_model->compute_modulation(timestep, 0.0f);
  CHECK_CUDA(cudaMemcpyAsync(g_mod.data, m.data, g_mod.nbytes(), cudaMemcpyDeviceToDevice, 0));
  CHECK_CUDA(cudaDeviceSynchronize());
  return static_cast<int>(cudaGetLastError());
}

// Times compute_modulation (the approximator, chroma.cuh:467-508: timestep embedding, in_proj,
// 5 residual MLP layers of 5120, out_proj to the [344, 3072] modulation vectors) with CUDA
// events on stream 0, `iters` calls after `warmup`; ms[i] is call i's time, a `flush_bytes`
// buffer rewritten before each call outside the events.
int fc_bench_modulation(float timestep, int iters, int warmup, int64_t flush_bytes, double* ms) {
  for (int i = 0; i < warmup; ++i) Tensor m = g_model->compute_modulation(timestep, 0.0f);
  void* flush = nullptr;
  if (flush_bytes > 0) CHECK_CUDA(cudaMalloc(&flush, flush_bytes));
  CHECK_CUDA(cudaDeviceSynchronize());
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  for (int i = 0; i < iters; ++i) {
    if (flush) cudaMemsetAsync(flush, i & 0xFF, flush_bytes, 0);
    cudaEventRecord(e0, 0);
    {
      Tensor m = g_model->compute_modulation(timestep, 0.0f);
    }
    cudaEventRecord(e1, 0);
    cudaEventSynchronize(e1);
    float t = 0;
    cudaEventElapsedTime(&t, e0, e1);
    ms[i] = t;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (flush) cudaFree(flush);
  return static_cast<int>(cudaGetLastError());
}

// Times NeRF GLU block `blk` (nerf_glu_block, chroma.cuh:1253-1306: the param_generator linear,
// the weight slices and L2 norms, rms_norm, three batched products, silu_mul and the residual
// add) on x [P, 256, 64] (updated in place by every call) and s [P, 3072], both F32 device
// pointers; CUDA events on stream 0 around each call, a `flush_bytes` buffer rewritten before
// each outside them; ms[i] is call i's time.
int fc_bench_nerf_glu_block(int blk, float* x, const float* s, int64_t P, int iters, int warmup, int64_t flush_bytes,
                            double* ms) {
  if (blk < 0 || blk >= static_cast<int>(g_model->nerf_block_weights.size())) return -1;
  Tensor tx = Tensor::wrap_gpu(x, {P, 256, 64}, DType::F32);
  Tensor ts = Tensor::wrap_gpu(const_cast<float*>(s), {P, (int64_t)ChromaRadiance::hidden_size}, DType::F32);
  const auto& w = g_model->nerf_block_weights[blk];
  for (int i = 0; i < warmup; ++i) g_model->nerf_glu_block(tx, ts, w);
  void* flush = nullptr;
  if (flush_bytes > 0) CHECK_CUDA(cudaMalloc(&flush, flush_bytes));
  CHECK_CUDA(cudaDeviceSynchronize());
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  for (int i = 0; i < iters; ++i) {
    if (flush) cudaMemsetAsync(flush, i & 0xFF, flush_bytes, 0);
    cudaEventRecord(e0, 0);
    g_model->nerf_glu_block(tx, ts, w);
    cudaEventRecord(e1, 0);
    cudaEventSynchronize(e1);
    float t = 0;
    cudaEventElapsedTime(&t, e0, e1);
    ms[i] = t;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (flush) cudaFree(flush);
  return static_cast<int>(cudaGetLastError());
}

// One NeRF decode (nerf_decode, chroma.cuh:1163-1251) of transformer image rows img [P, 3072]
// (a device pointer) into out [1,3,H,W] (a device pointer).
int fc_nerf_decode(const float* img, float* out) {
  const int64_t P = static_cast<int64_t>(g_H / 16) * (g_W / 16);
  Tensor t = Tensor::wrap_gpu(const_cast<float*>(img), {P, (int64_t)ChromaRadiance::hidden_size}, DType::F32);
  Tensor v = g_model->nerf_decode(t, g_x, g_dct, g_H, g_W);
  CHECK_CUDA(cudaMemcpyAsync(out, v.data, v.nbytes(), cudaMemcpyDeviceToDevice, 0));
  CHECK_CUDA(cudaDeviceSynchronize());
  return static_cast<int>(cudaGetLastError());
}

// Times forward_cfg with CUDA events on stream 0 after `warmup` untimed calls.
//   *ms_device: the forward alone (inputs resident), summed over `iters` calls;
//   *ms_e2e:    per call also the host-to-device copy of that step's inputs (noise and the two
//               contexts, 19.9 MB at 512^2) from pinned memory and the velocity copied back.
// Before every timed call a `flush_bytes` buffer is written outside the events.
int fc_bench(float timestep, float cfg_scale, int iters, int warmup, int64_t flush_bytes, double* ms_device,
             double* ms_e2e) {
  for (int i = 0; i < warmup; ++i) {
    Tensor v = g_model->forward_cfg(g_x, g_ctx_c, g_ctx_u, timestep, g_pe, g_dct, g_mask_c.f32(), g_mask_u.f32(),
                                    cfg_scale);
  }
  void* flush = nullptr;
  if (flush_bytes > 0) CHECK_CUDA(cudaMalloc(&flush, flush_bytes));
  CHECK_CUDA(cudaDeviceSynchronize());
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  const int64_t nx = 3LL * g_H * g_W, nc = static_cast<int64_t>(g_T) * 4096;
  double dev = 0, e2e = 0;
  for (int pass = 0; pass < 2; ++pass) {
    for (int i = 0; i < iters; ++i) {
      if (flush) cudaMemsetAsync(flush, i & 0xFF, flush_bytes, 0);
      cudaEventRecord(e0, 0);
      if (pass == 1) {
        cudaMemcpyAsync(g_x.data, g_host_in, nx * 4, cudaMemcpyHostToDevice, 0);
        cudaMemcpyAsync(g_ctx_c.data, g_host_in + nx, nc * 4, cudaMemcpyHostToDevice, 0);
        cudaMemcpyAsync(g_ctx_u.data, g_host_in + nx + nc, nc * 4, cudaMemcpyHostToDevice, 0);
      }
      {
        Tensor v = g_model->forward_cfg(g_x, g_ctx_c, g_ctx_u, timestep, g_pe, g_dct, g_mask_c.f32(),
                                        g_mask_u.f32(), cfg_scale);
        if (pass == 1) cudaMemcpyAsync(g_host_out, v.data, nx * 4, cudaMemcpyDeviceToHost, 0);
      }
      cudaEventRecord(e1, 0);
      cudaEventSynchronize(e1);
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      (pass == 0 ? dev : e2e) += ms;
    }
  }
  *ms_device = dev;
  *ms_e2e = e2e;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (flush) cudaFree(flush);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
