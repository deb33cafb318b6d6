// nerf_glu.cu — one NeRF GLU block (NerfGLUBlock::forward, chroma.cuh:1253-1306) fused into one
// persistent kernel on the tcgen05 tensor cores, for every patch of both guidance halves:
//
//   w_gate[m][h]  = G[h][m] / ||G[., m]||,  w_value likewise,  w_fc2[h][m] = F[m][h] / ||F[., h]||
//                   (G, V, F: the three slices of the patch's param_generator output row)
//   xn            = rms_norm(x) * scale                         x: the patch's state [256, 64]
//   x1, x2        = xn . w_gate^T,  xn . w_value^T              [256, 256], TF32 products
//   x            += (silu(x1) * x2) . w_fc2^T                   [256, 64],  TF32 products
//
// The reference runs this as 3 slice_transposes, 3 l2_norms, rms_norm, 3 cuBLAS batched GEMMs,
// silu_mul and add, with every intermediate in HBM (x1 and x2 alone are 268 MB per half at
// 512^2).  Here each patch's intermediates live in shared memory and TMEM; HBM sees the
// param_generator row once (192 KB) and the state once in and once out (64 KB each).
//
// A work item is one half of a patch (128 of its 256 pixel rows); the two halves of a patch
// are consecutive items, so two CTAs read its parameter row at about the same time (one from
// HBM, one from L2).  Two CTAs share an SM (84 KB of shared memory and 256 TMEM columns each),
// so one CTA's loads and normalisation overlap the other's MMAs and SiLU.  Per item, the 256
// MLP columns go in 4 chunks of 64:
//   threads   load the chunk's gate / value / fc2 slices, normalise (the fc2 norms, which
//             span all 256 columns, come from one pass before the chunks), round to TF32 and
//             write them as K-major operands with the 128-byte swizzle of the UMMA descriptors;
//   thread 0  issues x1, x2 (M = 128, N = 64, K = 64) into TMEM;
//   threads   read x1, x2 from TMEM (warp w: lanes 32(w%4).., columns 32(w/4)..), write
//             TF32(silu(x1) * x2) as the A operand of the fc2 product;
//   thread 0  issues x_out += h . w_fc2^T (N = 64, K = 64 of this chunk) into TMEM.
// Then every thread adds its part of x_out to the state and stores it.
//
// TF32 rounding (round to nearest even) happens where cuBLAS rounds the reference's
// CUBLAS_COMPUTE_32F_FAST_16BF operands: the normalised weights, the normed state and the
// SiLU product; accumulation is fp32.  Every mbarrier wait is bounded (ptx_sm100.cuh).
#include <cuda_runtime.h>
#include <cstdint>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {
namespace {

constexpr int kHid = 64, kMlp = 256, kRows = 128, kChunk = 64, kChunks = kMlp / kChunk;
constexpr int kPatchRows = 256;     // pixel rows of a patch; a work item is kRows of them
constexpr int kGluThreads = 256;
constexpr int kTmemCols = 256;       // D1 [0,64), D2 [64,128), D3 [128,192)
// Shared memory (bytes from a 1024-aligned base): K-major fp32 operands, 128-byte swizzle,
// one "atom" = 32 fp32 of K (128 bytes) per row, 8-row groups of 1024 bytes.
// The h chunk (A3) takes the place of the gate and value chunks (B1, B2): those are free once
// the x1, x2 MMAs have completed, and the next chunk's weights are written only after the fc2
// MMA that reads A3 has completed.
constexpr int kOffA1 = 0;                            // xn       [128 rows][K = 64 h]   2 atoms x 16 KB
constexpr int kOffB1 = kOffA1 + kRows * kHid * 4;    // gate    [64 m rows][K = 64 h] 2 atoms x 8 KB
constexpr int kOffB2 = kOffB1 + kChunk * kHid * 4;   // value   [64 m rows][K = 64 h]
constexpr int kOffA3 = kOffB1;                       // h chunk  [128 rows][K = 64 m]   2 atoms x 16 KB
constexpr int kOffB3 = kOffB2 + kChunk * kHid * 4;   // fc2     [64 h rows][K = 64 m]
static_assert(kRows * kChunk * 4 == 2 * kChunk * kHid * 4, "A3 fills exactly B1 and B2");
constexpr int kOffPart = kOffB3 + kHid * kChunk * 4;  // float [2][4][64] partial sums of squares
constexpr int kOffInvF = kOffPart + 2 * 4 * 64 * 4;   // float [64] fc2 inverse norms
constexpr int kOffBar = kOffInvF + 64 * 4;            // 3 mbarriers + TMEM slot
constexpr int kGluSmem = kOffBar + 64 + 1024;         // + alignment slack
static_assert(2 * kGluSmem <= 227 * 1024, "shared memory for two CTAs per SM");

// Byte offset of fp32 element (r, k) in a K-major operand of `rows` rows and K = 64.
__device__ __forceinline__ uint32_t sw_off(int rows, int r, int k) {
  const int a = k >> 5, c = k & 31;
  return static_cast<uint32_t>(a * rows * 128 + r * 128 + ((((c >> 2) ^ (r & 7))) << 4) + ((c & 3) << 2));
}

__device__ __forceinline__ float silu_f(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__global__ void __launch_bounds__(kGluThreads, 2)
    nerf_glu_kernel(const float* __restrict__ params, int64_t ldp, const float* __restrict__ scale,
                    float* __restrict__ x, int64_t patches, float eps, int* err) {
  const int64_t items = 2 * patches;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* part = reinterpret_cast<float*>(sm + kOffPart);
  float* invf = reinterpret_cast<float*>(sm + kOffInvF);
  uint64_t* bar12 = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint64_t* bar3 = bar12 + 1;
  uint64_t* drain = bar12 + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar12 + 3);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const uint32_t sbase = smem_u32(sm);

  if (t == 0) {
    mbar_init(bar12, 1);
    mbar_init(bar3, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t idesc = idesc_make(kFmtTF32, 128, kChunk);
  const int colh = warp >> 2, quarter = warp & 3;
  const int my_row = quarter * 32 + lane;  // the row this thread owns in the epilogues (columns 32 colh..)
  const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
  uint32_t ph12 = 0, ph3 = 0;
  bool ok = true;

  for (int64_t item = blockIdx.x; item < items && ok; item += gridDim.x) {
    const int64_t b = item >> 1;
    const float* prm = params + b * ldp;
    float* xb = x + (b * kPatchRows + (item & 1) * kRows) * kHid;
    // The next item's parameter row and state start moving into L2 now, so that its loads,
    // which this CTA issues in a few dependent rounds, are L2 hits rather than DRAM trips.
    if (item + gridDim.x < items) {
      const int64_t ni = item + gridDim.x;
      const char* np = reinterpret_cast<const char*>(params + (ni >> 1) * ldp);
      const char* nx = reinterpret_cast<const char*>(x + ((ni >> 1) * kPatchRows + (ni & 1) * kRows) * kHid);
      for (int i = t; i < 3 * kHid * kMlp * 4 / 128; i += kGluThreads) prefetch_l2(np + i * 128);
      for (int i = t; i < kRows * kHid * 4 / 128; i += kGluThreads) prefetch_l2(nx + i * 128);
    }
    // ---- normed state -> A1 (each warp 16 rows, each lane 2 columns)
    const float2 sc = reinterpret_cast<const float2*>(scale)[lane];
#pragma unroll 8
    for (int i = 0; i < kRows / 8; ++i) {
      const int r = warp * (kRows / 8) + i;
      const float2 v = reinterpret_cast<const float2*>(xb + r * kHid)[lane];
      float ss = v.x * v.x + v.y * v.y;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rr = rsqrtf(ss / static_cast<float>(kHid) + eps);
      *reinterpret_cast<float2*>(sm + kOffA1 + sw_off(kRows, r, 2 * lane)) =
          make_float2(round_tf32_cvt(v.x * rr * sc.x), round_tf32_cvt(v.y * rr * sc.y));
    }
    // ---- fc2 norms over its 256 rows m, for each column h
    {
      const int h = t & 63, q = t >> 6;
      float ss = 0.f;
#pragma unroll 16
      for (int m = q * 64; m < q * 64 + 64; ++m) {
        const float w = prm[2 * kHid * kMlp + m * kHid + h];
        ss += w * w;
      }
      part[q * 64 + h] = ss;
      __syncthreads();
      if (t < 64) invf[t] = 1.0f / fmaxf(sqrtf(part[t] + part[64 + t] + part[128 + t] + part[192 + t]), 1e-12f);
      __syncthreads();
    }
    for (int c = 0; c < kChunks && ok; ++c) {
      // ---- this chunk's 48 loads per thread, all issued before any is used
      const int mm = t & 63, hq = t >> 6;  // gate / value: column mm of the chunk, rows h of group hq
      const int fh = t & 63, mq = t >> 6;  // fc2: column h, rows m of group mq
      float g[16], v[16], f[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int h = hq * 16 + i;
        g[i] = prm[h * kMlp + c * kChunk + mm];
        v[i] = prm[kHid * kMlp + h * kMlp + c * kChunk + mm];
        f[i] = prm[2 * kHid * kMlp + (c * kChunk + mq * 16 + i) * kHid + fh];
      }
      // ---- gate / value chunk: L2-normalise each column mm over its 64 rows h
      {
        float sg = 0.f, sv = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          sg += g[i] * g[i];
          sv += v[i] * v[i];
        }
        part[hq * 64 + mm] = sg;
        part[256 + hq * 64 + mm] = sv;
        __syncthreads();
        const float ig = 1.0f / fmaxf(sqrtf(part[mm] + part[64 + mm] + part[128 + mm] + part[192 + mm]), 1e-12f);
        const float iv =
            1.0f / fmaxf(sqrtf(part[256 + mm] + part[320 + mm] + part[384 + mm] + part[448 + mm]), 1e-12f);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int h = hq * 16 + i;
          *reinterpret_cast<float*>(sm + kOffB1 + sw_off(kChunk, mm, h)) = round_tf32_cvt(g[i] * ig);
          *reinterpret_cast<float*>(sm + kOffB2 + sw_off(kChunk, mm, h)) = round_tf32_cvt(v[i] * iv);
        }
      }
      // ---- fc2 chunk: rows m of this chunk, column h; B3[n = h][k = m]
      {
        const float sf = invf[fh];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          *reinterpret_cast<float*>(sm + kOffB3 + sw_off(kHid, fh, mq * 16 + i)) = round_tf32_cvt(f[i] * sf);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      // ---- x1 = xn . gate^T, x2 = xn . value^T
      if (t == 0) {
        tc_fence_after();
#pragma unroll
        for (int ka = 0; ka < 2; ++ka) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t acc = (ka | k) ? 1u : 0u;
            const uint64_t ad = smem_desc_k_sw128(sbase + kOffA1 + ka * kRows * 128 + k * 32);
            umma_tf32(tmem, ad, smem_desc_k_sw128(sbase + kOffB1 + ka * kChunk * 128 + k * 32), idesc, acc);
            umma_tf32(tmem + kChunk, ad, smem_desc_k_sw128(sbase + kOffB2 + ka * kChunk * 128 + k * 32), idesc, acc);
          }
        }
        umma_commit(bar12);
      }
      ok = mbar_wait(bar12, ph12, err, kErrWaitEpilogue);
      ph12 ^= 1u;
      ok = __syncthreads_and(ok);
      if (!ok) break;
      tc_fence_after();
      // ---- h = TF32(silu(x1) * x2) -> A3 (this thread's row, the chunk's 64 columns)
      {
        uint32_t r1[32], r2[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + colh * 32, r1);
        tmem_ld_32x32b_x32(tmem + lane_addr + kChunk + colh * 32, r2);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 hv;
          hv.x = round_tf32_cvt(silu_f(__uint_as_float(r1[4 * j])) * __uint_as_float(r2[4 * j]));
          hv.y = round_tf32_cvt(silu_f(__uint_as_float(r1[4 * j + 1])) * __uint_as_float(r2[4 * j + 1]));
          hv.z = round_tf32_cvt(silu_f(__uint_as_float(r1[4 * j + 2])) * __uint_as_float(r2[4 * j + 2]));
          hv.w = round_tf32_cvt(silu_f(__uint_as_float(r1[4 * j + 3])) * __uint_as_float(r2[4 * j + 3]));
          *reinterpret_cast<float4*>(sm + kOffA3 + sw_off(kRows, my_row, colh * 32 + 4 * j)) = hv;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      // ---- x_out (+)= h . fc2^T over this chunk's 64 columns
      if (t == 0) {
        tc_fence_after();
#pragma unroll
        for (int ka = 0; ka < 2; ++ka) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_tf32(tmem + 2 * kChunk, smem_desc_k_sw128(sbase + kOffA3 + ka * kRows * 128 + k * 32),
                      smem_desc_k_sw128(sbase + kOffB3 + ka * kHid * 128 + k * 32), idesc, (c | ka | k) ? 1u : 0u);
          }
        }
        umma_commit(bar3);
      }
      ok = mbar_wait(bar3, ph3, err, kErrWaitEpilogue);
      ph3 ^= 1u;
      ok = __syncthreads_and(ok);
      tc_fence_after();
    }
    if (!ok) break;
    // ---- x += x_out for this thread's row, columns 32 colh ..
    {
      float* xr = xb + my_row * kHid + colh * 32;
      uint32_t r3[32];
      tmem_ld_32x32b_x32(tmem + lane_addr + 2 * kChunk + colh * 32, r3);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 v = reinterpret_cast<const float4*>(xr)[j];
        v.x += __uint_as_float(r3[4 * j]);
        v.y += __uint_as_float(r3[4 * j + 1]);
        v.z += __uint_as_float(r3[4 * j + 2]);
        v.w += __uint_as_float(r3[4 * j + 3]);
        reinterpret_cast<float4*>(xr)[j] = v;
      }
    }
    tc_fence_before();
    __syncthreads();  // every row stored and every TMEM read done before the next patch
  }
  if (!ok && t == 0) {
    // MMAs already issued must retire before TMEM is released.
    umma_commit(drain);
    mbar_wait_drain(drain, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace
}  // namespace b2g

using namespace b2g;

extern "C" b2g_status b2g_nerf_glu_block(const float* params, int64_t ldp, const float* norm_scale, float* x,
                                         int64_t patches, void* stream) {
  if (patches <= 0) return B2G_OK;
  if (!params || !norm_scale || !x || ldp < 3 * kHid * kMlp || (reinterpret_cast<uintptr_t>(x) & 15u) ||
      (reinterpret_cast<uintptr_t>(norm_scale) & 7u) || patches > (int64_t(1) << 31))
    return set_error(B2G_ERR_INVALID, "b2g_nerf_glu_block: arguments (ldp >= 49152, x 16-byte aligned)");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  static bool attr_set[64] = {};
  if (dev->device < 64 && !attr_set[dev->device]) {
    if ((s = check_cuda(cudaFuncSetAttribute(nerf_glu_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGluSmem),
                        "nerf glu smem")) != B2G_OK)
      return s;
    attr_set[dev->device] = true;
  }
  const int64_t grid = 2 * patches < 2 * dev->num_sms ? 2 * patches : 2 * dev->num_sms;
  nerf_glu_kernel<<<static_cast<unsigned>(grid), kGluThreads, kGluSmem, static_cast<cudaStream_t>(stream)>>>(
      params, ldp, norm_scale, x, patches, 1e-6f, dev->err_word);
  note_launch();
  return check_cuda(cudaGetLastError(), "nerf glu launch");
}
