// model.cu — the parts of the denoising step around the transformer blocks that are not GEMMs
// or attention: operand producers of the embedder GEMMs, the approximator's RMSNorm, the NeRF
// decoder's weight preparation and element-wise steps, and its final norm + 3x3 conv + CFG
// blend.  All HBM-bound: one pass over their operands, coalesced rows, no re-reads.
//
//   patchify -> bf16 rows        conv2d_img_in's im2col + linear()'s activation cast
//                                (chroma.cuh:1311-1327, patchify_kernel kernels.cu:975-1019)
//   nerf input -> bf16 rows      nerf_decode steps 1-3's operand: patch pixels [3] + DCT [64],
//                                zero-padded to 72 columns (chroma.cuh:1170-1200)
//   rms_norm rows                rms_norm_cuda (kernels.cu:174-212), F32 or bf16 out
//   nerf glu weights             slice_transpose x3 + l2_norm x3 (chroma.cuh:1264-1281)
//   silu_mul, add                silu_mul_cuda, add_cuda (kernels.cu:368-425)
//   nerf final                   permute + unpatchify + rms_norm_nchw + conv2d_3x3 (chroma.cuh:
//                                1225-1250) for both guidance halves, then cfg_blend (:1581)
#include <cuda_bf16.h>
#include <cstdint>
#include "engine.cuh"

namespace b2g {
namespace {

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// out[patch, c*p*p + py*p + px] = x[c, ph*p + py, pw*p + px] as bf16, two columns per thread.
__global__ void patchify_bf16_kernel(const float* __restrict__ x, int C, int H, int W, int p,
                                     __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int wp = W / p, feat = C * p * p;
  const int64_t total = static_cast<int64_t>(H / p) * wp * (feat / 2);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t patch = i / (feat / 2);
    const int f = static_cast<int>(i % (feat / 2)) * 2;
    const int c = f / (p * p), py = (f % (p * p)) / p, px = f % p;  // px even, px + 1 < p
    const int ih = static_cast<int>(patch / wp) * p + py, iw = static_cast<int>(patch % wp) * p + px;
    const float2 v = *reinterpret_cast<const float2*>(x + (static_cast<int64_t>(c) * H + ih) * W + iw);
    *reinterpret_cast<uint32_t*>(out + patch * ldo + f) = pack_bf16x2(v.x, v.y);
  }
}

// Row patch*256 + pix of the NeRF embedder's input: [x[0..2] at the pixel, dct[pix, 0..63],
// zeros up to ldo].  Two columns per thread.
__global__ void nerf_input_kernel(const float* __restrict__ x, const float* __restrict__ dct, int H, int W,
                                  __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int wp = W / 16;
  const int64_t rows = static_cast<int64_t>(H / 16) * wp * 256;
  const int pairs = static_cast<int>(ldo / 2);
  const int64_t total = rows * pairs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / pairs;
    const int col = static_cast<int>(i % pairs) * 2;
    const int pix = static_cast<int>(r & 255);
    const int64_t patch = r >> 8;
    const int ih = static_cast<int>(patch / wp) * 16 + pix / 16, iw = static_cast<int>(patch % wp) * 16 + pix % 16;
    float v[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int c = col + j;
      if (c < 3) v[j] = x[(static_cast<int64_t>(c) * H + ih) * W + iw];
      else if (c < 67) v[j] = dct[pix * 64 + (c - 3)];
      else v[j] = 0.f;
    }
    *reinterpret_cast<uint32_t*>(out + r * ldo + col) = pack_bf16x2(v[0], v[1]);
  }
}

template <typename T>
__device__ __forceinline__ void store1(T* p, float v);
template <>
__device__ __forceinline__ void store1<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store1<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16(v); }

// RMSNorm of rows of C <= 256 values (C % 64 == 0), one warp per row: out = x * rsqrt(mean(x^2)
// + eps) * scale.
template <typename T>
__global__ void rms_norm_warp_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ scale,
                                     T* __restrict__ out, int64_t ldo, int64_t rows, int C, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float* xr = x + row * ldx;
  float v[8];
  float ss = 0.f;
  const int per = C / 32;  // 2, 4 or 8 values per lane, pairs at lane*2 + 64*j
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (2 * j < per) {
      const float2 t = *reinterpret_cast<const float2*>(xr + 64 * j + 2 * lane);
      v[2 * j] = t.x;
      v[2 * j + 1] = t.y;
      ss += t.x * t.x + t.y * t.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / static_cast<float>(C) + eps);
  T* orow = out + row * ldo;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (2 * j < per) {
      const int c = 64 * j + 2 * lane;
      store1(orow + c, v[2 * j] * r * scale[c]);
      store1(orow + c + 1, v[2 * j + 1] * r * scale[c + 1]);
    }
  }
}

// RMSNorm of long rows (C % 4 == 0), one 256-thread block per row, the row held in registers
// when it fits (C <= 8192), else re-read.
template <typename T>
__global__ void __launch_bounds__(256) rms_norm_block_kernel(const float* __restrict__ x, int64_t ldx,
                                                             const float* __restrict__ scale, T* __restrict__ out,
                                                             int64_t ldo, int C, float eps) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const float* xr = x + row * ldx;
  const int n4 = C / 4;
  float4 keep[8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int i = threadIdx.x + 256 * j;
    if (i < n4) {
      keep[j] = reinterpret_cast<const float4*>(xr)[i];
      ss += keep[j].x * keep[j].x + keep[j].y * keep[j].y + keep[j].z * keep[j].z + keep[j].w * keep[j].w;
    }
  }
  for (int i = threadIdx.x + 256 * 8; i < n4; i += 256) {
    const float4 t = reinterpret_cast<const float4*>(xr)[i];
    ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float r = rsqrtf(tot / static_cast<float>(C) + eps);
  T* orow = out + row * ldo;
  auto emit = [&](int i, const float4 t) {
    const float4 s = reinterpret_cast<const float4*>(scale)[i];
    store1(orow + 4 * i, t.x * r * s.x);
    store1(orow + 4 * i + 1, t.y * r * s.y);
    store1(orow + 4 * i + 2, t.z * r * s.z);
    store1(orow + 4 * i + 3, t.w * r * s.w);
  };
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int i = threadIdx.x + 256 * j;
    if (i < n4) emit(i, keep[j]);
  }
  for (int i = threadIdx.x + 256 * 8; i < n4; i += 256) emit(i, reinterpret_cast<const float4*>(xr)[i]);
}

// The three per-patch weights of one NeRF GLU block from its param_generator output row
// params[b] (3 * 64 * 256 F32): block (b, s) handles slice s.
//   s = 0, 1 (gate, value): slice [64 h][256 m] -> out[b][m][h] / ||slice[., m]||
//   s = 2 (fc2):            slice [256 m][64 h] -> out[b][h][m] / ||slice[., h]||
// with ||.|| the L2 norm floored at eps (l2_norm_kernel).  The slice passes through shared
// memory once; reads and writes are both row-contiguous.
constexpr int kNerfHid = 64, kNerfMlp = 256, kNerfChunk = kNerfHid * kNerfMlp;
// Shared memory of the larger (fc2) layout: [256][65] tile + 256 partial sums.
constexpr int kGluSmemBytes = (kNerfMlp * (kNerfHid + 1) + kNerfMlp) * 4;
static_assert(kNerfHid * (kNerfMlp + 1) + kNerfMlp <= kNerfMlp * (kNerfHid + 1) + kNerfMlp, "gate layout fits");

__global__ void __launch_bounds__(256) nerf_glu_weights_kernel(const float* __restrict__ params, int64_t ldp,
                                                               float* __restrict__ gate, float* __restrict__ value,
                                                               float* __restrict__ fc2, float eps) {
  extern __shared__ float sm[];
  const int64_t b = blockIdx.x;
  const int s = blockIdx.y;
  const float* src = params + b * ldp + static_cast<int64_t>(s) * kNerfChunk;
  const int t = threadIdx.x;
  if (s < 2) {
    float* tile = sm;                      // [64][257]
    float* inv = sm + kNerfHid * (kNerfMlp + 1);
    for (int e = t; e < kNerfChunk; e += 256) tile[(e >> 8) * (kNerfMlp + 1) + (e & 255)] = src[e];
    __syncthreads();
    float ss = 0.f;
    for (int h = 0; h < kNerfHid; ++h) {
      const float v = tile[h * (kNerfMlp + 1) + t];
      ss += v * v;
    }
    const float n = fmaxf(sqrtf(ss), eps);
    inv[t] = 1.0f / n;
    __syncthreads();
    float* dst = (s == 0 ? gate : value) + b * kNerfChunk;
    for (int e = t; e < kNerfChunk; e += 256) {
      const int m = e >> 6, h = e & 63;
      dst[e] = tile[h * (kNerfMlp + 1) + m] * inv[m];
    }
  } else {
    float* tile = sm;                      // [256][65]
    float* part = sm + kNerfMlp * (kNerfHid + 1);  // [4][64] partial sums
    for (int e = t; e < kNerfChunk; e += 256) tile[(e >> 6) * (kNerfHid + 1) + (e & 63)] = src[e];
    __syncthreads();
    const int h = t & 63, q = t >> 6;
    float ss = 0.f;
    for (int m = q * 64; m < q * 64 + 64; ++m) {
      const float v = tile[m * (kNerfHid + 1) + h];
      ss += v * v;
    }
    part[q * 64 + h] = ss;
    __syncthreads();
    if (t < 64) {
      const float tot = part[t] + part[64 + t] + part[128 + t] + part[192 + t];
      part[t] = 1.0f / fmaxf(sqrtf(tot), eps);
    }
    __syncthreads();
    float* dst = fc2 + b * kNerfChunk;
    for (int e = t; e < kNerfChunk; e += 256) {
      const int hh = e >> 8, m = e & 255;
      dst[e] = tile[m * (kNerfHid + 1) + hh] * part[hh];
    }
  }
}

__device__ __forceinline__ float silu_val(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

// a = silu(a) * b, n % 4 == 0, 16-byte aligned.
__global__ void silu_mul_kernel(float* __restrict__ a, const float* __restrict__ b, int64_t n4) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 x = reinterpret_cast<float4*>(a)[i];
    const float4 y = reinterpret_cast<const float4*>(b)[i];
    x.x = silu_val(x.x) * y.x;
    x.y = silu_val(x.y) * y.y;
    x.z = silu_val(x.z) * y.z;
    x.w = silu_val(x.w) * y.w;
    reinterpret_cast<float4*>(a)[i] = x;
  }
}

// x += y, n % 4 == 0, 16-byte aligned.
__global__ void add_inplace_kernel(float* __restrict__ x, const float* __restrict__ y, int64_t n4) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 a = reinterpret_cast<float4*>(x)[i];
    const float4 c = reinterpret_cast<const float4*>(y)[i];
    a.x += c.x;
    a.y += c.y;
    a.z += c.z;
    a.w += c.w;
    reinterpret_cast<float4*>(x)[i] = a;
  }
}

// NeRF final layer (chroma.cuh:1225-1250) and cfg_blend (chroma.cuh:1581) in one kernel: for
// each half z, the decoder state feat_z[patch][pix][64] (patch = (h/16)*(W/16) + w/16,
// pix = (h%16)*16 + w%16) is RMS-normed over its 64 channels (eps, scale), convolved 3x3 to
// 3 channels (zero padding), and the halves blended: out = uncond + cfg * (cond - uncond), or
// cond alone with one half.
//
// A block owns a 16 x 16 pixel tile.  Its 18 x 18 halo cells, normed, sit in shared memory
// channel-major (plane stride kFinPlane, odd, so that the 16 lanes that store one cell's
// channels spread over the banks); the 64 x 27 conv weights sit beside them as [c][28] rows
// read as broadcast float4s.  Loading: each half-warp takes one cell per step (16 lanes x
// float4 = the cell's 64 channels, its sum of squares reduced over the half-warp), with
// kFinUnroll cells' loads in flight before any is used.  Convolution: the 256 threads are two
// groups of 128, one per 32-channel half; a thread computes two vertically adjacent pixels, so
// one channel costs it 12 tile loads and 7 weight loads for 54 FMAs; the second group's sums
// are added through shared memory.  HBM sees the state once (plus the halo rows, mostly L2
// hits) and the 3-channel output once.
constexpr int kFinTile = 16, kFinHalo = kFinTile + 2, kFinCells = kFinHalo * kFinHalo;
constexpr int kFinPlane = kFinCells + 1, kFinThreads = 256, kFinWRow = 28, kFinUnroll = 7;
constexpr int kFinSmem = (64 * kFinPlane + 64 * kFinWRow + 128 * 6) * 4;

__global__ void __launch_bounds__(kFinThreads) nerf_final_kernel(const float* __restrict__ feat0,
                                                                 const float* __restrict__ feat1,
                                                                 const float* __restrict__ scale,
                                                                 const float* __restrict__ wgt,
                                                                 const float* __restrict__ bias, float cfg, int H,
                                                                 int W, float eps, float* __restrict__ out) {
  extern __shared__ float4 fin_smem4[];
  float* tile = reinterpret_cast<float*>(fin_smem4);
  float* ws = tile + 64 * kFinPlane;  // [c][28]: co * 9 + kh * 3 + kw, one pad
  float* red = ws + 64 * kFinWRow;    // [6][128]: the second channel group's sums
  for (int i = threadIdx.x; i < 64 * kFinWRow; i += kFinThreads) {
    const int c = i / kFinWRow, j = i % kFinWRow;
    ws[i] = j < 27 ? wgt[((j / 9) * 64 + c) * 9 + j % 9] : 0.0f;
  }
  const int t = threadIdx.x, hl = t & 15, hw = t >> 4;  // half-warp lane / half-warp index
  const int grp = t >> 7, tt = t & 127;                  // channel group, thread within it
  const int tx = tt & 15, ty = tt >> 4;                  // pixels (2ty, tx) and (2ty + 1, tx)
  const int h0 = blockIdx.y * kFinTile, w0 = blockIdx.x * kFinTile;
  const int PW = W / 16;
  const float4 sc = reinterpret_cast<const float4*>(scale)[hl];
  float res[2][2][3];
  const int halves = feat1 ? 2 : 1;
  for (int z = 0; z < halves; ++z) {
    const float* feat = z ? feat1 : feat0;
    __syncthreads();  // the previous half's reads of the tile are done
    for (int base = hw; base < kFinCells; base += 16 * kFinUnroll) {
      float4 v[kFinUnroll];
#pragma unroll
      for (int u = 0; u < kFinUnroll; ++u) {
        const int cell = base + 16 * u;
        const int ih = h0 - 1 + cell / kFinHalo, iw = w0 - 1 + cell % kFinHalo;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (cell < kFinCells && ih >= 0 && ih < H && iw >= 0 && iw < W) {
          const int64_t patch = static_cast<int64_t>(ih >> 4) * PW + (iw >> 4);
          const int pix = (ih & 15) * 16 + (iw & 15);
          v[u] = __ldg(reinterpret_cast<const float4*>(feat + (patch * 256 + pix) * 64) + hl);
        }
      }
#pragma unroll
      for (int u = 0; u < kFinUnroll; ++u) {
        const int cell = base + 16 * u;
        float ss = v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (cell < kFinCells) {
          // Zero padding: outside cells load as 0 and stay 0 (r is finite for eps > 0).
          const float r = rsqrtf(ss / 64.0f + eps);
          tile[(4 * hl) * kFinPlane + cell] = v[u].x * r * sc.x;
          tile[(4 * hl + 1) * kFinPlane + cell] = v[u].y * r * sc.y;
          tile[(4 * hl + 2) * kFinPlane + cell] = v[u].z * r * sc.z;
          tile[(4 * hl + 3) * kFinPlane + cell] = v[u].w * r * sc.w;
        }
      }
    }
    __syncthreads();
    float acc[2][3];
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int co = 0; co < 3; ++co) acc[p][co] = grp ? 0.0f : bias[co];
#pragma unroll 4
    for (int c = 32 * grp; c < 32 * grp + 32; ++c) {
      const float* tc = tile + c * kFinPlane + (2 * ty) * kFinHalo + tx;
      float v[4][3];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int q = 0; q < 3; ++q) v[r][q] = tc[r * kFinHalo + q];
      const float4* wc = reinterpret_cast<const float4*>(ws + c * kFinWRow);
      float wk[28];
#pragma unroll
      for (int q = 0; q < 7; ++q) {
        const float4 f = wc[q];
        wk[4 * q] = f.x;
        wk[4 * q + 1] = f.y;
        wk[4 * q + 2] = f.z;
        wk[4 * q + 3] = f.w;
      }
#pragma unroll
      for (int p = 0; p < 2; ++p)
#pragma unroll
        for (int kh = 0; kh < 3; ++kh)
#pragma unroll
          for (int kw = 0; kw < 3; ++kw)
#pragma unroll
            for (int co = 0; co < 3; ++co) acc[p][co] += v[p + kh][kw] * wk[co * 9 + kh * 3 + kw];
    }
    if (grp) {
#pragma unroll
      for (int p = 0; p < 2; ++p)
#pragma unroll
        for (int co = 0; co < 3; ++co) red[(p * 3 + co) * 128 + tt] = acc[p][co];
    }
    __syncthreads();
    if (!grp) {
#pragma unroll
      for (int p = 0; p < 2; ++p)
#pragma unroll
        for (int co = 0; co < 3; ++co) res[z][p][co] = acc[p][co] + red[(p * 3 + co) * 128 + tt];
    }
  }
  if (grp) return;
  const int64_t HW = static_cast<int64_t>(H) * W;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int h = h0 + 2 * ty + p, w = w0 + tx;
#pragma unroll
    for (int co = 0; co < 3; ++co) {
      const float v = halves == 2 ? res[1][p][co] + cfg * (res[0][p][co] - res[1][p][co]) : res[0][p][co];
      out[co * HW + static_cast<int64_t>(h) * W + w] = v;
    }
  }
}

unsigned grid_for(int64_t work, int threads) {
  const int64_t b = (work + threads - 1) / threads;
  return static_cast<unsigned>(b < 148 * 32 ? (b < 1 ? 1 : b) : 148 * 32);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

b2g_status launched(const char* what) {
  note_launch();
  return check_cuda(cudaGetLastError(), what);
}

}  // namespace
}  // namespace b2g

using namespace b2g;

extern "C" {

b2g_status b2g_patchify_bf16(const float* x, int C, int H, int W, int p, void* out, int64_t ldo, void* stream) {
  if (!x || !out || C <= 0 || p <= 0 || p % 2 || H % p || W % p || W % 2 || ldo < static_cast<int64_t>(C) * p * p ||
      ldo % 2 || (reinterpret_cast<uintptr_t>(x) & 7u) || (reinterpret_cast<uintptr_t>(out) & 3u))
    return set_error(B2G_ERR_INVALID, "b2g_patchify_bf16: sizes / alignment");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const int64_t work = static_cast<int64_t>(H / p) * (W / p) * C * p * p / 2;
  patchify_bf16_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, C, H, W, p, static_cast<__nv_bfloat16*>(out), ldo);
  return launched("patchify launch");
}

b2g_status b2g_nerf_input_bf16(const float* x, const float* dct, int H, int W, void* out, int64_t ldo, void* stream) {
  if (!x || !dct || !out || H % 16 || W % 16 || ldo < 67 || ldo % 8 || (reinterpret_cast<uintptr_t>(out) & 15u))
    return set_error(B2G_ERR_INVALID, "b2g_nerf_input_bf16: sizes / alignment (ldo >= 67, multiple of 8)");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const int64_t work = static_cast<int64_t>(H / 16) * (W / 16) * 256 * (ldo / 2);
  nerf_input_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, dct, H, W, static_cast<__nv_bfloat16*>(out), ldo);
  return launched("nerf input launch");
}

b2g_status b2g_rms_norm(const float* x, int64_t ldx, const float* scale, void* out, b2g_dtype out_dtype, int64_t ldo,
                        int64_t rows, int64_t C, float eps, void* stream) {
  if (rows <= 0) return B2G_OK;
  if (!x || !scale || !out || C <= 0 || ldx < C || ldo < C || (out_dtype != B2G_F32 && out_dtype != B2G_BF16))
    return set_error(B2G_ERR_INVALID, "b2g_rms_norm: arguments");
  const bool warp_path = C <= 256 && C % 64 == 0;
  if ((!warp_path && C % 4) || !aligned16(x) || !aligned16(scale) || ldx % 4 || (warp_path ? false : ldo % 4))
    return set_error(B2G_ERR_UNSUPPORTED, "b2g_rms_norm: C a multiple of 4 (64 up to 256), 16-byte aligned rows");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (warp_path) {
    const unsigned blocks = static_cast<unsigned>((rows * 32 + 255) / 256);
    if (out_dtype == B2G_F32)
      rms_norm_warp_kernel<float><<<blocks, 256, 0, st>>>(x, ldx, scale, static_cast<float*>(out), ldo, rows,
                                                          static_cast<int>(C), eps);
    else
      rms_norm_warp_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(x, ldx, scale, static_cast<__nv_bfloat16*>(out),
                                                                  ldo, rows, static_cast<int>(C), eps);
  } else {
    if (rows > 0x7fffffff) return set_error(B2G_ERR_UNSUPPORTED, "b2g_rms_norm: too many rows");
    if (out_dtype == B2G_F32)
      rms_norm_block_kernel<float><<<static_cast<unsigned>(rows), 256, 0, st>>>(x, ldx, scale, static_cast<float*>(out),
                                                                                ldo, static_cast<int>(C), eps);
    else
      rms_norm_block_kernel<__nv_bfloat16><<<static_cast<unsigned>(rows), 256, 0, st>>>(
          x, ldx, scale, static_cast<__nv_bfloat16*>(out), ldo, static_cast<int>(C), eps);
  }
  return launched("rms_norm launch");
}

b2g_status b2g_nerf_glu_weights(const float* params, int64_t ldp, int64_t patches, float* gate, float* value,
                                float* fc2, void* stream) {
  if (patches <= 0) return B2G_OK;
  if (!params || !gate || !value || !fc2 || ldp < 3 * kNerfChunk || patches > 0x7fffffff)
    return set_error(B2G_ERR_INVALID, "b2g_nerf_glu_weights: arguments");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  static bool attr_set[64] = {};
  if (dev->device < 64 && !attr_set[dev->device]) {
    if ((s = check_cuda(cudaFuncSetAttribute(nerf_glu_weights_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kGluSmemBytes),
                        "nerf glu weights smem")) != B2G_OK)
      return s;
    attr_set[dev->device] = true;
  }
  nerf_glu_weights_kernel<<<dim3(static_cast<unsigned>(patches), 3), 256, kGluSmemBytes,
                            static_cast<cudaStream_t>(stream)>>>(params, ldp, gate, value, fc2, 1e-12f);
  return launched("nerf glu weights launch");
}

b2g_status b2g_silu_mul(float* a, const float* b, int64_t n, void* stream) {
  if (n <= 0) return B2G_OK;
  if (!a || !b || n % 4 || !aligned16(a) || !aligned16(b)) return set_error(B2G_ERR_INVALID, "b2g_silu_mul");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  silu_mul_kernel<<<grid_for(n / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(a, b, n / 4);
  return launched("silu_mul launch");
}

b2g_status b2g_add_inplace(float* x, const float* y, int64_t n, void* stream) {
  if (n <= 0) return B2G_OK;
  if (!x || !y || n % 4 || !aligned16(x) || !aligned16(y)) return set_error(B2G_ERR_INVALID, "b2g_add_inplace");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  add_inplace_kernel<<<grid_for(n / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n / 4);
  return launched("add launch");
}

b2g_status b2g_nerf_final(const float* feat_cond, const float* feat_uncond, const float* norm_scale,
                          const float* conv_w, const float* conv_b, float cfg_scale, int H, int W, float* out,
                          void* stream) {
  if (!feat_cond || !norm_scale || !conv_w || !conv_b || !out || H % 16 || W % 16 || H <= 0 || W <= 0 ||
      !aligned16(feat_cond) || (feat_uncond && !aligned16(feat_uncond)) || !aligned16(norm_scale))
    return set_error(B2G_ERR_INVALID, "b2g_nerf_final: arguments / alignment");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  static bool attr_set[64] = {};
  if (dev->device < 64 && !attr_set[dev->device]) {
    if ((s = check_cuda(cudaFuncSetAttribute(nerf_final_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kFinSmem),
                        "nerf final smem attribute")) != B2G_OK)
      return s;
    attr_set[dev->device] = true;
  }
  nerf_final_kernel<<<dim3(W / kFinTile, H / kFinTile), kFinThreads, kFinSmem, static_cast<cudaStream_t>(stream)>>>(
      feat_cond, feat_uncond, norm_scale, conv_w, conv_b, cfg_scale, H, W, 1e-6f, out);
  return launched("nerf final launch");
}

}  // extern "C"
