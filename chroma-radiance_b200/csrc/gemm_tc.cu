// gemm_tc.cu — the engine's tensor-core GEMM for sm_100a.
//
//   D[b, m, n] = epilogue( sum_k A[b, m, k] * B[b, n, k] + bias[n] )
//
// A (activations) and B (weights) are K-major bf16 / fp16 (kind::f16) or TF32-rounded fp32
// (kind::tf32) in global memory.  This is the computation of the reference's cuBLASLt call
// in linear_lt (cublas_ops.cuh:214-288: TRANSA=T on W, TRANSB=N on x, fp32 compute, bias
// epilogue), with the elementwise work that the reference runs as separate kernels after
// it (gelu_to_bf16 kernels.cu:297-310, gated_residual kernels.cu:942-968) fused into the
// store.
//
// Two persistent, warp-specialised kernels (320 threads, one CTA per SM):
//   warp 0      TMA producer: STAGES-deep ring of (A tile, B tile) shared-memory stages,
//               128-byte swizzle, guarded by full/empty mbarriers.
//   warp 1      allocates TMEM and issues tcgen05.mma from one thread; tcgen05.commit
//               frees a stage when the MMAs reading it retire and signals a finished
//               accumulator.  Two accumulators, so tile i's epilogue overlaps tile i+1.
//   warps 2-9   epilogue: two warps per TMEM lane quarter (warp w owns lanes 32*(w%4)..,
//               i.e. 32 tile rows), each taking half of the columns; tcgen05.ld 32 columns
//               at a time with the next chunk's load in flight, bias from shared memory,
//               GELU, then a swizzled shared-memory chunk written by one TMA store (or
//               direct stores for the gated residual, which reads D).
//   tc_gemm_kernel       1 CTA  per 128 x BN tile   (BN = 128 or 256), tcgen05 cta_group::1
//   tc_gemm_pair_kernel  2 CTAs per 256 x 256 tile, tcgen05 cta_group::2 (CTA r loads its
//                        own halves of A and B: no multicast anywhere)
// Split-K: a work item is (split, tile); each split stores its fp32 partial in a workspace
// and the split that arrives last on the tile's counter sums them in split order.
// Every wait is bounded (ptx_sm100.cuh): on timeout the kernel records an error word,
// drains its own TMA copies / MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;          // 64 x 2 B = one 128-byte swizzle row (16-bit operands)
constexpr int kThreads = 320;    // producer, MMA, 8 epilogue warps
// kind::tf32 1-CTA kernels add warps that round each landed operand stage to TF32 in shared
// memory (batched_matmul_Bt's fp32 operands): the conversion runs at a quarter of the FP32
// rate, so one warp (one scheduler) cannot keep up with the MMAs; four spread it over all four.
constexpr int kRoundWarps = 4;
template <int KIND>
constexpr int kThreadsK = KIND == 1 ? kThreads + 32 * kRoundWarps : kThreads;
constexpr int kEpiThreads = 256;
constexpr int kEpiWarps = 8;
// K elements per 128-byte stage row: 64 for bf16/fp16 (KIND 0), 32 for tf32 (KIND 1), 128
// for E4M3 (KIND 2, kind::f8f6f4).
template <int KIND>
constexpr int kKElems = KIND == 1 ? 32 : (KIND == 2 ? 128 : 64);
enum { OUT_F32 = 0, OUT_BF16 = 1, OUT_F16 = 2 };

// Output staging: one 4 KB buffer per epilogue warp (32 rows x 32 fp32 or 16-bit columns),
// swizzled like the D tensor map so neither the st.shared nor the TMA store conflicts.
constexpr int kOutBufBytes = 4096;
constexpr int kOutStageBytes = kEpiWarps * kOutBufBytes;  // 32 KB
constexpr int kBiasBytes = 256 * 4;                       // bias of one tile (<= 256 columns)
// E4M3 kernels also stage the tile's per-column weight scales (same size as the bias).
template <int KIND>
constexpr int kScaleBytes = KIND == 2 ? kBiasBytes : 0;

// A launch computes up to kMaxGroups independent problems that share N, K, dtypes and the
// epilogue (the txt and img streams of a double block: same layer shapes, their own rows,
// weights, biases and gates; with classifier-free guidance, each stream's conditional and
// unconditional rows as well).  Their tiles are numbered one group after the other.
constexpr int kMaxGroups = kMaxGemmGroups;

struct TcGroup {
  int M;                   // rows of A and D
  int num_m_blocks;        // tile rows
  int tile0;               // index of the group's first tile
  int vec_ok;              // D base/ldd allow 16-byte vector stores
  void* d;
  long long ldd;
  const void* bias;
  const float* gate;
  const float* a_scale;    // E4M3: per-row scale of A [M]
  const float* b_scale;    // E4M3: per-column scale of B [N]
  long long tp_row0;       // tensor-parallel reduce: first row in the partial/residual buffers
  const float* pe;         // kEpiQkvRope: RoPE table rows of the group's first token [M][64][4]
  const float* qn;         // kEpiQkvRope: RMSNorm scales of q and k heads [128] (NULL: none)
  const float* kn;
  int pe_period;           // kEpiQkvRope: the RoPE row of row m is m % pe_period (0: m)
  int pe_compact;          // kEpiQkvRope: pe rows are [64][2] (cos, sin) instead of [64][4]
};

// Tensor maps of every group (kernel parameter; indexed by group at run time).
struct TcMaps {
  CUtensorMap a[kMaxGroups], b[kMaxGroups], d[kMaxGroups];
};

struct TcParams {
  int N, K, batch;
  int num_n_blocks, num_k_blocks, num_tiles;  // num_tiles: all groups
  int groups;
  int raster_m;            // rasterisation group (m-blocks that share B panels in flight)
  long long d_bstride;
  int bias_kind;           // 0 none, 1 f32, 2 bf16
  int* err;
  uint32_t idesc;
  int a_keep;              // 1: keep A in L2 (evict_last), stream B (evict_first); 0: reverse
  int splits;              // split-K factor S of the split tiles (1 = none)
  int dp_tiles;            // tiles [0, dp_tiles) run whole; tiles [dp_tiles, num_tiles) split S ways
  int num_items;           // dp_tiles + (num_tiles - dp_tiles) * splits
  float* ws;               // split-K partials [slot][split][128][BN] fp32 (slots of the split tiles)
  int* counters;           // split-K arrival counter per slot (zero between launches)
  int tma_store;           // 1: outputs leave through smem staging + TMA bulk tensor stores
  float alpha;             // accumulator scale before the bias (1 for every linear layer)
  // tensor-parallel reduce epilogue (kEpiTpReduce)
  int tp_world, tp_rank;
  void* const* tp_part;    // [world] bf16 partial buffers
  float* const* tp_res;    // [world] F32 residual copies
  long long tp_ld_part, tp_ld_res;
  int* tp_counters;        // rank 0's per-slot arrival counters (epoch counting, never reset)
  int n_outer;             // tiles column-major over all groups' m-blocks (batch 1), see tile_coords
  int hd;                  // kEpiQkvRope: H * 128, the width of each of the q, k, v sections
  int split;               // kEpiQkvRope with a GELU tail: columns >= split (= 3 * hd) are bias +
                           // GELU, stored through the tensor map after the group's (0: no tail)
  float eps;               // kEpiQkvRope: RMSNorm epsilon
  int round_tf32;          // kind::tf32: round each landed stage to TF32 in shared memory first
  TcGroup g[kMaxGroups];
};

__host__ __device__ constexpr size_t smem_bytes(int a_bytes, int b_bytes, int stages, int scale_bytes) {
  return 1024 /* alignment slack */ + static_cast<size_t>(stages) * (a_bytes + b_bytes) + kOutStageBytes + kBiasBytes +
         scale_bytes + 256 /* barriers, TMEM slot, broadcast word */;
}

__device__ __forceinline__ void tile_coords(int tile, const TcParams& p, int& gi, int& bz, int& mb, int& nb) {
  if (p.n_outer) {
    // Column-major over the m-blocks of all groups: the last tiles are the last columns.  The
    // qkv projection uses it so that the final wave holds v tiles, whose epilogue (no norm,
    // no RoPE) is the short one and is not hidden behind a next mainloop.
    int nmb_all = 0;
    for (int i = 0; i < p.groups; ++i) nmb_all += p.g[i].num_m_blocks;
    nb = tile / nmb_all;
    int r = tile - nb * nmb_all;
    gi = 0;
    while (gi + 1 < p.groups && r >= p.g[gi].num_m_blocks) r -= p.g[gi++].num_m_blocks;
    mb = r;
    bz = 0;
    return;
  }
  gi = 0;
  for (int i = 1; i < p.groups; ++i)
    if (tile >= p.g[i].tile0) gi = i;
  const int nmb = p.g[gi].num_m_blocks;
  const int t = tile - p.g[gi].tile0;
  const int per_batch = nmb * p.num_n_blocks;
  bz = t / per_batch;
  int r = t - bz * per_batch;
  // Raster groups of raster_m m-blocks; inside one, m varies fastest, so the CTAs in flight
  // read the same few B panels and the same group of A rows (both stay in L2).
  const int rm = min(p.raster_m, nmb);
  const int group_size = rm * p.num_n_blocks;
  const int g = r / group_size;
  const int first_m = g * rm;
  const int gm = min(nmb - first_m, rm);
  r -= g * group_size;
  mb = first_m + r % gm;
  nb = r / gm;
}

// Rounds one shared-memory operand stage of BYTES (a multiple of 4 KB) to TF32 in place, the
// 32 lanes of a warp striding over it in 16-byte words, eight words per lane in flight at a
// time (one at a time, each load's latency made the rounding 5x slower than the MMAs); the
// values' positions (swizzle) are irrelevant to an elementwise rounding.
template <uint32_t BYTES>
__device__ __forceinline__ void round_stage_tf32(uint8_t* stage, int lane) {
  static_assert(BYTES % 4096 == 0, "whole groups of 8 x 32 words");
  float4* q = reinterpret_cast<float4*>(stage) + lane;
#pragma unroll 1
  for (uint32_t g = 0; g < BYTES / 4096; ++g, q += 256) {
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = q[j * 32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j].x = round_tf32_cvt(v[j].x);
      v[j].y = round_tf32_cvt(v[j].y);
      v[j].z = round_tf32_cvt(v[j].z);
      v[j].w = round_tf32_cvt(v[j].w);
      q[j * 32] = v[j];
    }
  }
}

// Work item -> (tile, split, k-block range).  Items [0, dp_tiles) are whole tiles (split -1);
// the rest cover the split tiles split-major, so the CTAs running at the same time share K
// ranges (and therefore A/B panels in L2).  dp_tiles = 0 is plain split-K over every tile;
// dp_tiles = num_tiles, no split.  A launch whose tiles fill some whole waves plus a partial
// one splits only the partial wave's tiles: their pieces fill the last wave instead of leaving
// most SMs idle through it.
__device__ __forceinline__ void item_coords(int item, const TcParams& p, int& tile, int& split, int& kb0, int& kb1) {
  if (item < p.dp_tiles) {
    tile = item;
    split = -1;
    kb0 = 0;
    kb1 = p.num_k_blocks;
    return;
  }
  const int rest = p.num_tiles - p.dp_tiles;
  const int j = item - p.dp_tiles;
  split = j / rest;
  tile = p.dp_tiles + (j - split * rest);
  kb0 = static_cast<int>(static_cast<long long>(split) * p.num_k_blocks / p.splits);
  kb1 = static_cast<int>(static_cast<long long>(split + 1) * p.num_k_blocks / p.splits);
}

// tanh-form GELU, the formula of the reference's gelu_val (kernels.cu:266-269).
// Evaluated through the identity 0.5 v (1 + tanh(u)) = v * sigmoid(2u) = v / (1 + e^(-2u)),
// with e^(-2u) = 2^(-2u log2(e)) from the hardware base-2 exponential (ex2.approx, relative
// error ~2^-22) and a fast division: a few instructions instead of an accurate tanhf, and
// within a few fp32 ulps of the formula.  The exponent is capped at 2^126 (the quotient is
// then -0 to fp32 precision, GELU's limit for large negative v).
__device__ __forceinline__ float gelu_tanh(float v) {
  const float u = 0.7978845608f * (v + 0.044715f * v * v * v);
  const float e = fast_exp2(fminf(-2.8853900817779268f * u, 126.0f));
  return __fdividef(v, 1.0f + e);
}

// SiLU, the formula of the reference's silu_val (kernels.cu): v / (1 + e^-v), with e^-v from
// the hardware base-2 exponential (capped at 2^126, where the quotient is -0 to fp32
// precision) and a fast division.
__device__ __forceinline__ float silu_fast(float v) {
  return __fdividef(v, 1.0f + fast_exp2(fminf(-1.4426950408889634f * v, 126.0f)));
}

// alpha * acc + bias (bias staged in shared memory, zero past N), then GELU or SiLU if asked.
template <int EPI>
__device__ __forceinline__ void chunk_values(const uint32_t (&r)[32], const float* sb, float alpha, float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (alpha != 1.0f) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= alpha;
  }
  if (sb) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 b = *reinterpret_cast<const float4*>(sb + j);
      v[j] += b.x;
      v[j + 1] += b.y;
      v[j + 2] += b.z;
      v[j + 3] += b.w;
    }
  }
  if constexpr (EPI == B2G_EPI_GELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
  }
  if constexpr (EPI == B2G_EPI_SILU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu_fast(v[j]);
  }
}

template <int OUT>
__device__ __forceinline__ void pack16(const float (&v)[32], uint32_t (&packed)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if constexpr (OUT == OUT_BF16) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      packed[j] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
      packed[j] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
}

// Direct stores of one thread's 32 values of row m, columns [n0, n0+32).
template <int EPI, int OUT>
__device__ __forceinline__ void store_chunk(const TcParams& p, const TcGroup& G, int bz, int m, int n0,
                                            const uint32_t (&r)[32], const float* sb) {
  float v[32];
  chunk_values<EPI>(r, sb, p.alpha, v);
  const bool full = (n0 + 32 <= p.N);
  const int nvalid = full ? 32 : (p.N - n0);
  const long long off = static_cast<long long>(bz) * p.d_bstride + static_cast<long long>(m) * G.ldd + n0;
  if constexpr (OUT == OUT_F32) {
    float* dp = static_cast<float*>(G.d) + off;
    if constexpr (EPI == B2G_EPI_GATED_RESIDUAL) {
      const float* gp = G.gate + n0;
      if (full && G.vec_ok && (reinterpret_cast<uintptr_t>(gp) & 15u) == 0) {
        float4 res[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) res[j] = reinterpret_cast<const float4*>(dp)[j];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 g = __ldg(reinterpret_cast<const float4*>(gp) + j);
          res[j].x += g.x * v[4 * j + 0];
          res[j].y += g.y * v[4 * j + 1];
          res[j].z += g.z * v[4 * j + 2];
          res[j].w += g.w * v[4 * j + 3];
          reinterpret_cast<float4*>(dp)[j] = res[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nvalid) dp[j] = dp[j] + __ldg(gp + j) * v[j];
      }
    } else {
      if (full && G.vec_ok) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          reinterpret_cast<float4*>(dp)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nvalid) dp[j] = v[j];
      }
    }
  } else {
    uint32_t packed[16];
    pack16<OUT>(v, packed);
    uint16_t* dp = static_cast<uint16_t*>(G.d) + off;
    if (full && G.vec_ok) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        reinterpret_cast<uint4*>(dp)[j] =
            make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) dp[j] = static_cast<uint16_t>((j & 1) ? (packed[j >> 1] >> 16) : (packed[j >> 1] & 0xFFFFu));
    }
  }
}

// Stages one 32x32 chunk (this warp's 32 rows x columns [n0, n0+32)) in shared memory and
// writes it with one TMA store; the tensor map clips rows >= M and columns >= N.  The warp's
// 4 KB staging area holds one fp32 chunk or two 16-bit chunks (double-buffered).  Gated
// residual: the chunk holds gate * (acc + bias) and leaves as a TMA reduce-add into the fp32
// residual, so residual + gate * y is formed in L2 (two roundings: the product, then the sum).
template <bool REDUCE, int OUT>
__device__ __forceinline__ void stage_store_values(const CUtensorMap* tmD, uint8_t* stage, int& obuf, int bz,
                                                   int m_warp0, int n0, const float (&v)[32], int lane);

template <int EPI, int OUT>
__device__ __forceinline__ void stage_store_chunk(const CUtensorMap* tmD, uint8_t* stage, int& obuf, int bz,
                                                  int m_warp0, int n0, const uint32_t (&r)[32], const float* sb,
                                                  float alpha, int lane, const float* gate, int N) {
  float v[32];
  chunk_values<EPI>(r, sb, alpha, v);
  if constexpr (EPI == B2G_EPI_GATED_RESIDUAL) {
    const float* gp = gate + n0;
    if (n0 + 32 <= N && (reinterpret_cast<uintptr_t>(gp) & 15u) == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(gp) + j);
        v[4 * j] *= g.x;
        v[4 * j + 1] *= g.y;
        v[4 * j + 2] *= g.z;
        v[4 * j + 3] *= g.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= (n0 + j < N) ? __ldg(gp + j) : 0.f;
    }
  }
  stage_store_values<EPI == B2G_EPI_GATED_RESIDUAL, OUT>(tmD, stage, obuf, bz, m_warp0, n0, v, lane);
}

// The 32x32 chunk of final values `v` (row `lane` of the warp's 32 rows) through the warp's
// staging buffer into one TMA store (REDUCE: TMA reduce-add) at columns n0, rows m_warp0...
template <bool REDUCE, int OUT>
__device__ __forceinline__ void stage_store_values(const CUtensorMap* tmD, uint8_t* stage, int& obuf, int bz,
                                                   int m_warp0, int n0, const float (&v)[32], int lane) {
  uint8_t* buf = stage;
  if constexpr (OUT == OUT_F32) {
    if (lane == 0) bulk_wait_group_read<0>();  // the previous store from this buffer has read it
  } else {
    buf = stage + (obuf & 1) * 2048;
    if (lane == 0) bulk_wait_group_read<1>();  // the store issued from this half two chunks ago
  }
  ++obuf;
  __syncwarp();
  if constexpr (OUT == OUT_F32) {
    // 128-byte rows, 128-byte swizzle: 16-byte chunk j of row `lane` goes to j ^ (lane % 8).
    uint8_t* rowp = buf + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(rowp + ((j ^ (lane & 7)) << 4)) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    uint32_t packed[16];
    pack16<OUT>(v, packed);
    // 64-byte rows, 64-byte swizzle: 16-byte chunk j of row `lane` goes to j ^ ((lane / 2) % 4).
    uint8_t* rowp = buf + lane * 64;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(rowp + ((j ^ ((lane >> 1) & 3)) << 4)) =
          make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if constexpr (REDUCE)
      tma_reduce_add_3d(tmD, buf, n0, m_warp0, bz);
    else
      tma_store_3d(tmD, buf, n0, m_warp0, bz);
    bulk_commit_group();
  }
}

// Writes one finished 32-column chunk: TMA-staged when enabled, else direct stores.
template <int EPI, int OUT>
__device__ __forceinline__ void emit_chunk(const TcParams& p, const TcGroup& G, const CUtensorMap* tmD, uint8_t* buf,
                                           int& obuf, int bz, int m, int m_warp0, int n0, const uint32_t (&r)[32],
                                           const float* sb, int lane) {
  if (p.tma_store) {
    if (m_warp0 < G.M && n0 < p.N)
      stage_store_chunk<EPI, OUT>(tmD, buf, obuf, bz, m_warp0, n0, r, sb, p.alpha, lane, G.gate, p.N);
  } else if (m < G.M && n0 < p.N) {
    store_chunk<EPI, OUT>(p, G, bz, m, n0, r, sb);
  }
}

// Per-CTA epilogue context (shared memory and the warp's place in the tile).
struct EpiCtx {
  uint8_t* buf;            // this warp's staging buffer
  float* sbias;            // tile bias in shared memory (BN floats)
  float* sscale;           // E4M3: tile column scales in shared memory (BN floats)
  volatile int* bcast;     // split-K arrival broadcast word
  int lane, row, q, half;  // row = TMEM lane = tile row; q = lane quarter; half = column half
};

// Loads this item's bias columns [n_base, n_base+BN) into shared memory (zero past N).
template <int BN>
__device__ __forceinline__ void stage_bias(const TcParams& p, const TcGroup& G, float* sbias, int n_base) {
  if (p.bias_kind == 0) return;
  for (int i = static_cast<int>(threadIdx.x) - 64; i < BN; i += kEpiThreads) {
    const int n = n_base + i;
    float b = 0.f;
    if (n < p.N)
      b = p.bias_kind == 1 ? __ldg(static_cast<const float*>(G.bias) + n)
                           : __bfloat162float(static_cast<const __nv_bfloat16*>(G.bias)[n]);
    sbias[i] = b;
  }
}

// E4M3: loads this item's per-column weight scales into shared memory (zero past N).
template <int BN>
__device__ __forceinline__ void stage_scale(const TcParams& p, const TcGroup& G, float* sscale, int n_base) {
  for (int i = static_cast<int>(threadIdx.x) - 64; i < BN; i += kEpiThreads) {
    const int n = n_base + i;
    sscale[i] = n < p.N ? __ldg(G.b_scale + n) : 0.f;
  }
}

// acc * a_scale[row] * b_scale[column] for one 32-column chunk (E4M3 operands).
__device__ __forceinline__ void scale_chunk(uint32_t (&r)[32], float rs, const float* cs) {
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const float4 c = *reinterpret_cast<const float4*>(cs + j);
    r[j] = __float_as_uint(__uint_as_float(r[j]) * rs * c.x);
    r[j + 1] = __float_as_uint(__uint_as_float(r[j + 1]) * rs * c.y);
    r[j + 2] = __float_as_uint(__uint_as_float(r[j + 2]) * rs * c.z);
    r[j + 3] = __float_as_uint(__uint_as_float(r[j + 3]) * rs * c.w);
  }
}

// Tensor-parallel row-split layer: this CTA's part of the tile leaves as a bf16 partial in this
// rank's peer-mapped buffer; the CTA that completes the tile's count on rank 0 (the last of the
// ranks to get there) sums all ranks' partials in rank order, adds the bias, and writes
// residual + gate * sum into every rank's residual copy.  Stores are made visible system-wide
// (__threadfence_system) before the arrival; peer data is read with .cv loads (not cached).
template <int BN, typename Release>
__device__ __forceinline__ void tp_epilogue_item(const TcParams& p, const TcGroup& G, const EpiCtx& e, uint32_t tacc,
                                                 Release release, int m, int n_base, int slot) {
  constexpr int NCH = BN / 64;
  const int c0 = e.half * NCH;
  const bool row_ok = m < G.M;
  const long long prow = G.tp_row0 + m;
  uint16_t* part = static_cast<uint16_t*>(p.tp_part[p.tp_rank]);
  uint32_t r[2][32];
  tmem_ld_32x32b_x32(tacc + c0 * 32, r[0]);
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    tmem_wait_ld();
    if (i + 1 < NCH) tmem_ld_32x32b_x32(tacc + (c0 + i + 1) * 32, r[(i + 1) & 1]);
    if (i == NCH - 1) release();
    const int n0 = n_base + (c0 + i) * 32;
    if (row_ok && n0 < p.N) {
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[i & 1][j]);
      uint32_t packed[16];
      pack16<OUT_BF16>(v, packed);
      uint4* dst = reinterpret_cast<uint4*>(part + prow * p.tp_ld_part + n0);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
    }
  }
  __threadfence_system();
  named_bar_sync(1, kEpiThreads);
  if (threadIdx.x == 64) *e.bcast = atomicAdd_system(p.tp_counters + slot, 1);
  named_bar_sync(1, kEpiThreads);
  const int arrived = *e.bcast;
  if (arrived % p.tp_world == p.tp_world - 1) {
    // This CTA completes the tile: reduce its 128 rows x BN columns cooperatively.  Warp w of
    // the 8 epilogue warps takes rows w, w+8, ..; lane l columns [8l, 8l+8) of the tile, so a
    // warp reads 512 contiguous bytes of each rank's partial row and writes 1 KB of each
    // rank's residual row; four rows' loads are in flight at once.
    __threadfence_system();
    const int et = static_cast<int>(threadIdx.x) - 64;
    const int wq = et >> 5, ln = et & 31;
    const int row_base = m - e.row;                       // first row of this CTA's tile part
    const int ncol = min(BN, p.N - n_base);               // N % 32 == 0
    const bool col_ok = ln * 8 < ncol;
    const int n0 = n_base + ln * 8;
    float bias8[8], gate8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) bias8[j] = 0.f, gate8[j] = 0.f;
    if (col_ok) {
      if (p.bias_kind) {
#pragma unroll
        for (int j = 0; j < 8; ++j) bias8[j] = e.sbias[ln * 8 + j];
      }
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(G.gate + n0));
      const float4 g1 = __ldg(reinterpret_cast<const float4*>(G.gate + n0) + 1);
      gate8[0] = g0.x; gate8[1] = g0.y; gate8[2] = g0.z; gate8[3] = g0.w;
      gate8[4] = g1.x; gate8[5] = g1.y; gate8[6] = g1.z; gate8[7] = g1.w;
    }
    constexpr int kRowsInFlight = 4;
#pragma unroll 1
    for (int r0 = wq; r0 < 128; r0 += 8 * kRowsInFlight) {
      float acc[kRowsInFlight][8];
      float4 rv[kRowsInFlight][2];
      bool ok[kRowsInFlight];
#pragma unroll
      for (int u = 0; u < kRowsInFlight; ++u) {
        const int rr = r0 + u * 8;
        ok[u] = col_ok && rr < 128 && row_base + rr < G.M;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[u][j] = 0.f;
        rv[u][0] = rv[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kRowsInFlight; ++u) {
        if (!ok[u]) continue;
        const long long prow = G.tp_row0 + row_base + r0 + u * 8;
        const float4* res = reinterpret_cast<const float4*>(p.tp_res[p.tp_rank] + prow * p.tp_ld_res + n0);
        rv[u][0] = __ldcv(res);
        rv[u][1] = __ldcv(res + 1);
      }
      for (int q = 0; q < p.tp_world; ++q) {  // fixed rank order: identical sums on every rank
        uint4 pv[kRowsInFlight];
#pragma unroll
        for (int u = 0; u < kRowsInFlight; ++u) {
          const long long prow = G.tp_row0 + row_base + r0 + u * 8;
          if (ok[u])
            pv[u] = __ldcv(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.tp_part[q]) +
                                                          prow * p.tp_ld_part + n0));
        }
#pragma unroll
        for (int u = 0; u < kRowsInFlight; ++u) {
          if (!ok[u]) continue;
          const uint32_t w[4] = {pv[u].x, pv[u].y, pv[u].z, pv[u].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            acc[u][2 * k] += __uint_as_float(w[k] << 16);
            acc[u][2 * k + 1] += __uint_as_float(w[k] & 0xFFFF0000u);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kRowsInFlight; ++u) {
        if (!ok[u]) continue;
        const float4 o0 = make_float4(rv[u][0].x + gate8[0] * (acc[u][0] + bias8[0]),
                                      rv[u][0].y + gate8[1] * (acc[u][1] + bias8[1]),
                                      rv[u][0].z + gate8[2] * (acc[u][2] + bias8[2]),
                                      rv[u][0].w + gate8[3] * (acc[u][3] + bias8[3]));
        const float4 o1 = make_float4(rv[u][1].x + gate8[4] * (acc[u][4] + bias8[4]),
                                      rv[u][1].y + gate8[5] * (acc[u][5] + bias8[5]),
                                      rv[u][1].z + gate8[6] * (acc[u][6] + bias8[6]),
                                      rv[u][1].w + gate8[7] * (acc[u][7] + bias8[7]));
        const long long prow = G.tp_row0 + row_base + r0 + u * 8;
        for (int q = 0; q < p.tp_world; ++q) {
          float4* dst = reinterpret_cast<float4*>(p.tp_res[q] + prow * p.tp_ld_res + n0);
          dst[0] = o0;
          dst[1] = o1;
        }
      }
    }
  }
  named_bar_sync(1, kEpiThreads);  // the broadcast word and staged bias are reused next item
}

// Gated residual: pulls this thread's row of the item's residual columns into L2 before the
// accumulator is ready, so the epilogue's read-modify-write finds it there instead of waiting
// on DRAM once per 32-column chunk.
template <int BN>
__device__ __forceinline__ void prefetch_residual(const TcParams& p, const TcGroup& G, const EpiCtx& e, int bz, int m,
                                                  int n_base) {
  if (m >= G.M) return;
  const int c_begin = n_base + e.half * (BN / 2);
  const float* row = static_cast<const float*>(G.d) + static_cast<long long>(bz) * p.d_bstride +
                     static_cast<long long>(m) * G.ldd;
#pragma unroll
  for (int c = 0; c < BN / 2; c += 32) {  // one 128-byte line per 32 columns
    if (c_begin + c < p.N)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(row + c_begin + c)) : "memory");
  }
}

// Attention input projection (kEpiQkvRope, BN = 256): the tile's columns lie in one of the q,
// k, v sections of [q | k | v] (each H heads of 128) and each thread owns one row of one
// 128-column head.  q and k heads get RMSNorm with their learned scale (rms_norm,
// kernels.cu:174-207, as qk_norm applies it, chroma.cuh:513-515: x * rsqrt(mean(x^2) + eps) *
// w) and RoPE from the table row of the token (apply_rope_fused_bf16, rope.cuh:180-221: pair
// (x0, x1) -> (x0 c0 + x1 c1, x0 c2 + x1 c3) with the row's (cos, -sin, sin, cos) group); v
// passes through.  Everything leaves as bf16 through the TMA store path: the attention kernel
// reads its operands from this buffer, so the fp32 projection never goes to memory.
// Pass 1 reads the head's 128 accumulator columns from TMEM for the sum of squares, pass 2
// reads them again and writes the result.  With a GELU tail (the single block's linear1: its
// weight rows are [q | k | v | mlp]), 128-column halves at or past p.split take bias + GELU
// and leave through the tensor map that follows tmD (the launch then has one group).  With
// E4M3 operands (KIND 2) every accumulator chunk is first scaled by the row's activation scale
// and the columns' weight scales, as in the other epilogues.
template <int BN, int KIND, typename Release>
__device__ __forceinline__ void qkv_rope_item(const TcParams& p, const TcGroup& G, const EpiCtx& e, int& obuf,
                                              uint32_t tacc, Release release, const CUtensorMap* tmD, int m,
                                              int n_base) {
  static_assert(BN == 256, "one 128-column head per thread");
  const int c0 = e.half * 4;           // this warp's first 32-column chunk in the tile
  const int col = n_base + c0 * 32;    // first column of the head (uniform across the warp)
  const int m_warp0 = m - e.lane;
  float rs = 0.f;                      // E4M3: this row's activation scale
  if constexpr (KIND == 2) rs = m < G.M ? __ldg(G.a_scale + m) : 0.f;
  if (p.split && col >= p.split) {
    const float* sbg = p.bias_kind ? e.sbias + c0 * 32 : nullptr;
    uint32_t r[2][32];
    tmem_ld_32x32b_x32(tacc + c0 * 32, r[0]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      tmem_wait_ld();
      if (i + 1 < 4) tmem_ld_32x32b_x32(tacc + (c0 + i + 1) * 32, r[(i + 1) & 1]);
      if (i == 3) release();
      if constexpr (KIND == 2) scale_chunk(r[i & 1], rs, e.sscale + (c0 + i) * 32);
      float v[32];
      chunk_values<B2G_EPI_GELU>(r[i & 1], sbg ? sbg + i * 32 : nullptr, p.alpha, v);
      if (m_warp0 < G.M && col + i * 32 < p.N)
        stage_store_values<false, OUT_BF16>(tmD + 1, e.buf, obuf, 0, m_warp0, col - p.split + i * 32, v, e.lane);
    }
    named_bar_sync(1, kEpiThreads);  // the staged bias is reused next item
    return;
  }
  const int sec = col / p.hd;          // 0 q, 1 k, 2 v
  const float* norm = sec == 0 ? G.qn : (sec == 1 ? G.kn : nullptr);
  const float* sb = p.bias_kind ? e.sbias + c0 * 32 : nullptr;
  float inv = 1.f;
  if (norm) {
    float ss = 0.f;
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      uint32_t r[32];
      float v[32];
      tmem_ld_32x32b_x32(tacc + (c0 + i) * 32, r);
      tmem_wait_ld();
      if constexpr (KIND == 2) scale_chunk(r, rs, e.sscale + (c0 + i) * 32);
      chunk_values<B2G_EPI_NONE>(r, sb ? sb + i * 32 : nullptr, p.alpha, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) ss += v[j] * v[j];
    }
    inv = rsqrtf(ss / 128.0f + p.eps);
  }
  // The table row of the token: [64][4] (c0, c1, c2, c3) per pair, or compact [64][2] (cos, sin)
  // for the rotation form (cos, -sin, sin, cos), half the bytes (the reads compete with the
  // L2-bound mainloop for L2 bandwidth).  Both forms go through the same roundings:
  // x0' = fma(x0, c0, x1 * c1), x1' = fma(x0, c2, x1 * c3).
  const int pe_m = m < G.M ? m : G.M - 1;
  const bool compact = G.pe_compact != 0;
  const float4* pe_row = reinterpret_cast<const float4*>(G.pe) +
                         static_cast<long long>(G.pe_period ? pe_m % G.pe_period : pe_m) * (compact ? 32 : 64);
  uint32_t r[2][32];
  tmem_ld_32x32b_x32(tacc + c0 * 32, r[0]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    tmem_wait_ld();
    if (i + 1 < 4) tmem_ld_32x32b_x32(tacc + (c0 + i + 1) * 32, r[(i + 1) & 1]);
    if (i == 3) release();
    if constexpr (KIND == 2) scale_chunk(r[i & 1], rs, e.sscale + (c0 + i) * 32);
    float v[32];
    chunk_values<B2G_EPI_NONE>(r[i & 1], sb ? sb + i * 32 : nullptr, p.alpha, v);
    if (sec < 2) {
      if (norm) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 w = __ldg(reinterpret_cast<const float4*>(norm + i * 32 + j));
          v[j] = v[j] * inv * w.x;
          v[j + 1] = v[j + 1] * inv * w.y;
          v[j + 2] = v[j + 2] * inv * w.z;
          v[j + 3] = v[j + 3] * inv * w.w;
        }
      }
      if (compact) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // pairs i*16 + 2j and 2j + 1 of the head
          const float4 cs = __ldg(pe_row + i * 8 + j);
          float x0 = v[4 * j], x1 = v[4 * j + 1];
          v[4 * j] = __fmaf_rn(x0, cs.x, __fmul_rn(x1, -cs.y));
          v[4 * j + 1] = __fmaf_rn(x0, cs.y, __fmul_rn(x1, cs.x));
          x0 = v[4 * j + 2];
          x1 = v[4 * j + 3];
          v[4 * j + 2] = __fmaf_rn(x0, cs.z, __fmul_rn(x1, -cs.w));
          v[4 * j + 3] = __fmaf_rn(x0, cs.w, __fmul_rn(x1, cs.z));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {  // pair i*16 + j of the head
          const float4 c = __ldg(pe_row + i * 16 + j);
          const float x0 = v[2 * j], x1 = v[2 * j + 1];
          v[2 * j] = __fmaf_rn(x0, c.x, __fmul_rn(x1, c.y));
          v[2 * j + 1] = __fmaf_rn(x0, c.z, __fmul_rn(x1, c.w));
        }
      }
    }
    if (m_warp0 < G.M && col < p.N) stage_store_values<false, OUT_BF16>(tmD, e.buf, obuf, 0, m_warp0, col + i * 32, v,
                                                                       e.lane);
  }
  named_bar_sync(1, kEpiThreads);  // the staged bias is reused next item
}

// Epilogue of one work item by the 8 epilogue warps of a CTA.  `tacc` addresses the
// accumulator's column 0 at this warp's lane quarter; `release()` hands the accumulator back
// after this warp's last chunk is read.  For a piece of a split tile (split >= 0), each split
// stores its raw fp32 partial; the split arriving last on the slot's counter sums all partials
// in split order (deterministic), runs the epilogue and re-arms the counter for the next
// launch.  `slot` numbers the split tiles' CTA-tiles (and, for the TP epilogue, every tile's).
template <int BN, int EPI, int OUT, int KIND, typename Release>
__device__ __forceinline__ void epilogue_item(const TcParams& p, const TcGroup& G, const EpiCtx& e, int& obuf,
                                              uint32_t tacc, Release release, const CUtensorMap* tmD, int bz, int m,
                                              int n_base, int slot, int split) {
  if constexpr (EPI == kEpiTpReduce) {
    tp_epilogue_item<BN>(p, G, e, tacc, release, m, n_base, slot);
    return;
  } else if constexpr (EPI == kEpiQkvRope) {
    if constexpr (BN == 256) qkv_rope_item<BN, KIND>(p, G, e, obuf, tacc, release, tmD, m, n_base);
    return;
  }
  float rs = 0.f;  // E4M3: this row's activation scale
  if constexpr (KIND == 2) rs = m < G.M ? __ldg(G.a_scale + m) : 0.f;
  constexpr int NCH = BN / 64;  // 32-column chunks per warp (half of the tile's columns)
  const int c0 = e.half * NCH;
  const int m_warp0 = m - e.lane;
  const float* sb = p.bias_kind ? e.sbias : nullptr;
  const bool splitk = split >= 0 && p.splits > 1;
  // Split-K partials: one 128 x BN fp32 block per (slot, split), stored so that a warp's 32
  // rows of one 4-column group are 32 consecutive 16-byte words (float4 index
  // (chunk * 8 + j) * 128 + row): every store and fixup load of a warp is one coalesced 512 bytes.
  float4* part = splitk ? reinterpret_cast<float4*>(p.ws + (static_cast<size_t>(slot) * p.splits + split) * 128 * BN)
                        : nullptr;
  uint32_t r[2][32];
  tmem_ld_32x32b_x32(tacc + c0 * 32, r[0]);
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    tmem_wait_ld();
    if (i + 1 < NCH) tmem_ld_32x32b_x32(tacc + (c0 + i + 1) * 32, r[(i + 1) & 1]);  // next chunk in flight
    if (i == NCH - 1) release();
    const int c = c0 + i;
    if (!splitk) {
      if constexpr (KIND == 2) scale_chunk(r[i & 1], rs, e.sscale + c * 32);
      emit_chunk<EPI, OUT>(p, G, tmD, e.buf, obuf, bz, m, m_warp0, n_base + c * 32, r[i & 1],
                           sb ? sb + c * 32 : nullptr, e.lane);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        part[(c * 8 + j) * 128 + e.row] =
            make_float4(__uint_as_float(r[i & 1][4 * j]), __uint_as_float(r[i & 1][4 * j + 1]),
                        __uint_as_float(r[i & 1][4 * j + 2]), __uint_as_float(r[i & 1][4 * j + 3]));
    }
  }
  if (splitk) {
    __threadfence();
    named_bar_sync(1, kEpiThreads);
    if (threadIdx.x == 64) *e.bcast = atomicAdd(p.counters + slot, 1);
    named_bar_sync(1, kEpiThreads);
    if (*e.bcast == p.splits - 1) {
      __threadfence();
      const float4* base = reinterpret_cast<const float4*>(p.ws + static_cast<size_t>(slot) * p.splits * 128 * BN);
#pragma unroll 1
      for (int i = 0; i < NCH; ++i) {
        const int c = c0 + i;
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = 0.f;
        for (int sp = 0; sp < p.splits; ++sp) {
          const float4* src = base + static_cast<size_t>(sp) * 32 * BN;  // 128 * BN floats per split
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 v = __ldcg(src + (c * 8 + j) * 128 + e.row);
            acc[4 * j] += v.x;
            acc[4 * j + 1] += v.y;
            acc[4 * j + 2] += v.z;
            acc[4 * j + 3] += v.w;
          }
        }
        uint32_t rr[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) rr[j] = __float_as_uint(acc[j]);
        if constexpr (KIND == 2) scale_chunk(rr, rs, e.sscale + c * 32);
        emit_chunk<EPI, OUT>(p, G, tmD, e.buf, obuf, bz, m, m_warp0, n_base + c * 32, rr,
                             sb ? sb + c * 32 : nullptr, e.lane);
      }
      if (threadIdx.x == 64) p.counters[slot] = 0;
    }
  }
  named_bar_sync(1, kEpiThreads);  // shared bias and the broadcast word are reused next item
}

// ---------------------------------------------------------------------------- 1-CTA kernel
template <int BN, int STAGES, int EPI, int OUT, int KIND>
__global__ void __launch_bounds__(kThreadsK<KIND>, 1)
    tc_gemm_kernel(const __grid_constant__ TcMaps maps, const __grid_constant__ TcParams p) {
  constexpr uint32_t A_BYTES = kBM * kBK * 2;
  constexpr uint32_t B_BYTES = BN * kBK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators; 256 or 512 (power of two)
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sOut = sB + STAGES * B_BYTES;
  float* sBias = reinterpret_cast<float*>(sOut + kOutStageBytes);
  float* sScale = reinterpret_cast<float*>(sOut + kOutStageBytes + kBiasBytes);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sOut + kOutStageBytes + kBiasBytes + kScaleBytes<KIND>);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* rnd_bar = drain_bar + 1;  // kind::tf32 with round_tf32: stage s rounded (kRoundWarps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rnd_bar + STAGES);
  volatile int* bcast = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  bool round_stages = false;
  if constexpr (KIND == 1) round_stages = p.round_tf32 != 0;
  uint64_t* ready_bar = round_stages ? rnd_bar : full_bar;  // what the MMA waits for per stage

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      if (round_stages) mbar_init(&rnd_bar[s], kRoundWarps);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
    for (int gi = 0; gi < p.groups; ++gi) {
      tma_prefetch_desc(&maps.a[gi]);
      tma_prefetch_desc(&maps.b[gi]);
      if (p.tma_store) tma_prefetch_desc(&maps.d[gi]);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // the set-up above overlapped the previous kernel's tail
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      const uint64_t stream = policy_evict_first();
      const uint64_t pa = p.a_keep ? keep : stream;
      const uint64_t pb = p.a_keep ? stream : keep;
      int stage = 0;
      uint32_t phase = 0, issued = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < p.num_items && ok; item += gridDim.x) {
        int tile, split, kb0, kb1, gi, bz, mb, nb;
        item_coords(item, p, tile, split, kb0, kb1);
        tile_coords(tile, p, gi, bz, mb, nb);
        const CUtensorMap* tmA = &maps.a[gi];
        const CUtensorMap* tmB = &maps.b[gi];
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], A_BYTES + B_BYTES);
          tma_load_3d(sA + stage * A_BYTES, tmA, &full_bar[stage], kb * kKElems<KIND>, mb * kBM, bz, pa);
          tma_load_3d(sB + stage * B_BYTES, tmB, &full_bar[stage], kb * kKElems<KIND>, nb * BN, bz, pb);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let the copies this thread started land before the CTA's smem goes away.
        const uint32_t n = issued < static_cast<uint32_t>(STAGES) ? issued : static_cast<uint32_t>(STAGES);
        for (uint32_t k = issued - n; k < issued; ++k) mbar_wait_drain(&full_bar[k % STAGES], (k / STAGES) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, local = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < p.num_items && ok; item += gridDim.x, ++local) {
        int tile, split, kb0, kb1;
        item_coords(item, p, tile, split, kb0, kb1);
        const uint32_t acc = local & 1u;
        const uint32_t acc_phase = (local >> 1) & 1u;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, p.err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&ready_bar[stage], phase, p.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // One MMA consumes 32 bytes of K (16 bf16/fp16, 8 tf32 or 32 E4M3 elements) inside the
            // 128-byte swizzle row: advance the descriptors by 32 bytes.
            const uint64_t ad = smem_desc_k_sw128(a0 + k * 32), bd = smem_desc_k_sw128(b0 + k * 32);
            const uint32_t accum = (kb != kb0 || k != 0) ? 1u : 0u;
            if constexpr (KIND == 1) umma_tf32(d_tmem, ad, bd, p.idesc, accum);
            else if constexpr (KIND == 2) umma_f8(d_tmem, ad, bd, p.idesc, accum);
            else umma_f16(d_tmem, ad, bd, p.idesc, accum);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
      if (!ok) {
        // MMAs already issued must retire before TMEM is released.
        umma_commit(drain_bar);
        mbar_wait_drain(drain_bar, 0);
      }
    }
  } else if (warp >= 2 + kEpiWarps) {
    // ------------------------------------------------------------ TF32 rounders (warps 10..13)
    // Every landed stage is rounded to TF32 in place, each warp a quarter of A and of B; the
    // warp's shared-memory writes are made visible to the tensor core (proxy fence) before its
    // arrival on the stage's rounded barrier, which the MMA issuer waits for.
    if (round_stages) {
      const int r = warp - 2 - kEpiWarps;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < p.num_items && ok; item += gridDim.x) {
        int tile, split, kb0, kb1;
        item_coords(item, p, tile, split, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          ok = __all_sync(0xffffffffu, mbar_wait(&full_bar[stage], phase, p.err, kErrWaitMma));
          if (!ok) break;
          round_stage_tf32<A_BYTES / kRoundWarps>(sA + stage * A_BYTES + r * (A_BYTES / kRoundWarps), lane);
          round_stage_tf32<B_BYTES / kRoundWarps>(sB + stage * B_BYTES + r * (B_BYTES / kRoundWarps), lane);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&rnd_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    EpiCtx e;
    e.lane = lane;
    e.q = warp & 3;  // TMEM lane quarter this warp may access
    e.half = (warp - 2) >> 2;
    e.row = e.q * 32 + lane;
    e.buf = sOut + (warp - 2) * kOutBufBytes;
    e.sbias = sBias;
    e.sscale = sScale;
    e.bcast = bcast;
    int obuf = 0;
    uint32_t local = 0;
    for (int item = blockIdx.x; item < p.num_items; item += gridDim.x, ++local) {
      int tile, split, kb0, kb1, gi, bz, mb, nb;
      item_coords(item, p, tile, split, kb0, kb1);
      tile_coords(tile, p, gi, bz, mb, nb);
      const TcGroup& G = p.g[gi];
      if constexpr (EPI == B2G_EPI_GATED_RESIDUAL) prefetch_residual<BN>(p, G, e, bz, mb * kBM + e.row, nb * BN);
      stage_bias<BN>(p, G, sBias, nb * BN);
      if constexpr (KIND == 2) stage_scale<BN>(p, G, sScale, nb * BN);
      const uint32_t acc = local & 1u;
      const uint32_t acc_phase = (local >> 1) & 1u;
      const bool ok = mbar_wait(&tfull_bar[acc], acc_phase, p.err, kErrWaitEpilogue);
      if (!named_bar_all(1, kEpiThreads, ok)) break;  // also publishes the staged bias
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(e.q * 32) << 16) + acc * BN;
      auto release = [&] {
        // This warp's part of the accumulator is read: hand it back to the MMA warp.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      };
      epilogue_item<BN, EPI, OUT, KIND>(p, G, e, obuf, tacc, release, &maps.d[gi], bz, mb * kBM + e.row, nb * BN,
                                        split >= 0 ? tile - p.dp_tiles : tile, split);
    }
    if (lane == 0) bulk_wait_group_all();  // staged stores done before the CTA's smem goes away
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- 2-CTA kernel
//
// A cluster of two CTAs (on two SMs) computes one 256x256 output tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16).  CTA r of the pair loads rows
// [m0 + 128r, +128) of A and rows [n0 + 128r, +128) of B into its own shared memory; the
// MMA, issued by CTA 0, reads both halves and leaves rows [m0 + 128r, +128) x 256 columns
// of the accumulator in CTA r's TMEM.  Per SM this moves 32 KB of operands per 64-wide
// k-block instead of 48 KB for a 1-CTA 128x256 tile with the same MMA time.
//   full[s]   (CTA 0 only)  both CTAs' TMA bytes for stage s; CTA 0 arms it for 64 KB.
//   empty[s]  (each CTA)    the pair's MMAs reading stage s have retired (broadcast commit).
//   tfull[a]  (each CTA)    accumulator a is complete (broadcast commit).
//   tempty[a] (CTA 0 only)  all 16 epilogue warps of the pair have read accumulator a.
template <int STAGES, int EPI, int OUT, int KIND>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    tc_gemm_pair_kernel(const __grid_constant__ TcMaps maps, const __grid_constant__ TcParams p) {
  constexpr int BN = 256;
  constexpr uint32_t A_BYTES = kBM * kBK * 2;  // this CTA's 128 rows of A
  constexpr uint32_t B_BYTES = 128 * kBK * 2;  // this CTA's 128 rows of B
  constexpr uint32_t TMEM_COLS = 512;          // two 128-lane x 256-column accumulators

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sOut = sB + STAGES * B_BYTES;
  float* sBias = reinterpret_cast<float*>(sOut + kOutStageBytes);
  float* sScale = reinterpret_cast<float*>(sOut + kOutStageBytes + kBiasBytes);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sOut + kOutStageBytes + kBiasBytes + kScaleBytes<KIND>);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* bcast = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = static_cast<int>(cluster_id_x());
  const int nclusters = static_cast<int>(num_clusters_x());

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * kEpiWarps);  // epilogue warps of both CTAs
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
    for (int gi = 0; gi < p.groups; ++gi) {
      tma_prefetch_desc(&maps.a[gi]);
      tma_prefetch_desc(&maps.b[gi]);
      if (p.tma_store) tma_prefetch_desc(&maps.d[gi]);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barrier inits and the TMEM allocation are visible pair-wide
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // the set-up above overlapped the previous kernel's tail
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      const uint64_t stream = policy_evict_first();
      const uint64_t pa = p.a_keep ? keep : stream;
      const uint64_t pb = p.a_keep ? stream : keep;
      int stage = 0;
      uint32_t phase = 0, issued = 0;
      bool ok = true;
      for (int item = cluster; item < p.num_items && ok; item += nclusters) {
        int tile, split, kb0, kb1, gi, bz, mb, nb;
        item_coords(item, p, tile, split, kb0, kb1);
        tile_coords(tile, p, gi, bz, mb, nb);
        const CUtensorMap* tmA = &maps.a[gi];
        const CUtensorMap* tmB = &maps.b[gi];
        const int arow = mb * 256 + static_cast<int>(rank) * 128;
        const int brow = nb * BN + static_cast<int>(rank) * 128;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * (A_BYTES + B_BYTES));
          const uint32_t leader_full = map_to_cta(smem_u32(&full_bar[stage]), 0);
          tma_load_3d_pair(sA + stage * A_BYTES, tmA, leader_full, kb * kKElems<KIND>, arow, bz, pa);
          tma_load_3d_pair(sB + stage * B_BYTES, tmB, leader_full, kb * kKElems<KIND>, brow, bz, pb);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && rank == 0) {
        const uint32_t n = issued < static_cast<uint32_t>(STAGES) ? issued : static_cast<uint32_t>(STAGES);
        for (uint32_t k = issued - n; k < issued; ++k) mbar_wait_drain(&full_bar[k % STAGES], (k / STAGES) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (CTA 0 only)
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = p.idesc;  // M=256, N=256
      int stage = 0;
      uint32_t phase = 0, local = 0;
      bool ok = true;
      for (int item = cluster; item < p.num_items && ok; item += nclusters, ++local) {
        int tile, split, kb0, kb1;
        item_coords(item, p, tile, split, kb0, kb1);
        const uint32_t acc = local & 1u;
        const uint32_t acc_phase = (local >> 1) & 1u;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, p.err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, p.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = smem_desc_k_sw128(a0 + k * 32), bd = smem_desc_k_sw128(b0 + k * 32);
            const uint32_t accum = (kb != kb0 || k != 0) ? 1u : 0u;
            if constexpr (KIND == 1) umma_tf32_pair(d_tmem, ad, bd, idesc, accum);
            else if constexpr (KIND == 2) umma_f8_pair(d_tmem, ad, bd, idesc, accum);
            else umma_f16_pair(d_tmem, ad, bd, idesc, accum);
          }
          umma_commit_pair_bcast(&empty_bar[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit_pair_bcast(&tfull_bar[acc], 0x3);
      }
      if (!ok) {
        umma_commit_pair(drain_bar);
        mbar_wait_drain(drain_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9, both CTAs)
    EpiCtx e;
    e.lane = lane;
    e.q = warp & 3;
    e.half = (warp - 2) >> 2;
    e.row = e.q * 32 + lane;
    e.buf = sOut + (warp - 2) * kOutBufBytes;
    e.sbias = sBias;
    e.sscale = sScale;
    e.bcast = bcast;
    const uint32_t leader_tempty0 = map_to_cta(smem_u32(&tempty_bar[0]), 0);
    const uint32_t leader_tempty1 = map_to_cta(smem_u32(&tempty_bar[1]), 0);
    int obuf = 0;
    uint32_t local = 0;
    for (int item = cluster; item < p.num_items; item += nclusters, ++local) {
      int tile, split, kb0, kb1, gi, bz, mb, nb;
      item_coords(item, p, tile, split, kb0, kb1);
      tile_coords(tile, p, gi, bz, mb, nb);
      const TcGroup& G = p.g[gi];
      if constexpr (EPI == B2G_EPI_GATED_RESIDUAL)
        prefetch_residual<BN>(p, G, e, bz, mb * 256 + static_cast<int>(rank) * 128 + e.row, nb * BN);
      stage_bias<BN>(p, G, sBias, nb * BN);
      if constexpr (KIND == 2) stage_scale<BN>(p, G, sScale, nb * BN);
      const uint32_t acc = local & 1u;
      const uint32_t acc_phase = (local >> 1) & 1u;
      const bool ok = mbar_wait(&tfull_bar[acc], acc_phase, p.err, kErrWaitEpilogue);
      if (!named_bar_all(1, kEpiThreads, ok)) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(e.q * 32) << 16) + acc * BN;
      auto release = [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
      };
      epilogue_item<BN, EPI, OUT, KIND>(p, G, e, obuf, tacc, release, &maps.d[gi], bz,
                                  mb * 256 + static_cast<int>(rank) * 128 + e.row, nb * BN,
                                  (split >= 0 ? tile - p.dp_tiles : tile) * 2 + static_cast<int>(rank), split);
    }
    if (lane == 0) bulk_wait_group_all();
  }

  // Neither CTA may leave (or free TMEM) while its peer can still touch its shared memory
  // or barriers: every role has finished, then both CTAs release the pair's TMEM.
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- host side

// Time per 64-wide k-block of one work item relative to a 2-CTA 256x256 pair tile, from the
// sustained rates measured on B200 at the linear1 shape (pair 1469, 128x256 1247, 128x128
// 913 TFLOP/s): a 128x128 tile on one SM takes 0.805 of a pair k-block, a 128x256 tile 1.178.
constexpr double kCost128 = 0.805;
constexpr double kCost256 = 1.178;
constexpr double kCostPair = 1.0;
// Fixed split-K overhead in pair-k-block units (partial store, arrival, last-split reduce).
// Measured: the reduction is latency-bound and rarely pays, so automatic selection only
// splits when it removes at least this much time.
constexpr double kSplitOverhead = 24.0;
// A launch that splits only the tiles of its last, partial wave (their pieces fill that wave):
// a fixed cost plus one per split (each piece stores a 128 x BN fp32 partial; the last sums
// them all), fitted to B200 timings of such launches at S = 2, 4, 8.
constexpr double kTailFixed = 17.0;
constexpr double kTailPerSplit = 5.0;
// Shared-memory ring depth (6 x 32 KB measured slightly faster than 7 on B200).
constexpr int kPairStages = 6;
constexpr int kStages128 = 6;
constexpr int kStages256 = 4;  // 4 x 48 KB
int g_force_variant = -1;  // -1 auto, 0 = 1-CTA 128, 1 = 1-CTA 256, 2 = 2-CTA pair
int g_force_splits = 0;    // 0 auto, > 0 split-K factor of every tile, < 0 split factor of the last wave's tiles
bool g_allow_pair = true;
int g_tma_store = -1;      // stage outputs through smem and TMA stores (B2G_TMA_STORE=0 disables)

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

b2g_status get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return set_error(B2G_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  return B2G_OK;
}

}  // namespace

// 3-D K-major operand map: dims {K, rows, batch}, box {128 bytes of K, box_rows, 1}, 128-byte
// swizzle, out-of-bounds elements read as zero (so ragged M, N and K tiles need no special case).
b2g_status make_operand_map(CUtensorMap* map, const void* base, b2g_dtype dt, int64_t K, int64_t rows,
                            int64_t ld, int64_t batch, int64_t bstride, uint32_t box_rows) {
  b2g_status s = get_encode();
  if (s != B2G_OK) return s;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(batch)};
  const cuuint64_t esz = dt == B2G_F32 ? 4u : (dt == B2G_E4M3 ? 1u : 2u);
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * esz, static_cast<cuuint64_t>(bstride) * esz};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / esz), box_rows, 1u};  // 128-byte rows
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType t = dt == B2G_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                : dt == B2G_F16  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                : dt == B2G_E4M3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = g_encode(map, t, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(B2G_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return B2G_OK;
}

namespace {

// 3-D output map: dims {N, M, batch}, box {32, 32, 1} (one epilogue warp's chunk), swizzle
// matching the staging layout (128 B for fp32 rows, 64 B for 16-bit rows).
b2g_status make_output_map(CUtensorMap* map, void* base, b2g_dtype dt, int64_t N, int64_t M, int64_t ld,
                           int64_t batch, int64_t bstride) {
  const cuuint64_t esz = dt == B2G_F32 ? 4u : 2u;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * esz, static_cast<cuuint64_t>(bstride) * esz};
  const cuuint32_t box[3] = {32u, 32u, 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType t = dt == B2G_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                : dt == B2G_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUtensorMapSwizzle sw = esz == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = g_encode(map, t, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(B2G_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (" + std::to_string(r) + ")");
  return B2G_OK;
}

template <typename Kern>
b2g_status launch_kernel(Kern kern, size_t smem, const TcMaps& maps, const TcParams& prm, int grid, int threads,
                         cudaStream_t st) {
  b2g_status s = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "cudaFuncSetAttribute(tc_gemm)");
  if (s != B2G_OK) return s;
  return launch_pdl(kern, dim3(grid), dim3(threads), smem, st, "tc_gemm launch", maps, prm);
}

// Variant selector: PAIR = 2-CTA 256x256 kernel, else 1-CTA 128xBN kernel.
template <bool PAIR, int BN, int STAGES, int EPI, int OUT, int KIND>
b2g_status launch_one(const TcMaps& maps, const TcParams& prm, int grid, cudaStream_t st) {
  if constexpr (PAIR) {
    constexpr size_t smem = smem_bytes(kBM * kBK * 2, 128 * kBK * 2, STAGES, kScaleBytes<KIND>);
    static_assert(smem <= 227 * 1024, "shared memory budget");
    return launch_kernel(tc_gemm_pair_kernel<STAGES, EPI, OUT, KIND>, smem, maps, prm, grid, kThreads, st);
  } else {
    constexpr size_t smem = smem_bytes(kBM * kBK * 2, BN * kBK * 2, STAGES, kScaleBytes<KIND>);
    static_assert(smem <= 227 * 1024, "shared memory budget");
    return launch_kernel(tc_gemm_kernel<BN, STAGES, EPI, OUT, KIND>, smem, maps, prm, grid, kThreadsK<KIND>, st);
  }
}

// Epilogue and output-type dispatch for 16-bit (KIND 0) and E4M3 (KIND 2) operands.
template <bool PAIR, int BN, int STAGES, int KIND>
b2g_status dispatch_out(const TcMaps& maps, const TcParams& prm, int grid, b2g_epilogue epi, b2g_dtype out,
                        cudaStream_t st) {
  if constexpr (KIND == 0) {
    if (static_cast<int>(epi) == kEpiTpReduce)
      return launch_one<PAIR, BN, STAGES, kEpiTpReduce, OUT_F32, 0>(maps, prm, grid, st);
  }
  if (static_cast<int>(epi) == kEpiQkvRope) {
    if constexpr (BN == 256) return launch_one<PAIR, BN, STAGES, kEpiQkvRope, OUT_BF16, KIND>(maps, prm, grid, st);
    return set_error(B2G_ERR_UNSUPPORTED, "qkv rope epilogue: 256-column tiles only");
  }
  if (epi == B2G_EPI_GATED_RESIDUAL)
    return launch_one<PAIR, BN, STAGES, B2G_EPI_GATED_RESIDUAL, OUT_F32, KIND>(maps, prm, grid, st);
  if (epi == B2G_EPI_GELU) {
    if (out == B2G_F32) return launch_one<PAIR, BN, STAGES, B2G_EPI_GELU, OUT_F32, KIND>(maps, prm, grid, st);
    if (out == B2G_BF16) return launch_one<PAIR, BN, STAGES, B2G_EPI_GELU, OUT_BF16, KIND>(maps, prm, grid, st);
    return launch_one<PAIR, BN, STAGES, B2G_EPI_GELU, OUT_F16, KIND>(maps, prm, grid, st);
  }
  if constexpr (KIND == 0) {
    if (epi == B2G_EPI_SILU) {
      if (out == B2G_F32) return launch_one<PAIR, BN, STAGES, B2G_EPI_SILU, OUT_F32, KIND>(maps, prm, grid, st);
      if (out == B2G_BF16) return launch_one<PAIR, BN, STAGES, B2G_EPI_SILU, OUT_BF16, KIND>(maps, prm, grid, st);
      return launch_one<PAIR, BN, STAGES, B2G_EPI_SILU, OUT_F16, KIND>(maps, prm, grid, st);
    }
  }
  if (out == B2G_F32) return launch_one<PAIR, BN, STAGES, B2G_EPI_NONE, OUT_F32, KIND>(maps, prm, grid, st);
  if (out == B2G_BF16) return launch_one<PAIR, BN, STAGES, B2G_EPI_NONE, OUT_BF16, KIND>(maps, prm, grid, st);
  return launch_one<PAIR, BN, STAGES, B2G_EPI_NONE, OUT_F16, KIND>(maps, prm, grid, st);
}

// kind: 0 = bf16/fp16 (kind::f16), 1 = tf32, 2 = E4M3 (kind::f8f6f4, STAGES8 ring stages: the
// column-scale staging area costs one stage's worth of shared memory in the larger variants).
template <bool PAIR, int BN, int STAGES, int STAGES8>
b2g_status dispatch_epi(const TcMaps& maps, const TcParams& prm, int grid, b2g_epilogue epi, b2g_dtype out, int kind,
                        cudaStream_t st) {
  if (kind == 1) {
    // fp32 operands (batched_matmul_Bt): plain F32 output only.
    if (epi != B2G_EPI_NONE || out != B2G_F32) return set_error(B2G_ERR_UNSUPPORTED, "tf32 path: F32 output only");
    return launch_one<PAIR, BN, STAGES, B2G_EPI_NONE, OUT_F32, 1>(maps, prm, grid, st);
  }
  if (kind == 2) return dispatch_out<PAIR, BN, STAGES8, 2>(maps, prm, grid, epi, out, st);
  return dispatch_out<PAIR, BN, STAGES, 0>(maps, prm, grid, epi, out, st);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool tc_gemm_supported(const GemmProblem& p, std::string* why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  const bool tf32 = p.a_dtype == B2G_F32 && p.b_dtype == B2G_F32 && p.allow_tf32;
  const bool fp8 = p.a_dtype == B2G_E4M3 && p.b_dtype == B2G_E4M3;
  if (!((p.a_dtype == B2G_BF16 && p.b_dtype == B2G_BF16) || (p.a_dtype == B2G_F16 && p.b_dtype == B2G_F16) || tf32 ||
        fp8))
    return no("operand dtypes");
  if (fp8 && (!p.a_scale || !p.b_scale)) return no("E4M3 operands need row and column scales");
  if (tf32 && (p.epilogue != B2G_EPI_NONE || p.d_dtype != B2G_F32)) return no("tf32: F32 output, no epilogue");
  if (p.d_dtype != B2G_F32 && p.d_dtype != B2G_BF16 && p.d_dtype != B2G_F16) return no("output dtype");
  if (p.epilogue == B2G_EPI_GATED_RESIDUAL && p.d_dtype != B2G_F32) return no("gated residual needs F32 output");
  if (p.bias && p.bias_dtype != B2G_F32 && p.bias_dtype != B2G_BF16) return no("bias dtype");
  if (!aligned16(p.a) || !aligned16(p.b)) return no("operand base not 16-byte aligned");
  const int64_t align = tf32 ? 3 : (fp8 ? 15 : 7);  // 16-byte row and batch strides
  if ((p.lda & align) || (p.ldb & align)) return no("operand row stride not a multiple of 16 bytes");
  if (p.batch > 1 && ((p.a_bstride & align) || (p.b_bstride & align))) return no("batch stride not 16-byte aligned");
  if (p.M > (1ll << 31) - 256 || p.N > (1ll << 31) - 256 || p.K > (1ll << 31)) return no("size");
  if (p.batch > 65535) return no("batch");
  return true;
}

// Problems that can share one launch: same N, K, batch (1 when grouped), operand, bias and
// output dtypes, epilogue and alpha.
bool tc_gemm_groupable(const GemmProblem& a, const GemmProblem& b) {
  return a.N == b.N && a.K == b.K && a.batch == 1 && b.batch == 1 && a.a_dtype == b.a_dtype &&
         a.b_dtype == b.b_dtype && a.d_dtype == b.d_dtype && a.epilogue == b.epilogue && a.alpha == b.alpha &&
         (a.bias == nullptr) == (b.bias == nullptr) && (!a.bias || a.bias_dtype == b.bias_dtype) &&
         a.allow_split == b.allow_split && (a.a_scale == nullptr) == (b.a_scale == nullptr) && a.tp == b.tp &&
         (a.rope == nullptr) == (b.rope == nullptr) &&
         (!a.rope || (a.rope->heads == b.rope->heads && a.rope->eps == b.rope->eps));
}

b2g_status tc_gemm_launch(const GemmProblem& p, cudaStream_t st) { return tc_gemm_launch_group(&p, 1, st); }

b2g_status tc_gemm_launch_group(const GemmProblem* ps, int count, cudaStream_t st) {
  if (count < 1 || count > kMaxGroups) return set_error(B2G_ERR_INVALID, "tc_gemm: 1 to 4 problems per launch");
  for (int i = 1; i < count; ++i)
    if (!tc_gemm_groupable(ps[0], ps[i])) return set_error(B2G_ERR_INVALID, "tc_gemm: problems cannot share a launch");
  const GemmProblem& p = ps[0];
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  if ((s = get_encode()) != B2G_OK) return s;
  if (g_tma_store < 0) {
    const char* t = getenv("B2G_TMA_STORE");
    g_tma_store = (t && t[0] == '0') ? 0 : 1;
  }

  const int sms = dev->num_sms;
  const int pairs = sms / 2;
  const bool tf32 = p.a_dtype == B2G_F32;
  const int kind = tf32 ? 1 : (p.a_dtype == B2G_E4M3 ? 2 : 0);
  const int kelems = kind == 1 ? 32 : (kind == 2 ? 128 : 64);
  const long long nkb = (p.K + kelems - 1) / kelems;
  // Kernel variant and split-K factor from a cost model in units of one 64-wide k-block of
  // a pair tile: whole waves of work items over the SMs (or SM pairs), times the k-blocks
  // per item, times the variant's measured relative cost per k-block, plus the split-K
  // reduction overhead.  The tiles of all problems of the launch form one pool of work.
  enum { V128 = 0, V256 = 1, VPAIR = 2 };
  int v = VPAIR, splits = 1;
  bool tail_only = false;  // split only the tiles of the last, partial wave
  double best = 1e300;
  for (int cand = 0; cand < 3; ++cand) {
    if (cand == VPAIR && !g_allow_pair) continue;
    if (cand != V128 && p.N <= 128) continue;
    if (cand == V128 && p.rope) continue;  // the rope epilogue needs a whole head per thread
    if (cand == VPAIR && p.round_tf32) continue;  // in-kernel TF32 rounding: 1-CTA kernels only
    const long long tm = cand == VPAIR ? 256 : 128, tn = cand == V128 ? 128 : 256;
    long long tiles = 0;
    for (int i = 0; i < count; ++i) tiles += ps[i].batch * ((ps[i].M + tm - 1) / tm) * ((p.N + tn - 1) / tn);
    const long long slots = cand == VPAIR ? pairs : sms;
    const double kb_cost = cand == V128 ? kCost128 : (cand == V256 ? kCost256 : kCostPair);
    for (int sk = 1; sk <= 8 && sk <= nkb; ++sk) {
      const long long items = tiles * sk;
      const double waves = static_cast<double>((items + slots - 1) / slots);
      const double per = static_cast<double>((nkb + sk - 1) / sk);
      const double cost = kb_cost * (waves * per + (sk > 1 ? kSplitOverhead * sk : 0.0));
      if (cost < best - 1e-9) {
        best = cost;
        v = cand;
        splits = sk;
        tail_only = false;
      }
    }
    // Whole tiles for the full waves, the partial wave's tiles split to fill one wave.
    const long long full = tiles / slots, rest = tiles % slots;
    if (full >= 1 && rest > 0) {
      for (long long sk = 2; sk <= 8 && sk <= nkb && rest * sk <= slots; ++sk) {
        const double last = static_cast<double>((nkb + sk - 1) / sk);
        const double cost = kb_cost * (static_cast<double>(full) * nkb + last + kTailFixed + kTailPerSplit * sk);
        if (cost < best - 1e-9) {
          best = cost;
          v = cand;
          splits = static_cast<int>(sk);
          tail_only = true;
        }
      }
    }
  }
  if (g_force_variant >= 0) {
    v = g_force_variant;
    if (g_force_splits == 0) splits = 1;
  }
  if (g_force_splits != 0) {
    const int f = g_force_splits > 0 ? g_force_splits : -g_force_splits;
    splits = static_cast<int>(f < nkb ? f : nkb);
    tail_only = g_force_splits < 0;
  }
  if (nkb == 0 || !p.allow_split || p.tp || p.rope) splits = 1;
  if (p.rope && v == V128) v = g_allow_pair ? VPAIR : V256;
  if (p.round_tf32 && v == VPAIR) v = V256;
  const bool pair = v == VPAIR;
  const int bn = v == V128 ? 128 : 256;
  const int tile_m = pair ? 256 : kBM;

  TcParams prm{};
  prm.N = static_cast<int>(p.N);
  prm.K = static_cast<int>(p.K);
  prm.batch = static_cast<int>(p.batch);
  prm.num_n_blocks = static_cast<int>((p.N + bn - 1) / bn);
  prm.num_k_blocks = static_cast<int>(nkb);
  prm.groups = count;
  prm.raster_m = pair ? 8 : 16;
  const int out_bytes = p.d_dtype == B2G_F32 ? 4 : 2;
  bool all_vec = true;
  double a_bytes = 0, b_bytes = 0;
  int tiles = 0;
  for (int i = 0; i < count; ++i) {
    const GemmProblem& q = ps[i];
    TcGroup& G = prm.g[i];
    G.M = static_cast<int>(q.M);
    G.num_m_blocks = static_cast<int>((q.M + tile_m - 1) / tile_m);
    G.tile0 = tiles;
    tiles += prm.batch * G.num_m_blocks * prm.num_n_blocks;
    G.d = q.d;
    G.ldd = q.ldd;
    G.bias = q.bias;
    G.gate = q.gate;
    G.a_scale = q.a_scale;
    G.b_scale = q.b_scale;
    G.tp_row0 = q.tp_row0;
    G.pe = q.rope ? q.rope->pe : nullptr;
    G.qn = q.rope ? q.rope->q_norm : nullptr;
    G.kn = q.rope ? q.rope->k_norm : nullptr;
    G.pe_period = q.rope ? static_cast<int>(q.rope->pe_period) : 0;
    G.pe_compact = q.rope ? (q.rope->pe_compact ? 1 : 0) : 0;
    G.vec_ok = aligned16(q.d) && ((q.ldd * out_bytes) % 16 == 0) &&
               (q.batch <= 1 || (q.d_bstride * out_bytes) % 16 == 0);
    all_vec = all_vec && G.vec_ok;
    a_bytes += static_cast<double>(q.M) * q.K;
    b_bytes += static_cast<double>(q.N) * q.K;
  }
  prm.num_tiles = tiles;
  {
    // Split tiles: all of them, or (tail_only) those of the last wave when it is partial.
    const int slots = pair ? pairs : sms;
    const int rest = tiles % slots;
    prm.dp_tiles = splits <= 1 ? tiles : (tail_only ? (rest == 0 ? tiles : (tiles < slots ? 0 : tiles - rest)) : 0);
    if (splits > 1 && prm.dp_tiles == tiles) splits = 1;
  }
  prm.splits = splits;
  prm.num_items = prm.dp_tiles + (prm.num_tiles - prm.dp_tiles) * splits;
  prm.d_bstride = p.batch > 1 ? p.d_bstride : 0;
  prm.bias_kind = p.bias ? (p.bias_dtype == B2G_F32 ? 1 : 2) : 0;
  prm.alpha = p.alpha;
  prm.round_tf32 = (kind == 1 && p.round_tf32) ? 1 : 0;
  prm.err = dev->err_word;
  prm.idesc = idesc_make(kind == 1 ? kFmtTF32 : (kind == 2 ? kFmtE4M3 : (p.a_dtype == B2G_BF16 ? kFmtBF16 : kFmtF16)),
                         tile_m, bn);
  prm.a_keep = a_bytes <= b_bytes ? 1 : 0;
  if (prm.num_tiles == 0) return B2G_OK;

  if (splits > 1) {
    const size_t slots = static_cast<size_t>(prm.num_tiles - prm.dp_tiles) * (pair ? 2 : 1);
    void* ws = nullptr;
    void* ctr = nullptr;
    if ((s = workspace_get(slots * splits * 128 * bn * sizeof(float), &ws, kWsSplitK)) != B2G_OK) return s;
    if ((s = workspace_get(slots * sizeof(int), &ctr, kWsCounters)) != B2G_OK) return s;
    prm.ws = static_cast<float*>(ws);
    prm.counters = static_cast<int*>(ctr);
  }

  TcMaps maps;
  memset(&maps, 0, sizeof(maps));
  const uint32_t b_box = v == V256 ? 256u : 128u;
  prm.tma_store = all_vec && g_tma_store && !p.tp ? 1 : 0;
  if (p.rope) {
    const QkvRope& r = *p.rope;
    if (kind == 1 || p.d_dtype != B2G_BF16 || p.batch != 1)
      return set_error(B2G_ERR_UNSUPPORTED, "qkv rope epilogue: bf16/fp16/E4M3 operands, bf16 output, no batch");
    const bool tail = r.gelu_out != nullptr;
    if (r.heads < 1 || (tail ? p.N <= 3 * r.heads * 128 : p.N != 3 * r.heads * 128))
      return set_error(B2G_ERR_INVALID, "qkv rope epilogue: N must be 3 * heads * 128 (more with a GELU tail)");
    if (tail && (count != 1 || (reinterpret_cast<uintptr_t>(r.gelu_out) & 15u) || (r.gelu_ld * 2) % 16 != 0 ||
                 r.gelu_ld < p.N - 3 * r.heads * 128))
      return set_error(B2G_ERR_UNSUPPORTED, "qkv rope epilogue: GELU tail needs one problem and 16-byte aligned rows");
    if (!prm.tma_store) return set_error(B2G_ERR_UNSUPPORTED, "qkv rope epilogue: 16-byte aligned output rows required");
    for (int i = 0; i < count; ++i) {
      const QkvRope& ri = *ps[i].rope;
      if (!ri.pe || !aligned16(ri.pe) || (ri.q_norm && !aligned16(ri.q_norm)) || (ri.k_norm && !aligned16(ri.k_norm)))
        return set_error(B2G_ERR_INVALID, "qkv rope epilogue: pe and norm scales must be 16-byte aligned");
    }
    prm.hd = static_cast<int>(r.heads * 128);
    prm.eps = r.eps;
    prm.n_outer = 1;
    prm.split = tail ? 3 * prm.hd : 0;
  }
  if (p.tp) {
    const TpReduce& t = *p.tp;
    if (kind != 0) return set_error(B2G_ERR_UNSUPPORTED, "tp reduce: bf16/fp16 operands only");
    if (t.world < 1 || t.world > 8 || t.rank < 0 || t.rank >= t.world || !t.part_ptrs || !t.res_ptrs || !t.counters)
      return set_error(B2G_ERR_INVALID, "tp reduce: world/rank/pointers");
    if (p.N % 32 != 0 || t.ld_part % 8 != 0 || t.ld_res % 4 != 0 || t.ld_part < p.N || t.ld_res < p.N)
      return set_error(B2G_ERR_UNSUPPORTED, "tp reduce: N % 32 and 16-byte partial / residual rows required");
    if (static_cast<int64_t>(prm.num_tiles) * (pair ? 2 : 1) > t.counter_slots)
      return set_error(B2G_ERR_INVALID, "tp reduce: not enough counter slots for this launch");
    for (int i = 0; i < count; ++i)
      if (!ps[i].gate) return set_error(B2G_ERR_INVALID, "tp reduce: a gate is required");
    prm.tp_world = t.world;
    prm.tp_rank = t.rank;
    prm.tp_part = t.part_ptrs;
    prm.tp_res = t.res_ptrs;
    prm.tp_ld_part = t.ld_part;
    prm.tp_ld_res = t.ld_res;
    prm.tp_counters = t.counters;
  }
  for (int i = 0; i < count; ++i) {
    const GemmProblem& q = ps[i];
    const int64_t a_bs = q.batch > 1 ? q.a_bstride : q.lda * q.M;
    const int64_t b_bs = q.batch > 1 ? q.b_bstride : q.ldb * q.N;
    if ((s = make_operand_map(&maps.a[i], q.a, q.a_dtype, q.K, q.M, q.lda, q.batch, a_bs, kBM)) != B2G_OK) return s;
    if ((s = make_operand_map(&maps.b[i], q.b, q.b_dtype, q.K, q.N, q.ldb, q.batch, b_bs, b_box)) != B2G_OK) return s;
    if (prm.tma_store && q.d) {
      const int64_t d_bs = q.batch > 1 ? q.d_bstride : q.ldd * q.M;
      const int64_t n_d = prm.split ? prm.split : q.N;  // a GELU tail has its own map, next
      if ((s = make_output_map(&maps.d[i], q.d, q.d_dtype, n_d, q.M, q.ldd, q.batch, d_bs)) != B2G_OK) return s;
      if (prm.split) {
        const QkvRope& r = *q.rope;
        if ((s = make_output_map(&maps.d[i + 1], r.gelu_out, B2G_BF16, q.N - prm.split, q.M, r.gelu_ld, 1,
                                 r.gelu_ld * q.M)) != B2G_OK)
          return s;
      }
    }
  }

  if (pair) {
    const int grid = 2 * static_cast<int>(prm.num_items < pairs ? prm.num_items : pairs);
    return dispatch_epi<true, 256, kPairStages, kPairStages - 1>(maps, prm, grid, p.epilogue, p.d_dtype, kind, st);
  }
  const int grid = static_cast<int>(prm.num_items < sms ? prm.num_items : sms);
  if (v == V256)
    return dispatch_epi<false, 256, kStages256, kStages256 - 1>(maps, prm, grid, p.epilogue, p.d_dtype, kind, st);
  return dispatch_epi<false, 128, kStages128, kStages128 - 1>(maps, prm, grid, p.epilogue, p.d_dtype, kind, st);
}

void tc_gemm_set_variant(int force_variant, int allow_pair, int force_splits) {
  g_force_variant = force_variant;
  g_allow_pair = allow_pair != 0;
  g_force_splits = force_splits;
}

}  // namespace b2g
