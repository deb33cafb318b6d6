// gemm_tc.cu — the engine's tensor-core GEMM for sm_100a.
//
//   D[b, m, n] = epilogue( sum_k A[b, m, k] * B[b, n, k] + bias[n] )
//
// A (activations) and B (weights) are K-major bf16 or fp16 in global memory.  This is the
// computation of the reference's cuBLASLt call in linear_lt (cublas_ops.cuh:214-288:
// TRANSA=T on W, TRANSB=N on x, fp32 compute, bias epilogue), with the elementwise work
// that the reference runs as separate kernels after it (gelu_to_bf16 kernels.cu:297-310,
// gated_residual kernels.cu:942-968) fused into the store.
//
// Design (one persistent CTA per SM, 192 threads, warp-specialised):
//   warp 0      TMA producer: 128x64 A tile + BNx64 B tile per stage, 128-byte swizzle,
//               STAGES-deep ring of shared-memory stages guarded by full/empty mbarriers.
//   warp 1      allocates TMEM (2 accumulators of 128 lanes x BN fp32 columns) and issues
//               tcgen05.mma (M=128, N=BN, K=16) from one thread; tcgen05.commit frees a
//               smem stage when the MMAs reading it retire, and signals a finished
//               accumulator to the epilogue.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time (warp w owns TMEM lanes
//               32*(w%4)..+31 = tile rows), add bias, apply GELU or gate*y+residual,
//               convert and store with 16-byte vector stores.  The accumulator is handed
//               back as soon as it is read, so tile i's epilogue overlaps tile i+1's MMAs.
// Every wait is bounded (ptx_sm100.cuh): on timeout the kernel records an error word,
// waits for its own TMA copies / MMAs in flight, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <mutex>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;          // 64 x 2 B = one 128-byte swizzle row (16-bit operands)
// K elements per 128-byte stage row: 64 for bf16/fp16 (KIND 0), 32 for tf32 (KIND 1).
template <int KIND>
constexpr int kKElems = KIND == 1 ? 32 : 64;
constexpr int kThreads = 192;
enum { OUT_F32 = 0, OUT_BF16 = 1, OUT_F16 = 2 };

struct TcParams {
  int M, N, K, batch;
  int num_m_blocks, num_n_blocks, num_k_blocks, num_tiles;
  int group_m;             // rasterisation group (m-blocks that share B panels in flight)
  void* d;
  long long ldd, d_bstride;
  const void* bias;
  int bias_kind;           // 0 none, 1 f32, 2 bf16
  const float* gate;
  int* err;
  uint32_t idesc;
  int vec_ok;              // D base/ldd allow 16-byte vector stores
  int a_keep;              // 1: keep A in L2 (evict_last), stream B (evict_first); 0: reverse
};

__host__ __device__ constexpr size_t smem_bytes(int bn, int stages) {
  return 1024 /* alignment slack */ + static_cast<size_t>(stages) * (kBM * kBK * 2 + bn * kBK * 2) +
         256 /* barriers + TMEM slot */;
}

__device__ __forceinline__ void tile_coords(int tile, const TcParams& p, int& bz, int& mb, int& nb) {
  const int per_batch = p.num_m_blocks * p.num_n_blocks;
  bz = tile / per_batch;
  int r = tile - bz * per_batch;
  // Groups of group_m m-blocks; inside a group m varies fastest, so the CTAs in flight
  // read the same few B panels and the same group of A rows (both stay in L2).
  const int group_size = p.group_m * p.num_n_blocks;
  const int g = r / group_size;
  const int first_m = g * p.group_m;
  const int gm = min(p.num_m_blocks - first_m, p.group_m);
  r -= g * group_size;
  mb = first_m + r % gm;
  nb = r / gm;
}

// tanh-form GELU, the formula of the reference's gelu_val (kernels.cu:266-269).
__device__ __forceinline__ float gelu_tanh(float v) {
  const float inner = 0.7978845608f * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner));
}

template <int EPI, int OUT>
__device__ __forceinline__ void store_chunk(const TcParams& p, int bz, int m, int n0, const uint32_t (&r)[32]) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  const bool full = (n0 + 32 <= p.N);
  const int nvalid = full ? 32 : (p.N - n0);
  if (p.bias_kind == 1) {
    const float* bp = static_cast<const float*>(p.bias) + n0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (full || j < nvalid) v[j] += __ldg(bp + j);
  } else if (p.bias_kind == 2) {
    const __nv_bfloat16* bp = static_cast<const __nv_bfloat16*>(p.bias) + n0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (full || j < nvalid) v[j] += __bfloat162float(bp[j]);
  }
  if constexpr (EPI == B2G_EPI_GELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
  }
  const long long off = static_cast<long long>(bz) * p.d_bstride + static_cast<long long>(m) * p.ldd + n0;
  if constexpr (OUT == OUT_F32) {
    float* dp = static_cast<float*>(p.d) + off;
    if constexpr (EPI == B2G_EPI_GATED_RESIDUAL) {
      const float* gp = p.gate + n0;
      if (full && p.vec_ok) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 res = reinterpret_cast<const float4*>(dp)[j];
          res.x += __ldg(gp + 4 * j + 0) * v[4 * j + 0];
          res.y += __ldg(gp + 4 * j + 1) * v[4 * j + 1];
          res.z += __ldg(gp + 4 * j + 2) * v[4 * j + 2];
          res.w += __ldg(gp + 4 * j + 3) * v[4 * j + 3];
          reinterpret_cast<float4*>(dp)[j] = res;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nvalid) dp[j] = dp[j] + __ldg(gp + j) * v[j];
      }
    } else {
      if (full && p.vec_ok) {
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
    uint16_t* dp = static_cast<uint16_t*>(p.d) + off;
    if (full && p.vec_ok) {
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

template <int BN, int STAGES, int EPI, int OUT, int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const TcParams p) {
  constexpr uint32_t A_BYTES = kBM * kBK * 2;
  constexpr uint32_t B_BYTES = BN * kBK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators; 256 or 512 (power of two)
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

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
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int bz, mb, nb;
        tile_coords(tile, p, bz, mb, nb);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], A_BYTES + B_BYTES);
          tma_load_3d(sA + stage * A_BYTES, &tmA, &full_bar[stage], kb * kKElems<KIND>, mb * kBM, bz, pa);
          tma_load_3d(sB + stage * B_BYTES, &tmB, &full_bar[stage], kb * kKElems<KIND>, nb * BN, bz, pb);
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
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
        const uint32_t acc = local & 1u;
        const uint32_t acc_phase = (local >> 1) & 1u;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, p.err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, p.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // One MMA consumes 32 bytes of K (16 bf16/fp16 or 8 tf32 elements) inside the
            // 128-byte swizzle row: advance the descriptors by 32 bytes.
            const uint64_t ad = smem_desc_k_sw128(a0 + k * 32), bd = smem_desc_k_sw128(b0 + k * 32);
            if constexpr (KIND == 1) umma_tf32(d_tmem, ad, bd, p.idesc, (kb | k) != 0 ? 1u : 0u);
            else umma_f16(d_tmem, ad, bd, p.idesc, (kb | k) != 0 ? 1u : 0u);
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
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    uint32_t local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      int bz, mb, nb;
      tile_coords(tile, p, bz, mb, nb);
      const uint32_t acc = local & 1u;
      const uint32_t acc_phase = (local >> 1) & 1u;
      const bool ok = mbar_wait(&tfull_bar[acc], acc_phase, p.err, kErrWaitEpilogue);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int m = mb * kBM + row;
      const uint32_t t0 = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t0 + c * 32, r);
        tmem_wait_ld();
        if (c == BN / 32 - 1) {
          // Accumulator fully read: hand it back to the MMA warp before the last stores.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty_bar[acc]);
        }
        const int n0 = nb * BN + c * 32;
        if (m < p.M && n0 < p.N) store_chunk<EPI, OUT>(p, bz, m, n0, r);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- 2-CTA variant
//
// A cluster of two CTAs (on two SMs) computes one 256x256 output tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16).  CTA r of the pair loads rows
// [m0 + 128r, +128) of A and rows [n0 + 128r, +128) of B into its own shared memory; the
// MMA, issued by CTA 0, reads both halves and leaves rows [m0 + 128r, +128) x 256 columns
// of the accumulator in CTA r's TMEM.  Per SM this moves 32 KB of operands per 64-wide
// k-block instead of 48 KB for a 1-CTA 128x256 tile with the same MMA time, and the
// smaller stage allows a 6-deep ring.
//   full[s]   (CTA 0 only)  both CTAs' TMA bytes for stage s; CTA 0 arms it for 64 KB.
//   empty[s]  (each CTA)    the pair's MMAs reading stage s have retired (broadcast commit).
//   tfull[a]  (each CTA)    accumulator a is complete (broadcast commit).
//   tempty[a] (CTA 0 only)  all 8 epilogue warps of the pair have read accumulator a.
template <int STAGES, int EPI, int OUT, int KIND>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const TcParams p) {
  constexpr int BN = 256;                          // pair tile is 256 x 256
  constexpr uint32_t A_BYTES = kBM * kBK * 2;      // this CTA's 128 rows of A
  constexpr uint32_t B_BYTES = 128 * kBK * 2;      // this CTA's 128 rows of B
  constexpr uint32_t TMEM_COLS = 2 * BN;           // two 128-lane x 256-column accumulators

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);

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
      mbar_init(&tempty_bar[a], 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barrier inits and the TMEM allocation are visible pair-wide
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

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
      for (int tile = cluster; tile < p.num_tiles && ok; tile += nclusters) {
        int bz, mb, nb;
        tile_coords(tile, p, bz, mb, nb);
        const int arow = mb * 256 + static_cast<int>(rank) * 128;
        const int brow = nb * 256 + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * (A_BYTES + B_BYTES));
          const uint32_t leader_full = map_to_cta(smem_u32(&full_bar[stage]), 0);
          tma_load_3d_pair(sA + stage * A_BYTES, &tmA, leader_full, kb * kKElems<KIND>, arow, bz, pa);
          tma_load_3d_pair(sB + stage * B_BYTES, &tmB, leader_full, kb * kKElems<KIND>, brow, bz, pb);
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
      for (int tile = cluster; tile < p.num_tiles && ok; tile += nclusters, ++local) {
        const uint32_t acc = local & 1u;
        const uint32_t acc_phase = (local >> 1) & 1u;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, p.err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
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
            if constexpr (KIND == 1) umma_tf32_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            else umma_f16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
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
    // ------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const int q = warp & 3;
    const int row = q * 32 + lane;
    uint32_t local = 0;
    const uint32_t leader_tempty0 = map_to_cta(smem_u32(&tempty_bar[0]), 0);
    const uint32_t leader_tempty1 = map_to_cta(smem_u32(&tempty_bar[1]), 0);
    for (int tile = cluster; tile < p.num_tiles; tile += nclusters, ++local) {
      int bz, mb, nb;
      tile_coords(tile, p, bz, mb, nb);
      const uint32_t acc = local & 1u;
      const uint32_t acc_phase = (local >> 1) & 1u;
      const bool ok = mbar_wait(&tfull_bar[acc], acc_phase, p.err, kErrWaitEpilogue);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int m = mb * 256 + static_cast<int>(rank) * 128 + row;
      const uint32_t t0 = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t0 + c * 32, r);
        tmem_wait_ld();
        if (c == BN / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
        }
        const int n0 = nb * BN + c * 32;
        if (m < p.M && n0 < p.N) store_chunk<EPI, OUT>(p, bz, m, n0, r);
      }
    }
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

// Relative per-tile time of the 2-CTA kernel vs the 1-CTA 128x256 kernel (tuned on B200).
constexpr double kPairSpeed = 0.85;
int g_force_variant = -1;  // -1 auto, 0 = 1-CTA 128, 1 = 1-CTA 256, 2 = 2-CTA pair
bool g_allow_pair = true;

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

// 3-D K-major operand map: dims {K, rows, batch}, box {128 bytes of K, box_rows, 1}, 128-byte swizzle,
// out-of-bounds elements read as zero (so ragged M, N and K tiles need no special case).
b2g_status make_operand_map(CUtensorMap* map, const void* base, b2g_dtype dt, int64_t K, int64_t rows,
                            int64_t ld, int64_t batch, int64_t bstride, uint32_t box_rows) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(batch)};
  const cuuint64_t esz = dt == B2G_F32 ? 4u : 2u;
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * esz, static_cast<cuuint64_t>(bstride) * esz};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / esz), box_rows, 1u};  // 128-byte rows
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType t = dt == B2G_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                : dt == B2G_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = g_encode(map, t, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(B2G_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return B2G_OK;
}

template <typename Kern>
b2g_status launch_kernel(Kern kern, size_t smem, const CUtensorMap& ta, const CUtensorMap& tb, const TcParams& prm,
                         int grid, cudaStream_t st) {
  b2g_status s = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "cudaFuncSetAttribute(tc_gemm)");
  if (s != B2G_OK) return s;
  kern<<<grid, kThreads, smem, st>>>(ta, tb, prm);
  note_launch();
  return check_cuda(cudaGetLastError(), "tc_gemm launch");
}

// Variant selector: PAIR = 2-CTA 256x256 kernel, else 1-CTA 128xBN kernel.
template <bool PAIR, int BN, int STAGES, int EPI, int OUT, int KIND>
b2g_status launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const TcParams& prm, int grid, cudaStream_t st) {
  if constexpr (PAIR) {
    constexpr size_t smem = 1024 + static_cast<size_t>(STAGES) * (kBM * kBK * 2 + 128 * kBK * 2) + 256;
    static_assert(smem <= 227 * 1024, "shared memory budget");
    return launch_kernel(tc_gemm_pair_kernel<STAGES, EPI, OUT, KIND>, smem, ta, tb, prm, grid, st);
  } else {
    constexpr size_t smem = smem_bytes(BN, STAGES);
    static_assert(smem <= 227 * 1024, "shared memory budget");
    return launch_kernel(tc_gemm_kernel<BN, STAGES, EPI, OUT, KIND>, smem, ta, tb, prm, grid, st);
  }
}

template <bool PAIR, int BN, int STAGES>
b2g_status dispatch_epi(const CUtensorMap& ta, const CUtensorMap& tb, const TcParams& prm, int grid,
                        b2g_epilogue epi, b2g_dtype out, bool tf32, cudaStream_t st) {
  if (tf32) {
    // fp32 operands (batched_matmul_Bt): plain F32 output only.
    if (epi != B2G_EPI_NONE || out != B2G_F32) return set_error(B2G_ERR_UNSUPPORTED, "tf32 path: F32 output only");
    return launch_one<PAIR, BN, STAGES, B2G_EPI_NONE, OUT_F32, 1>(ta, tb, prm, grid, st);
  }
  if (epi == B2G_EPI_GATED_RESIDUAL)
    return launch_one<PAIR, BN, STAGES, B2G_EPI_GATED_RESIDUAL, OUT_F32, 0>(ta, tb, prm, grid, st);
  if (epi == B2G_EPI_GELU) {
    if (out == B2G_F32) return launch_one<PAIR, BN, STAGES, B2G_EPI_GELU, OUT_F32, 0>(ta, tb, prm, grid, st);
    if (out == B2G_BF16) return launch_one<PAIR, BN, STAGES, B2G_EPI_GELU, OUT_BF16, 0>(ta, tb, prm, grid, st);
    return launch_one<PAIR, BN, STAGES, B2G_EPI_GELU, OUT_F16, 0>(ta, tb, prm, grid, st);
  }
  if (out == B2G_F32) return launch_one<PAIR, BN, STAGES, B2G_EPI_NONE, OUT_F32, 0>(ta, tb, prm, grid, st);
  if (out == B2G_BF16) return launch_one<PAIR, BN, STAGES, B2G_EPI_NONE, OUT_BF16, 0>(ta, tb, prm, grid, st);
  return launch_one<PAIR, BN, STAGES, B2G_EPI_NONE, OUT_F16, 0>(ta, tb, prm, grid, st);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool tc_gemm_supported(const GemmProblem& p, std::string* why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  const bool tf32 = p.a_dtype == B2G_F32 && p.b_dtype == B2G_F32 && p.allow_tf32;
  if (!((p.a_dtype == B2G_BF16 && p.b_dtype == B2G_BF16) || (p.a_dtype == B2G_F16 && p.b_dtype == B2G_F16) || tf32))
    return no("operand dtypes");
  if (tf32 && (p.epilogue != B2G_EPI_NONE || p.d_dtype != B2G_F32)) return no("tf32: F32 output, no epilogue");
  if (p.d_dtype != B2G_F32 && p.d_dtype != B2G_BF16 && p.d_dtype != B2G_F16) return no("output dtype");
  if (p.epilogue == B2G_EPI_GATED_RESIDUAL && p.d_dtype != B2G_F32) return no("gated residual needs F32 output");
  if (p.bias && p.bias_dtype != B2G_F32 && p.bias_dtype != B2G_BF16) return no("bias dtype");
  if (!aligned16(p.a) || !aligned16(p.b)) return no("operand base not 16-byte aligned");
  const int64_t align = tf32 ? 3 : 7;  // 16-byte row and batch strides
  if ((p.lda & align) || (p.ldb & align)) return no("operand row stride not a multiple of 16 bytes");
  if (p.batch > 1 && ((p.a_bstride & align) || (p.b_bstride & align))) return no("batch stride not 16-byte aligned");
  if (p.M > (1ll << 31) - kBM || p.N > (1ll << 31) - 256 || p.K > (1ll << 31)) return no("size");
  if (p.batch > 65535) return no("batch");
  return true;
}

b2g_status tc_gemm_launch(const GemmProblem& p, cudaStream_t st) {
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  if ((s = get_encode()) != B2G_OK) return s;

  const int sms = dev->num_sms;
  const long long m128 = (p.M + 127) / 128, m256 = (p.M + 255) / 256;
  const long long t128 = p.batch * m128 * ((p.N + 127) / 128);
  const long long t256 = p.batch * m128 * ((p.N + 255) / 256);
  const long long tpair = p.batch * m256 * ((p.N + 255) / 256);
  const int pairs = sms / 2;
  // Estimated time in units of one 128x256 tile on one SM at the 1-CTA kernel's rate:
  // whole waves over the SMs.  A 128-wide tile does half the work of a 256-wide one but
  // re-reads A (10% penalty); a 2-CTA pair tile is one such unit on two SMs and runs at a
  // higher tensor-pipe utilisation (operand bandwidth per SM is a third lower).
  const double cost256 = static_cast<double>((t256 + sms - 1) / sms);
  const double cost128 = static_cast<double>((t128 + sms - 1) / sms) * 0.55;
  const double costpair = static_cast<double>((tpair + pairs - 1) / pairs) * kPairSpeed;
  enum { V128, V256, VPAIR } v;
  if (p.N <= 128) v = V128;
  else if (costpair <= cost256 && costpair <= cost128 && g_allow_pair) v = VPAIR;
  else v = cost128 < cost256 ? V128 : V256;
  if (g_force_variant >= 0) v = static_cast<decltype(v)>(g_force_variant);
  const int bn = v == V128 ? 128 : 256;
  const int tile_m = v == VPAIR ? 256 : kBM;

  TcParams prm{};
  prm.M = static_cast<int>(p.M);
  prm.N = static_cast<int>(p.N);
  prm.K = static_cast<int>(p.K);
  prm.batch = static_cast<int>(p.batch);
  prm.num_m_blocks = static_cast<int>((p.M + tile_m - 1) / tile_m);
  prm.num_n_blocks = static_cast<int>((p.N + bn - 1) / bn);
  const bool tf32 = p.a_dtype == B2G_F32;
  const int kelems = tf32 ? 32 : 64;
  prm.num_k_blocks = static_cast<int>((p.K + kelems - 1) / kelems);
  prm.num_tiles = prm.batch * prm.num_m_blocks * prm.num_n_blocks;
  const int group = v == VPAIR ? 8 : 16;
  prm.group_m = prm.num_m_blocks <= group ? prm.num_m_blocks : group;
  prm.d = p.d;
  prm.ldd = p.ldd;
  prm.d_bstride = p.batch > 1 ? p.d_bstride : 0;
  prm.bias = p.bias;
  prm.bias_kind = p.bias ? (p.bias_dtype == B2G_F32 ? 1 : 2) : 0;
  prm.gate = p.gate;
  prm.err = dev->err_word;
  prm.idesc = idesc_make(tf32 ? kFmtTF32 : (p.a_dtype == B2G_BF16 ? kFmtBF16 : kFmtF16), tile_m, bn);
  const int out_bytes = p.d_dtype == B2G_F32 ? 4 : 2;
  prm.vec_ok = aligned16(p.d) && ((p.ldd * out_bytes) % 16 == 0) &&
               (p.batch <= 1 || (p.d_bstride * out_bytes) % 16 == 0);
  const double a_bytes = static_cast<double>(p.M) * p.K, b_bytes = static_cast<double>(p.N) * p.K;
  prm.a_keep = a_bytes <= b_bytes ? 1 : 0;
  if (prm.num_tiles == 0) return B2G_OK;

  CUtensorMap ta, tb;
  const int64_t a_bs = p.batch > 1 ? p.a_bstride : p.lda * p.M;
  const int64_t b_bs = p.batch > 1 ? p.b_bstride : p.ldb * p.N;
  const uint32_t b_box = v == V128 ? 128u : (v == V256 ? 256u : 128u);
  if ((s = make_operand_map(&ta, p.a, p.a_dtype, p.K, p.M, p.lda, p.batch, a_bs, kBM)) != B2G_OK) return s;
  if ((s = make_operand_map(&tb, p.b, p.b_dtype, p.K, p.N, p.ldb, p.batch, b_bs, b_box)) != B2G_OK) return s;

  if (v == VPAIR) {
    const int grid = 2 * static_cast<int>(prm.num_tiles < pairs ? prm.num_tiles : pairs);
    return dispatch_epi<true, 256, 6>(ta, tb, prm, grid, p.epilogue, p.d_dtype, tf32, st);
  }
  const int grid = static_cast<int>(prm.num_tiles < sms ? prm.num_tiles : sms);
  if (v == V256) return dispatch_epi<false, 256, 4>(ta, tb, prm, grid, p.epilogue, p.d_dtype, tf32, st);
  return dispatch_epi<false, 128, 6>(ta, tb, prm, grid, p.epilogue, p.d_dtype, tf32, st);
}

void tc_gemm_set_variant(int force_variant, int allow_pair) {
  g_force_variant = force_variant;
  g_allow_pair = allow_pair != 0;
}

}  // namespace b2g
