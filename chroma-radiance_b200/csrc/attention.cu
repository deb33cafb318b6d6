// attention.cu — the Chroma transformer's attention on the tensor cores.
//
// Replaces cudnn_attention_with_rope (cudnn_attention.cuh:449-476): RoPE + bf16 on Q and K
// (apply_rope_fused_bf16, rope.cuh:180-221), V to bf16, softmax(Q K^T / sqrt(D) + key_bias) V
// (cuDNN SDPA, cudnn_attention.cuh:408-443), output F32 [L, H*D] (or bf16 for the block path).
//
//   1. attn_prep         one launch: Q, K F32 rows [L, H*D] -> optional per-head RMSNorm
//                        (qk_norm) -> RoPE -> bf16 [L, H*D]; V F32 -> bf16 [L, H*D].  The
//                        attention kernel reads head h of each through TMA (row stride H*D,
//                        head stride D).  The block path skips this launch: its qkv GEMM
//                        applies norm and RoPE in the epilogue and writes bf16 [L, 3*H*D]
//                        (attention_bf16 below).
//   2. flash_attn        two 128-query tiles of one head per CTA: S = Q K^T on the tensor
//                        cores into TMEM, online softmax in registers, P (bf16) back into
//                        TMEM as the A operand of O += P V (V read MN-major, as stored), O /
//                        rowsum written to the output layout.  S never leaves the SM.
#include <cuda_bf16.h>
#include <cstdint>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

// Key-split override for the fused attention (b2g_set_attention_splits): 0 automatic, -1
// never, > 0 that many slices.
int g_attn_splits = 0;

namespace {

// Attention prologue (256 threads per block): Q, K and V rows, each warp 2 (token l, head h)
// rows of D values.  Q and K: RMSNorm with a learned scale (rms_norm, kernels.cu:174-207, as
// qk_norm applies it, chroma.cuh:513-515; rows l >= norm_split use the second scale set), RoPE
// with pe row l = D/2 groups of (cos, -sin, sin, cos) (the table gen_pe builds, rope.cuh:84,
// applied as apply_rope_fused_bf16 does, rope.cuh:180-221), bf16 out [L, H*D].  V: bf16 out
// [L, H*D] (cudnn_attention.cuh:459 converts V the same way).
struct PrepArgs {
  const float* x[3];        // Q, K, V
  long long ldx[3];
  const float* norm1[2];    // may be NULL (no qk_norm)
  const float* norm2[2];
  __nv_bfloat16* out[3];    // [L, H*D] each
  int norm_split;
  float eps;
  const float* pe;
  int L, H;
};

constexpr int kRowsPerWarp = 2;

// Per 128-key block the softmax warps derive what the key bias holds: kind (bit 0: some keys
// are -inf, i.e. masked, keys past L included; bit 1: some other nonzero value) and, for bit
// 0, a 128-bit mask of the -inf keys (word c, bit i = key 32c+i).  Unmasked blocks skip the
// bias; blocks that are only a 0/-inf mask (the key padding mask) apply it with one select
// per score.
constexpr int kBiasMask = 1, kBiasGeneral = 2;

// kRowsPerWarp Q, K or V rows (token l, head h) of D values starting at `row0`: RMSNorm, RoPE,
// bf16 for Q and K, bf16 for V (see attn_prep_kernel).  All rows' loads are issued before any
// arithmetic.
template <int D>
__device__ __forceinline__ void prep_rows(const PrepArgs& a, long long row0, int lane) {
  constexpr int kPerLane = D / 32;  // 4 (D=128) or 2 (D=64) consecutive values per lane
  const long long per = static_cast<long long>(a.L) * a.H;
  float v[kRowsPerWarp][kPerLane];
  float4 pe[kRowsPerWarp][kPerLane / 2];
  int which[kRowsPerWarp], l[kRowsPerWarp], h[kRowsPerWarp];
#pragma unroll
  for (int rr = 0; rr < kRowsPerWarp; ++rr) {
    const long long row = row0 + rr;
    const bool live = row < 3 * per;
    which[rr] = live ? static_cast<int>(row / per) : 0;
    const long long r = live ? row - which[rr] * per : 0;
    l[rr] = static_cast<int>(r / a.H);
    h[rr] = static_cast<int>(r % a.H);
    // (selects, not indexing: a dynamically indexed parameter array is copied to local memory)
    const int w = which[rr];
    const float* xb = w == 0 ? a.x[0] : (w == 1 ? a.x[1] : a.x[2]);
    const long long ldx = w == 0 ? a.ldx[0] : (w == 1 ? a.ldx[1] : a.ldx[2]);
    const float* xr = xb + l[rr] * ldx + h[rr] * D + lane * kPerLane;
    if constexpr (kPerLane == 4) {
      const float4 t = live ? *reinterpret_cast<const float4*>(xr) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[rr][0] = t.x; v[rr][1] = t.y; v[rr][2] = t.z; v[rr][3] = t.w;
    } else {
      const float2 t = live ? *reinterpret_cast<const float2*>(xr) : make_float2(0.f, 0.f);
      v[rr][0] = t.x; v[rr][1] = t.y;
    }
    const float4* pr = reinterpret_cast<const float4*>(a.pe) + static_cast<long long>(l[rr]) * (D / 2) +
                       lane * kPerLane / 2;
#pragma unroll
    for (int i = 0; i < kPerLane / 2; ++i)
      pe[rr][i] = live && which[rr] < 2 ? __ldg(pr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int rr = 0; rr < kRowsPerWarp; ++rr) {
    if (row0 + rr >= 3 * per) break;
    const int w = which[rr];
    __nv_bfloat16* ob = w == 0 ? a.out[0] : (w == 1 ? a.out[1] : a.out[2]);
    __nv_bfloat16* dst = ob + static_cast<long long>(l[rr]) * a.H * D + h[rr] * D + lane * kPerLane;
    if (w == 2) {  // V: bf16 only
      uint32_t packed[kPerLane / 2];
#pragma unroll
      for (int i = 0; i < kPerLane / 2; ++i) {
        __nv_bfloat162 o = __floats2bfloat162_rn(v[rr][2 * i], v[rr][2 * i + 1]);
        packed[i] = *reinterpret_cast<uint32_t*>(&o);
      }
      if constexpr (kPerLane == 4) *reinterpret_cast<uint2*>(dst) = make_uint2(packed[0], packed[1]);
      else *reinterpret_cast<uint32_t*>(dst) = packed[0];
      continue;
    }
    const float* norm = l[rr] < a.norm_split ? (w == 0 ? a.norm1[0] : a.norm1[1]) : (w == 0 ? a.norm2[0] : a.norm2[1]);
    if (norm) {
      float nv[kPerLane];
      if constexpr (kPerLane == 4) {
        const float4 t4 = __ldg(reinterpret_cast<const float4*>(norm) + lane);
        nv[0] = t4.x; nv[1] = t4.y; nv[2] = t4.z; nv[3] = t4.w;
      } else {
        const float2 t2 = __ldg(reinterpret_cast<const float2*>(norm) + lane);
        nv[0] = t2.x; nv[1] = t2.y;
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < kPerLane; ++i) ss += v[rr][i] * v[rr][i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = rsqrtf(ss / static_cast<float>(D) + a.eps);
#pragma unroll
      for (int i = 0; i < kPerLane; ++i) v[rr][i] = v[rr][i] * inv * nv[i];
    }
    // pair p = lane*kPerLane/2 + i rotates (v[2i], v[2i+1]) by pe row l, group p.
    uint32_t packed[kPerLane / 2];
#pragma unroll
    for (int i = 0; i < kPerLane / 2; ++i) {
      const float4 c = pe[rr][i];
      __nv_bfloat162 o = __floats2bfloat162_rn(v[rr][2 * i] * c.x + v[rr][2 * i + 1] * c.y,
                                               v[rr][2 * i] * c.z + v[rr][2 * i + 1] * c.w);
      packed[i] = *reinterpret_cast<uint32_t*>(&o);
    }
    if constexpr (kPerLane == 4) *reinterpret_cast<uint2*>(dst) = make_uint2(packed[0], packed[1]);
    else *reinterpret_cast<uint32_t*>(dst) = packed[0];
  }
}

template <int D>
__global__ void __launch_bounds__(256, 4) attn_prep_kernel(const PrepArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  prep_rows<D>(a, (static_cast<long long>(blockIdx.x) * 8 + warp) * kRowsPerWarp, lane);
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// A shared-memory int read afresh at every use (volatile asm is neither hoisted nor merged), so
// that a value set once per CTA need not occupy a register across long loops.
__device__ __forceinline__ int ld_shared_volatile(const int* p) {
  int v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
  return v;
}

// ---------------------------------------------------------------------------- fused attention
//
// CTA = (two query tiles A and B of 128 rows = 256 queries, head h), 384 threads:
//   warp 0      TMA: both Q tiles once, then K tile j [128 keys x D] into a 3-deep ring.
//   warp 2      TMA: V tile j [128 keys x D] (as stored) into a 2-deep ring.
//   warp 1      one thread issues tcgen05.mma for both tiles, alternating so the tensor core
//               works for one tile while the other tile's softmax runs:
//                 S_A(0), S_B(0), then per key block j:
//                 O_A += P_A(j) V_j, S_A(j+1), O_B += P_B(j) V_j, S_B(j+1)
//               S = Q K_j^T (M=128, N=128, K=D, both from shared memory) goes to the tile's
//               TMEM S columns; P (bf16 pairs) overwrites the first 64 of them and is the A
//               operand of P.V read straight from TMEM, V_j the MN-major B operand; O
//               accumulates in TMEM.  S(j+1) overwrites P(j) but is issued right behind
//               P(j).V_j without waiting for it: tcgen05.mma operations issued by one thread
//               execute in issue order, so P.V has read P before S is written.  The softmax
//               hands P over in two parts (keys 0-95, then 96-127), so P.V starts on the
//               first 96 keys while the last 32 are still being exponentiated.
//   warp 3      idle (completes the first warpgroup, which runs on 64 registers per thread)
//   warps 4-7   softmax of tile A, warps 8-11 of tile B (216 registers per thread); warp w
//               reads TMEM lanes 32*(w%4)..,
//               one thread per query row:
//               the block's 128 scores in registers (one TMEM load round trip); row max of
//               t = S*log2(e)/sqrt(D) + key_bias_log2; running max m raised only when the
//               block exceeds it by more than 2^8 (then O is rescaled in TMEM: rare);
//               P = 2^(t - m) (ex2.approx) written as bf16 pairs over the S columns; l += sum P.
//               At the end O / l is written in the caller's layout.
// TMEM: tile t at columns [256t, 256t+128) S/P and [256t+128, +D) O: 512 columns.
// Barriers: q_full; k_full[3], k_empty[3] (commit after S_B(j)); v_full[2], v_empty[2]
// (commit after P_B(j).V_j); per tile s_full (commit after S), p_part and p_full (4 softmax
// warps each: keys 0-95 / 96-127 of P written), pv_done (commit after P.V).  Every wait is bounded; on timeout the kernel records the error
// word and winds down.
constexpr int kFaThreads = 384;  // 3 warpgroups
// Registers: launched at 168 per thread (64,512 per CTA); the producer/MMA warpgroup gives
// most of its share to the two softmax warpgroups, which hold a 128-key row in registers:
// 4 x 32 x 64 + 8 x 32 x 216 = 63,488 <= 64,512.
constexpr int kFaRegsIdle = 64;
constexpr int kFaRegsSoftmax = 216;
static_assert(4 * 32 * kFaRegsIdle + 8 * 32 * kFaRegsSoftmax <= kFaThreads * 168, "register split");
constexpr int kFaRows = 128;    // queries per tile
constexpr int kFaTiles = 2;     // query tiles per CTA
constexpr int kFaKeys = 128;    // keys per block
constexpr int kFaKStages = 3;
constexpr int kFaVStages = 2;
constexpr uint32_t kFaBox = 128 * 128;  // bytes of one 128-row x 128-byte swizzled box
constexpr float kFaRescaleLog2 = 8.0f;
// Key blocks whose 128 keys are all masked (bias -inf, or past L) contribute nothing: P = 0
// there, and the running max ignores them.  A CTA lists its live blocks once and runs its loads,
// MMAs and softmax over those only, which gives the same result.  A CTA covers at most
// kFaMaxLive key blocks (64K keys): longer sequences are split into key slices (kv_splits).
constexpr int kFaMaxLive = 512;

template <int D>
struct FaLayout {
  static constexpr uint32_t kQTileBytes = kFaRows * D * 2;  // D/64 boxes
  static constexpr uint32_t kKBytes = kFaKeys * D * 2;      // D/64 boxes
  static constexpr uint32_t kVBytes = kFaKeys * D * 2;      // D/64 boxes, like K
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kK = kQ + kFaTiles * kQTileBytes;
  static constexpr uint32_t kV = kK + kFaKStages * kKBytes;
  static constexpr uint32_t kBars = kV + kFaVStages * kVBytes;
  static constexpr uint32_t kLive = kBars + 256;  // live key-block list (kFaMaxLive uint16) + count
  static constexpr uint32_t kSmem = 1024 + kLive + 2 * kFaMaxLive + 16;
  static constexpr uint32_t kTmemCols = 512;
};

struct FaParams {
  int L;
  int num_kb;             // key blocks of 128
  float scale_log2;       // log2(e) / sqrt(D)
  const float* bias;      // [L] additive key bias (0 / -inf mask or general), NULL: none
  long long bias_stride;  // floats between consecutive sequences' biases (0: one shared bias)
  void* out;
  long long ldo;
  int out_bf16;
  int* err;
  // Key splits (kv_splits > 1, for launches too small to fill the GPU): CTA x covers query
  // pair x / kv_splits and the x % kv_splits-th slice of the key blocks, and stores its
  // unnormalised O and its row statistics (running max m in log2 units, row sum l) instead of
  // the output; attn_combine_kernel then merges the slices.
  int kv_splits;
  int lpad;               // rows per (sequence, head, split) in the partial buffers
  float* part_o;          // [batch][H][kv_splits][lpad][D]
  float2* part_ml;        // [batch][H][kv_splits][lpad]: (m, l)
};

template <int D>
__global__ void __launch_bounds__(kFaThreads, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const FaParams p) {
  using Ly = FaLayout<D>;
  constexpr int KS = kFaKStages, VS = kFaVStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + Ly::kQ;
  uint8_t* sK = smem + Ly::kK;
  uint8_t* sV = smem + Ly::kV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Ly::kBars);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;     // [tile]
  uint64_t* p_full = s_full + kFaTiles;
  uint64_t* pv_done = p_full + kFaTiles;
  uint64_t* drain_bar = pv_done + kFaTiles;
  uint64_t* p_part = drain_bar + 1;    // [tile]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(p_part + kFaTiles);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qpair = static_cast<int>(blockIdx.x) / p.kv_splits;
  const int kslice = static_cast<int>(blockIdx.x) % p.kv_splits;
  const int head = blockIdx.y;
  // Sequence blockIdx.z of a batch stored one after another (rows [z*L, (z+1)*L) of q, k, v
  // and out; keys past L of the last block are masked like any key past L).
  const int row0 = static_cast<int>(blockIdx.z) * p.L;
  const float* key_bias = p.bias ? p.bias + static_cast<long long>(blockIdx.z) * p.bias_stride : nullptr;
  // This CTA's key blocks: [kb0, kb0 + nkb).
  const int kb0 = static_cast<int>(static_cast<long long>(kslice) * p.num_kb / p.kv_splits);
  const int nkb = static_cast<int>(static_cast<long long>(kslice + 1) * p.num_kb / p.kv_splits) - kb0;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int t = 0; t < kFaTiles; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&p_part[t], 4);
      mbar_init(&pv_done[t], 1);
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Ly::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();  // the set-up above overlapped the previous kernel's tail
  griddep_launch_dependents();

  // ---- live key blocks of [kb0, kb0 + nkb): warp w checks blocks w, w + 12, .. (4 keys a lane)
  uint16_t* live = reinterpret_cast<uint16_t*>(smem + Ly::kLive);
  int* live_count = reinterpret_cast<int*>(smem + Ly::kLive + 2 * kFaMaxLive);
  {
    for (int j = warp; j < nkb; j += kFaThreads / 32) {
      bool any = key_bias == nullptr;
      if (!any) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int k = (kb0 + j) * kFaKeys + 32 * c + lane;
          any |= k < p.L && __ldg(key_bias + k) != -INFINITY;
        }
      }
      any = __any_sync(0xffffffffu, any);
      if (lane == 0) live[j] = any ? 1 : 0;
    }
    __syncthreads();
    if (warp == 0) {
      int count = 0;
      for (int base = 0; base < nkb; base += 32) {
        const int j = base + lane;
        const bool f = j < nkb && live[j] != 0;
        const uint32_t m = __ballot_sync(0xffffffffu, f);
        __syncwarp();  // every lane has read its flag before any slot below it is overwritten
        if (f) live[count + __popc(m & ((1u << lane) - 1u))] = static_cast<uint16_t>(j);
        count += __popc(m);
        __syncwarp();
      }
      if (lane == 0) *live_count = count;
    }
    __syncthreads();
  }
  // The number of blocks this CTA runs (read where used: nothing keeps it in a register across
  // the roles' loops); local index j is key block KBLOCK(j).
#define NRUN ld_shared_volatile(live_count)
#define KBLOCK(j) (kb0 + static_cast<int>(live[(j)]))

  if (warp < 4) {
   regs_dec<kFaRegsIdle>();
   if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ TMA producers
    if (lane == 0) {
      const bool is_k = warp == 0;
      const uint64_t shared_kv = policy_evict_last();  // K/V tiles are read by every query pair
      const int stages = is_k ? KS : VS;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      if (is_k) {
        mbar_arrive_expect_tx(q_full, kFaTiles * Ly::kQTileBytes);
        const uint64_t once = policy_evict_first();
#pragma unroll
        for (int t = 0; t < kFaTiles; ++t)
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_3d(sQ + t * Ly::kQTileBytes + c * kFaBox, &tmQ, q_full, c * 64,
                        row0 + (qpair * kFaTiles + t) * kFaRows, head, once);
      }
      int issued = 0;
      for (int j = 0; j < NRUN; ++j) {
        const int st = j % stages;
        if (!mbar_wait(&empty[st], ((j / stages) & 1) ^ 1u, p.err, kErrWaitProducer)) break;
        if (is_k) {
          mbar_arrive_expect_tx(&full[st], Ly::kKBytes);
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_3d(sK + st * Ly::kKBytes + c * kFaBox, &tmK, &full[st], c * 64, row0 + KBLOCK(j) * kFaKeys, head,
                        shared_kv);
        } else {
          mbar_arrive_expect_tx(&full[st], Ly::kVBytes);
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_3d(sV + st * Ly::kVBytes + c * kFaBox, &tmV, &full[st], c * 64, row0 + KBLOCK(j) * kFaKeys, head,
                        shared_kv);
        }
        ++issued;
      }
      // Let this thread's copies land before the CTA's shared memory goes away (they have,
      // unless another role gave up early).
      if (is_k) mbar_wait_drain(q_full, 0);
      for (int j = issued - stages < 0 ? 0 : issued - stages; j < issued; ++j)
        mbar_wait_drain(&full[j % stages], (j / stages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_make(kFmtBF16, kFaRows, kFaKeys);
      constexpr uint32_t idesc_o = idesc_make(kFmtBF16, kFaRows, D) | kIdescBMajorMN;
      bool ok = mbar_wait(q_full, 0, p.err, kErrWaitMma);
      auto issue_s = [&](int t, int j) {  // K_j is loaded
        const uint32_t q0 = smem_u32(sQ + t * Ly::kQTileBytes), k0 = smem_u32(sK + (j % KS) * Ly::kKBytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + t * 256, smem_desc_k_sw128(q0 + c * kFaBox + k * 32),
                     smem_desc_k_sw128(k0 + c * kFaBox + k * 32), idesc_s, (c | k) != 0 ? 1u : 0u);
        umma_commit(&s_full[t]);
        if (t == kFaTiles - 1) umma_commit(&k_empty[j % KS]);  // both tiles have read K_j
      };
      if (ok && NRUN > 0) {  // (a range with no live key block issues nothing)
        tc_fence_after();
        ok = mbar_wait(&k_full[0], 0, p.err, kErrWaitMma);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < kFaTiles; ++t) issue_s(t, 0);
        }
      }
      for (int j = 0; j < NRUN && ok; ++j) {
        const int vs = j % VS;
        for (int t = 0; t < kFaTiles && ok; ++t) {
          const uint32_t v0 = smem_u32(sV + vs * Ly::kVBytes);
          // 16 keys per MMA: P columns 8k.., V rows 16k.. (2 KB step).  Keys 0-95 as soon as the
          // softmax has written them, keys 96-127 when all of P is there.
          if (!(ok = mbar_wait(&p_part[t], j & 1, p.err, kErrWaitMma))) break;
          if (t == 0 && !(ok = mbar_wait(&v_full[vs], (j / VS) & 1, p.err, kErrWaitMma))) break;
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 6; ++k)
            umma_f16_ts(tmem + t * 256 + 128, tmem + t * 256 + 8 * k, smem_desc_mn_sw128(v0 + k * 2048, kFaBox),
                        idesc_o, (j | k) != 0 ? 1u : 0u);
          if (!(ok = mbar_wait(&p_full[t], j & 1, p.err, kErrWaitMma))) break;
          tc_fence_after();
#pragma unroll
          for (int k = 6; k < 8; ++k)
            umma_f16_ts(tmem + t * 256 + 128, tmem + t * 256 + 8 * k, smem_desc_mn_sw128(v0 + k * 2048, kFaBox),
                        idesc_o, 1u);
          umma_commit(&pv_done[t]);
          if (t == kFaTiles - 1) umma_commit(&v_empty[vs]);  // both tiles have read V_j
          if (j + 1 < NRUN) {
            if (t == 0 && !(ok = mbar_wait(&k_full[(j + 1) % KS], ((j + 1) / KS) & 1, p.err, kErrWaitMma))) break;
            // S(j+1) overwrites P(j); issued behind P(j).V_j, which reads P first (issue order).
            issue_s(t, j + 1);
          }
        }
      }
      if (!ok) {
        umma_commit(drain_bar);  // MMAs already issued retire before TMEM is released
        mbar_wait_drain(drain_bar, 0);
      }
    }
   }
  } else {
    regs_inc<kFaRegsSoftmax>();
    // ------------------------------------------------------------ softmax (warps 4..11)
    const int t = (warp - 4) >> 2;            // query tile
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t sbase = tmem + t * 256 + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t obase = sbase + 128;
    float m_used = -INFINITY, l_sum = 0.f;
    bool good = true;
    for (int j = 0; j < NRUN && good; ++j) {
      // The block's key bias, key 32c + lane in kb2[c], in base-2 exponent units (keys past L
      // are -inf); loaded before the wait, which hides the latency.
      float kb2[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int key = KBLOCK(j) * kFaKeys + c * 32 + lane;
        kb2[c] = key < p.L ? (key_bias ? __ldg(key_bias + key) * 1.4426950408889634f : 0.f) : -INFINITY;
      }
      good = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, p.err, kErrWaitEpilogue));
      if (!good) break;
      // Warp votes: the -inf mask words and whether any other nonzero bias is present.
      uint32_t words[4];
      bool other = false;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        words[c] = __ballot_sync(0xffffffffu, kb2[c] == -INFINITY);
        other |= kb2[c] != 0.f && kb2[c] != -INFINITY;
      }
      const bool biased = __any_sync(0xffffffffu, other);
      const int kind = ((words[0] | words[1] | words[2] | words[3]) != 0u ? kBiasMask : 0) |
                       (biased ? kBiasGeneral : 0);
      tc_fence_after();
      // The whole 128-key row in registers: one TMEM round trip per block.  u = raw score
      // (P = 2^(u*scale - m); masked keys set to -inf, giving P = 0) or, for a block with a
      // general bias, scaled score + bias folded in place (P = 2^(u - m)).
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(sbase + c * 32, r[c]);
      tmem_wait_ld();
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (biased) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; i += 4)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float u =
                  fmaf(__uint_as_float(r[c][i + q]), p.scale_log2, __shfl_sync(0xffffffffu, kb2[c], i + q));
              r[c][i + q] = __float_as_uint(u);
              mx4[q] = fmaxf(mx4[q], u);
            }
      } else {
        if (kind & kBiasMask) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if ((words[c] >> i) & 1u) r[c][i] = 0xFF800000u;  // -inf
        }
        // three-input max: two scores per instruction, 16 chains
        float m16[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) m16[q] = fmaxf(__uint_as_float(r[0][q]), __uint_as_float(r[0][q + 16]));
#pragma unroll
        for (int c = 1; c < 4; ++c)
#pragma unroll
          for (int q = 0; q < 16; ++q) m16[q] = max3f(m16[q], __uint_as_float(r[c][q]), __uint_as_float(r[c][q + 16]));
#pragma unroll
        for (int q = 0; q < 4; ++q) mx4[q] = max3f(max3f(m16[4 * q], m16[4 * q + 1], m16[4 * q + 2]), m16[4 * q + 3], mx4[q]);
      }
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      if (!biased) mx *= p.scale_log2;  // scale > 0: the max commutes with it
      const bool raise = mx > m_used + kFaRescaleLog2;
      const float alpha = raise ? fast_exp2(m_used - mx) : 1.f;  // 2^-inf = 0 on the first raise
      if (raise) m_used = mx;
      if (__any_sync(0xffffffffu, raise && j > 0)) {
        // O holds blocks < j: wait for P(j-1).Vt_{j-1}, then scale this row of O.
        good = __all_sync(0xffffffffu, mbar_wait(&pv_done[t], (j - 1) & 1, p.err, kErrWaitEpilogue));
        if (!good) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(obase + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_32x32b_x32(obase + c * 32, o);
        }
      }
      l_sum *= alpha;
      const float neg_m = m_used == -INFINITY ? 0.f : -m_used;
      // P chunk by chunk from the registers: keys 32c..32c+31 become bf16 pairs in columns
      // 16c..16c+15 (S has been read in full above).
      // Packed fp32 pairs (fma/add .f32x2) for the exponent arguments and the row sum: half the
      // instructions of the scalar forms, same per-element rounding.
      const uint64_t ua2 = f2_splat(biased ? 1.f : p.scale_log2), nm2 = f2_splat(neg_m);
      uint64_t ls2[2] = {f2_splat(0.f), f2_splat(0.f)};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 xx = f2_unpack(f2_fma(f2_pack(r[c][i], r[c][i + 1]), ua2, nm2));
          const float e0 = fast_exp2(xx.x);
          const float e1 = fast_exp2(xx.y);
          uint32_t eb0 = __float_as_uint(e0), eb1 = __float_as_uint(e1);
          ls2[(i >> 1) & 1] = f2_add(ls2[(i >> 1) & 1], f2_pack(eb0, eb1));
          __nv_bfloat162 hh = __floats2bfloat162_rn(e0, e1);
          pk[i >> 1] = *reinterpret_cast<uint32_t*>(&hh);
        }
        tmem_st_32x32b_x16(sbase + c * 16, pk);
        if (c == 2) {  // keys 0-95 of P are in TMEM: P.V can start on them
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_part[t]);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
      const float2 la = f2_unpack(ls2[0]), lb = f2_unpack(ls2[1]);
      l_sum += (la.x + la.y) + (lb.x + lb.y);
    }
    // Final: wait for the last P.Vt of this tile, write O / l.
    if (good)
      good = NRUN == 0 || __all_sync(0xffffffffu, mbar_wait(&pv_done[t], (NRUN - 1) & 1, p.err, kErrWaitEpilogue));
    if (good && p.kv_splits > 1) {
      // One key slice: the unnormalised O and (m, l) of each row go to the partial buffers.
      tc_fence_after();
      const bool none = NRUN == 0;
      const int q = (qpair * kFaTiles + t) * kFaRows + row;
      const long long prow = ((static_cast<long long>(blockIdx.z) * gridDim.y + head) * p.kv_splits + kslice) * p.lpad + q;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(obase + c * 32, o);
        tmem_wait_ld();
        if (none) {  // no live key block: O was never written (its TMEM holds anything)
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (q < p.L) {
          float4* dst = reinterpret_cast<float4*>(p.part_o + prow * D + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                 __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
        }
      }
      if (q < p.L) p.part_ml[prow] = make_float2(m_used, l_sum);
    } else if (good) {
      tc_fence_after();
      const int q = (qpair * kFaTiles + t) * kFaRows + row;
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
      const long long col0 = static_cast<long long>(head) * D;
      const bool none = NRUN == 0;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(obase + c * 32, o);
        tmem_wait_ld();
        if (none) {  // no live key block: O was never written (its TMEM holds anything)
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (q < p.L) {
          if (p.out_bf16) {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) +
                                               static_cast<long long>(row0 + q) * p.ldo + col0 + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              __nv_bfloat162 a0 = __floats2bfloat162_rn(__uint_as_float(o[8 * i]) * inv,
                                                        __uint_as_float(o[8 * i + 1]) * inv);
              __nv_bfloat162 a1 = __floats2bfloat162_rn(__uint_as_float(o[8 * i + 2]) * inv,
                                                        __uint_as_float(o[8 * i + 3]) * inv);
              __nv_bfloat162 a2 = __floats2bfloat162_rn(__uint_as_float(o[8 * i + 4]) * inv,
                                                        __uint_as_float(o[8 * i + 5]) * inv);
              __nv_bfloat162 a3 = __floats2bfloat162_rn(__uint_as_float(o[8 * i + 6]) * inv,
                                                        __uint_as_float(o[8 * i + 7]) * inv);
              dst[i] = make_uint4(*reinterpret_cast<uint32_t*>(&a0), *reinterpret_cast<uint32_t*>(&a1),
                                  *reinterpret_cast<uint32_t*>(&a2), *reinterpret_cast<uint32_t*>(&a3));
            }
          } else {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) +
                                                    static_cast<long long>(row0 + q) * p.ldo + col0 + c * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                   __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Ly::kTmemCols);
  }
#undef KBLOCK
#undef NRUN
}

// Merges the key slices of a split launch: for query row q of head h, with slice s holding
// (m_s, l_s) and O_s = sum over its keys of 2^(t - m_s) v, the output is
// sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s, M = max_s m_s (rows with no live key: 0).
// One warp per (sequence, row, head); lane i covers columns [4i, 4i + 4) (D = 128) or
// [2i, 2i + 2) (D = 64).
template <int D>
__global__ void attn_combine_kernel(FaParams p, int H, int batch) {
  griddep_wait();  // launched dependent on the attention kernel: its partials must be complete
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long total = static_cast<long long>(batch) * p.L * H;
  if (w >= total) return;
  const int h = static_cast<int>(w % H);
  const long long zq = w / H;
  const int q = static_cast<int>(zq % p.L), z = static_cast<int>(zq / p.L);
  const long long base = (static_cast<long long>(z) * H + h) * p.kv_splits * p.lpad + q;
  float M = -INFINITY;
  for (int s = 0; s < p.kv_splits; ++s) M = fmaxf(M, p.part_ml[base + static_cast<long long>(s) * p.lpad].x);
  constexpr int kPer = D / 32;
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.f;
  float den = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < p.kv_splits; ++s) {
      const long long r = base + static_cast<long long>(s) * p.lpad;
      const float2 ml = p.part_ml[r];
      if (ml.x == -INFINITY) continue;  // a slice without a live key holds no information
      const float wgt = exp2f(ml.x - M);
      den += wgt * ml.y;
      const float* src = p.part_o + r * D + lane * kPer;
#pragma unroll
      for (int i = 0; i < kPer; ++i) acc[i] += wgt * src[i];
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  const long long orow = static_cast<long long>(z) * p.L + q;
  const long long col = static_cast<long long>(h) * D + lane * kPer;
  if (p.out_bf16) {
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out) + orow * p.ldo + col;
#pragma unroll
    for (int i = 0; i < kPer; i += 2)
      *reinterpret_cast<__nv_bfloat162*>(dst + i) = __floats2bfloat162_rn(acc[i] * inv, acc[i + 1] * inv);
  } else {
    float* dst = static_cast<float*>(p.out) + orow * p.ldo + col;
#pragma unroll
    for (int i = 0; i < kPer; ++i) dst[i] = acc[i] * inv;
  }
}

// Q, K, V bf16 [L, ld] with head h at columns [h*D, (h+1)*D): one 3-D tensor map each
// (D-wide rows, head stride D); rows past L are zero-filled by TMA.
template <int D>
b2g_status launch_flash(const __nv_bfloat16* q, int64_t ldq, const __nv_bfloat16* k, int64_t ldk,
                        const __nv_bfloat16* v, int64_t ldv, const FaParams& fp, int64_t L, int64_t H,
                        int64_t batch, cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  b2g_status s;
  const int64_t rows = L * batch;  // the batch's sequences, one after another
  if ((s = make_operand_map(&tq, q, B2G_BF16, D, rows, ldq, H, D, kFaRows)) != B2G_OK) return s;
  if ((s = make_operand_map(&tk, k, B2G_BF16, D, rows, ldk, H, D, kFaKeys)) != B2G_OK) return s;
  if ((s = make_operand_map(&tv, v, B2G_BF16, D, rows, ldv, H, D, kFaKeys)) != B2G_OK) return s;
  constexpr uint32_t smem = FaLayout<D>::kSmem;
  static_assert(smem <= 227 * 1024, "shared memory budget");
  if ((s = check_cuda(cudaFuncSetAttribute(flash_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem)),
                      "cudaFuncSetAttribute(flash_attn)")) != B2G_OK)
    return s;
  const dim3 grid(static_cast<unsigned>((L + kFaTiles * kFaRows - 1) / (kFaTiles * kFaRows) * fp.kv_splits),
                  static_cast<unsigned>(H), static_cast<unsigned>(batch));
  if ((s = launch_pdl(flash_attn_kernel<D>, grid, dim3(kFaThreads), smem, st, "flash_attn launch", tq, tk, tv, fp)) !=
      B2G_OK)
    return s;
  if (fp.kv_splits <= 1) return B2G_OK;
  const long long warps = batch * L * H;
  return launch_pdl(attn_combine_kernel<D>, dim3(static_cast<unsigned>((warps * 32 + 255) / 256)), dim3(256), 0, st,
                    "attention combine launch", fp, static_cast<int>(H), static_cast<int>(batch));
}

// Shared checks and launch of the fused kernel on bf16 operands.
b2g_status flash_checked(const AttnBf16Args& a, cudaStream_t st) {
  const int64_t L = a.L, H = a.H, D = a.D;
  if (a.out_dtype != B2G_F32 && a.out_dtype != B2G_BF16)
    return set_error(B2G_ERR_UNSUPPORTED, "attention: output must be F32 or BF16");
  const size_t ob = a.out_dtype == B2G_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(a.out) & 15u) != 0 || (a.ldo * ob) % 16 != 0 || a.ldo < H * D)
    return set_error(B2G_ERR_UNSUPPORTED, "attention: output base and row stride must be 16-byte aligned");
  const uintptr_t bits = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                         reinterpret_cast<uintptr_t>(a.v);
  if ((bits & 15u) != 0 || (a.ldq | a.ldk | a.ldv) % 8 != 0 || a.ldq < H * D || a.ldk < H * D || a.ldv < H * D)
    return set_error(B2G_ERR_UNSUPPORTED, "attention: bf16 q, k, v need 16-byte aligned bases and row strides");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  FaParams fp{};
  fp.L = static_cast<int>(L);
  fp.num_kb = static_cast<int>((L + kFaKeys - 1) / kFaKeys);
  fp.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  fp.bias = a.key_bias;
  fp.bias_stride = a.bias_stride;
  fp.out = a.out;
  fp.ldo = a.ldo;
  fp.out_bf16 = a.out_dtype == B2G_BF16 ? 1 : 0;
  fp.err = dev->err_word;
  if (a.batch < 1 || a.batch > 65535 || L * a.batch > (1ll << 30) || a.bias_stride < 0)
    return set_error(B2G_ERR_INVALID, "attention: batch in [1, 65535], batch * L < 2^30, bias stride >= 0");
  // Key splits when the launch fills under half of the SMs (a tensor-parallel rank's few heads):
  // as many slices as keep every CTA on the GPU at once, each of at least 4 key blocks.
  const long long ctas = (L + kFaTiles * kFaRows - 1) / (kFaTiles * kFaRows) * H * a.batch;
  int splits = 1;
  if (g_attn_splits > 0) {
    splits = g_attn_splits;
  } else if (g_attn_splits == 0 && 2 * ctas <= dev->num_sms) {
    splits = static_cast<int>(dev->num_sms / ctas);
  }
  if (splits > fp.num_kb / 4) splits = fp.num_kb / 4;
  if (splits < 1) splits = 1;
  // A CTA lists at most kFaMaxLive key blocks: longer sequences always split.
  if ((fp.num_kb + splits - 1) / splits > kFaMaxLive) splits = (fp.num_kb + kFaMaxLive - 1) / kFaMaxLive;
  fp.kv_splits = splits;
  if (splits > 1) {
    fp.lpad = static_cast<int>(round_up(L, kFaTiles * kFaRows));
    const size_t rows = static_cast<size_t>(a.batch) * H * splits * fp.lpad;
    const size_t o_bytes = round_up(static_cast<int64_t>(rows * D * sizeof(float)), 256);
    void* ws = nullptr;
    if ((s = workspace_get(o_bytes + rows * sizeof(float2), &ws, kWsAttnSplit)) != B2G_OK) return s;
    fp.part_o = static_cast<float*>(ws);
    fp.part_ml = reinterpret_cast<float2*>(static_cast<char*>(ws) + o_bytes);
  }
  if (D == 128) return launch_flash<128>(a.q, a.ldq, a.k, a.ldk, a.v, a.ldv, fp, L, H, a.batch, st);
  return launch_flash<64>(a.q, a.ldq, a.k, a.ldk, a.v, a.ldv, fp, L, H, a.batch, st);
}

}  // namespace

b2g_status attention_bf16(const AttnBf16Args& a, cudaStream_t st) {
  if (a.L <= 0 || a.H <= 0) return B2G_OK;
  if (a.D != 64 && a.D != 128) return set_error(B2G_ERR_UNSUPPORTED, "attention: head dim must be 64 or 128");
  if (a.L > (1ll << 30) || a.H > 65535) return set_error(B2G_ERR_UNSUPPORTED, "attention: size");
  if (!a.q || !a.k || !a.v || !a.out) return set_error(B2G_ERR_INVALID, "attention: null operand");
  return flash_checked(a, st);
}

b2g_status attention_rope_ex(const AttnArgs& a, cudaStream_t st) {
  const int64_t L = a.L, H = a.H, D = a.D;
  if (L <= 0 || H <= 0) return B2G_OK;
  if (D != 64 && D != 128) return set_error(B2G_ERR_UNSUPPORTED, "attention: head dim must be 64 or 128");
  const uintptr_t qkv_bits = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                             reinterpret_cast<uintptr_t>(a.v);
  if ((qkv_bits & 15u) != 0 || (a.ldq | a.ldk | a.ldv) % 4 != 0 || (a.pe && (reinterpret_cast<uintptr_t>(a.pe) & 15u)))
    return set_error(B2G_ERR_UNSUPPORTED, "attention: q, k, v and pe must be 16-byte aligned with row strides % 4 == 0");
  if (!a.pe) return set_error(B2G_ERR_INVALID, "attention: pe is required");
  if (L > (1ll << 30) || H > 65535) return set_error(B2G_ERR_UNSUPPORTED, "attention: size");
  const int64_t HD = H * D;
  const size_t op_bytes = static_cast<size_t>(round_up(L * HD * 2, 256));
  void* ws = nullptr;
  b2g_status s;
  if ((s = workspace_get(3 * op_bytes, &ws, kWsAttention)) != B2G_OK) return s;
  char* base = static_cast<char*>(ws);
  __nv_bfloat16* qb = reinterpret_cast<__nv_bfloat16*>(base);
  __nv_bfloat16* kb = reinterpret_cast<__nv_bfloat16*>(base + op_bytes);
  __nv_bfloat16* vb = reinterpret_cast<__nv_bfloat16*>(base + 2 * op_bytes);

  PrepArgs pa{};
  pa.x[0] = a.q; pa.x[1] = a.k; pa.x[2] = a.v;
  pa.ldx[0] = a.ldq; pa.ldx[1] = a.ldk; pa.ldx[2] = a.ldv;
  pa.norm1[0] = a.q_norm; pa.norm1[1] = a.k_norm;
  pa.norm2[0] = a.q_norm2 ? a.q_norm2 : a.q_norm;
  pa.norm2[1] = a.k_norm2 ? a.k_norm2 : a.k_norm;
  pa.out[0] = qb; pa.out[1] = kb; pa.out[2] = vb;
  pa.norm_split = a.norm_split >= 0 && a.norm_split < L ? static_cast<int>(a.norm_split) : static_cast<int>(L);
  pa.eps = a.eps;
  pa.pe = a.pe;
  pa.L = static_cast<int>(L); pa.H = static_cast<int>(H);
  const unsigned blocks = static_cast<unsigned>((3 * L * H + 8 * kRowsPerWarp - 1) / (8 * kRowsPerWarp));
  s = D == 128 ? launch_pdl(attn_prep_kernel<128>, dim3(blocks), dim3(256), 0, st, "attention prologue kernel", pa)
               : launch_pdl(attn_prep_kernel<64>, dim3(blocks), dim3(256), 0, st, "attention prologue kernel", pa);
  if (s != B2G_OK) return s;

  AttnBf16Args f;
  f.q = qb; f.k = kb; f.v = vb;
  f.ldq = f.ldk = f.ldv = HD;
  f.key_bias = a.key_bias;
  f.out = a.out; f.out_dtype = a.out_dtype; f.ldo = a.ldo;
  f.L = L; f.H = H; f.D = D;
  return flash_checked(f, st);
}

b2g_status attention_rope(const float* q, const float* k, const float* v, const float* pe, const float* key_bias,
                          float* out, int64_t L, int64_t H, int64_t D, cudaStream_t st) {
  AttnArgs a;
  a.q = q; a.k = k; a.v = v;
  a.ldq = a.ldk = a.ldv = H * D;
  a.pe = pe; a.key_bias = key_bias;
  a.out = out; a.out_dtype = B2G_F32; a.ldo = H * D;
  a.L = L; a.H = H; a.D = D;
  return attention_rope_ex(a, st);
}

}  // namespace b2g
