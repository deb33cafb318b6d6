// attention.cu — the Chroma transformer's attention on the tensor cores.
//
// Replaces cudnn_attention_with_rope (cudnn_attention.cuh:449-476): RoPE + bf16 on Q and K
// (apply_rope_fused_bf16, rope.cuh:180-221), V to bf16, softmax(Q K^T / sqrt(D) + key_bias) V
// (cuDNN SDPA, cudnn_attention.cuh:408-443), output F32 [L, H*D] (or bf16 for the block path).
//
//   1. attn_prep         one launch: Q, K F32 rows [L, H*D] -> optional per-head RMSNorm
//                        (qk_norm) -> RoPE -> bf16 [L, H*D] (the attention kernel reads head
//                        h through TMA: row stride H*D, head stride D); V F32 -> bf16
//                        [H, D, L] (K-major operand of P.V); key mask (0 / -inf) scaled by
//                        log2(e), -inf past L, padded to a multiple of 128 keys.
//   2. flash_attn        one CTA per (128-query tile, head): S = Q K^T on the tensor cores
//                        into TMEM, online softmax in registers, P (bf16) through shared
//                        memory into O += P V, O / rowsum written to the output layout.
//                        S never leaves the SM.
#include <cuda_bf16.h>
#include <cstdint>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

namespace {

// Attention prologue, one launch, work items in three ranges of blocks (256 threads each):
//   [0, n_rows)            Q then K rows: one warp per (token l, head h) row of D values:
//                          RMSNorm with a learned scale (rms_norm, kernels.cu:174-207, as
//                          qk_norm applies it, chroma.cuh:513-515; rows l >= norm_split use the
//                          second scale set), RoPE with pe row l = D/2 groups of (cos, -sin,
//                          sin, cos) (the table gen_pe builds, rope.cuh:84, applied as
//                          apply_rope_fused_bf16 does, rope.cuh:180-221), bf16 out [L, H*D].
//   [n_rows, +n_vtiles)    V [L, H*D] F32 -> Vt [H*D, L] bf16 through 64x64 smem tiles.
//   last block             key bias in base-2 exponent units: bias[k]*log2(e) for k < L, -inf
//                          up to the padded key count (keys past L are TMA zero fill).
struct PrepArgs {
  const float* x[2];        // Q, K
  long long ldx[2];
  const float* norm1[2];    // may be NULL (no qk_norm)
  const float* norm2[2];
  __nv_bfloat16* out[2];    // [L, H*D]
  int norm_split;
  float eps;
  const float* pe;
  const float* v;
  long long ldv;
  __nv_bfloat16* vt;        // [H*D, L]
  const float* bias;        // may be NULL
  float* bias_log2;         // [padded]
  int L, H, padded;
  int rows_blocks, vt_cols_tiles, vt_blocks;
};

template <int D>
__global__ void __launch_bounds__(256) attn_prep_kernel(const PrepArgs a) {
  constexpr int kPerLane = D / 32;  // 4 (D=128) or 2 (D=64) consecutive values per lane
  __shared__ float tile[64][65];
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (b < a.rows_blocks) {
    const long long row = static_cast<long long>(b) * 8 + warp;
    const long long per = static_cast<long long>(a.L) * a.H;
    if (row >= 2 * per) return;
    const int which = row >= per ? 1 : 0;
    const long long r = row - which * per;
    const int l = static_cast<int>(r / a.H), h = static_cast<int>(r % a.H);
    const float* xr = a.x[which] + l * a.ldx[which] + h * D + lane * kPerLane;
    float v[kPerLane];
    if constexpr (kPerLane == 4) {
      const float4 t = *reinterpret_cast<const float4*>(xr);
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
      const float2 t = *reinterpret_cast<const float2*>(xr);
      v[0] = t.x; v[1] = t.y;
    }
    const float* norm = l < a.norm_split ? a.norm1[which] : a.norm2[which];
    if (norm) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < kPerLane; ++i) ss += v[i] * v[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = rsqrtf(ss / static_cast<float>(D) + a.eps);
#pragma unroll
      for (int i = 0; i < kPerLane; ++i) v[i] = v[i] * inv * __ldg(norm + lane * kPerLane + i);
    }
    // pair p = lane*kPerLane/2 + i rotates (v[2i], v[2i+1]) by pe row l, group p.
    const float4* pe = reinterpret_cast<const float4*>(a.pe) + static_cast<long long>(l) * (D / 2) + lane * kPerLane / 2;
    uint32_t packed[kPerLane / 2];
#pragma unroll
    for (int i = 0; i < kPerLane / 2; ++i) {
      const float4 c = __ldg(pe + i);
      __nv_bfloat162 o = __floats2bfloat162_rn(v[2 * i] * c.x + v[2 * i + 1] * c.y, v[2 * i] * c.z + v[2 * i + 1] * c.w);
      packed[i] = *reinterpret_cast<uint32_t*>(&o);
    }
    __nv_bfloat16* dst = a.out[which] + static_cast<long long>(l) * a.H * D + h * D + lane * kPerLane;
    if constexpr (kPerLane == 4) *reinterpret_cast<uint2*>(dst) = make_uint2(packed[0], packed[1]);
    else *reinterpret_cast<uint32_t*>(dst) = packed[0];
    return;
  }
  const int vb = b - a.rows_blocks;
  if (vb < a.vt_blocks) {
    const int HD = a.H * D;
    const int l0 = (vb / a.vt_cols_tiles) * 64, c0 = (vb % a.vt_cols_tiles) * 64;
    // read 64 rows (tokens) x 64 columns (features), float4 per thread, 4 passes of 16 rows
    const int tc = (threadIdx.x & 15) * 4, tr = threadIdx.x >> 4;
#pragma unroll
    for (int pass = 0; pass < 4; ++pass) {
      const int rr = pass * 16 + tr, l = l0 + rr;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (l < a.L && c0 + tc < HD) t = *reinterpret_cast<const float4*>(a.v + l * a.ldv + c0 + tc);
      tile[rr][tc] = t.x;
      tile[rr][tc + 1] = t.y;
      tile[rr][tc + 2] = t.z;
      tile[rr][tc + 3] = t.w;
    }
    __syncthreads();
    // write 64 feature rows x 64 tokens, 4 tokens (8 bytes) per thread, 4 passes of 16 rows
#pragma unroll
    for (int pass = 0; pass < 4; ++pass) {
      const int cc = pass * 16 + tr, c = c0 + cc, l = l0 + tc;
      if (c < HD && l < a.L) {
        __nv_bfloat162 p0 = __floats2bfloat162_rn(tile[tc][cc], tile[tc + 1][cc]);
        __nv_bfloat162 p1 = __floats2bfloat162_rn(tile[tc + 2][cc], tile[tc + 3][cc]);
        *reinterpret_cast<uint2*>(a.vt + static_cast<long long>(c) * a.L + l) =
            make_uint2(*reinterpret_cast<uint32_t*>(&p0), *reinterpret_cast<uint32_t*>(&p1));
      }
    }
    return;
  }
  for (int k = threadIdx.x; k < a.padded; k += blockDim.x)
    a.bias_log2[k] = k < a.L ? (a.bias ? a.bias[k] * 1.4426950408889634f : 0.f) : -INFINITY;
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// ---------------------------------------------------------------------------- fused attention
//
// CTA = (query tile of 128 rows, head h), 192 threads:
//   warp 0      TMA producer: Q tile once; K tile j [128 keys x D] and Vt tile j [D x 128
//               keys] into a 2-deep ring (128-byte swizzle, the layout the MMA reads).
//   warp 1      one thread issues tcgen05.mma: S_j = Q K_j^T (M=128, N=128, K=D) into one of
//               two TMEM S buffers, then O += P_j Vt_j^T (M=128, N=D, K=128) into TMEM O.
//               S_{j+1} is issued before P_j is ready, so the tensor core computes the next
//               scores while the softmax warps work on the current ones.
//   warps 2-5   softmax, one thread per query row (warp w reads TMEM lanes 32*(w%4)..):
//               t = S*log2(e)/sqrt(D) + key_bias_log2; running max m (raised only when a
//               block's max exceeds it by more than 8, i.e. a factor 256, so O in TMEM is
//               rescaled rarely); P = 2^(t - m) as bf16 into a swizzled shared-memory tile
//               (double-buffered); l += sum P.  At the end O / l goes to the output.
// Barriers: q_full; k_full[2], v_full[2] (TMA bytes); kv_empty[2] (MMA commit after P_j.Vt_j);
// s_full[2] (MMA commit), s_empty[2] (4 softmax warps); p_full[2] (4 softmax warps),
// p_empty[2] (MMA commit after P_j.Vt_j: P buffer free, and O holds blocks <= j).
// Every wait is bounded; on timeout the kernel records the error word and winds down.
constexpr int kFaThreads = 192;
constexpr int kFaRows = 128;   // queries per CTA
constexpr int kFaKeys = 128;   // keys per block
constexpr uint32_t kFaBox = 128 * 128;  // bytes of one 128-row x 128-byte swizzled box
constexpr float kFaRescaleLog2 = 8.0f;

template <int D>
struct FaLayout {
  static constexpr uint32_t kQBytes = kFaRows * D * 2;   // D/64 boxes
  static constexpr uint32_t kKBytes = kFaKeys * D * 2;   // D/64 boxes
  static constexpr uint32_t kVBytes = D * kFaKeys * 2;   // 2 boxes of D rows x 64 keys
  static constexpr uint32_t kVBox = D * 128;             // one D-row x 64-key box
  static constexpr uint32_t kPBytes = kFaRows * kFaKeys * 2;  // 2 boxes
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kK = kQ + kQBytes;
  static constexpr uint32_t kV = kK + 2 * kKBytes;
  static constexpr uint32_t kP = kV + 2 * kVBytes;
  static constexpr uint32_t kBars = kP + 2 * kPBytes;
  static constexpr uint32_t kSmem = 1024 + kBars + 256;
  static constexpr uint32_t kTmemCols = 512;  // S0 [0,128), S1 [128,256), O [256, 256+D)
};

struct FaParams {
  int L;
  int num_kb;             // key blocks of 128
  float scale_log2;       // log2(e) / sqrt(D)
  const float* bias_log2; // [num_kb * 128]
  void* out;
  long long ldo;
  int out_bf16;
  int* err;
};

template <int D>
__global__ void __launch_bounds__(kFaThreads, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const FaParams p) {
  using Ly = FaLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + Ly::kQ;
  uint8_t* sK = smem + Ly::kK;
  uint8_t* sV = smem + Ly::kV;
  uint8_t* sP = smem + Ly::kP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Ly::kBars);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = bars + 3;
  uint64_t* kv_empty = bars + 5;
  uint64_t* s_full = bars + 7;
  uint64_t* s_empty = bars + 9;
  uint64_t* p_full = bars + 11;
  uint64_t* p_empty = bars + 13;
  uint64_t* drain_bar = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qtile = blockIdx.x;
  const int head = blockIdx.y;
  const int nkb = p.num_kb;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t once = policy_evict_first();
      const uint64_t shared_kv = policy_evict_last();  // K/V tiles are read by every query tile
      mbar_arrive_expect_tx(q_full, Ly::kQBytes);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tma_load_3d(sQ + c * kFaBox, &tmQ, q_full, c * 64, qtile * kFaRows, head, once);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1u, p.err, kErrWaitProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], Ly::kKBytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(sK + st * Ly::kKBytes + c * kFaBox, &tmK, &k_full[st], c * 64, j * kFaKeys, head, shared_kv);
        mbar_arrive_expect_tx(&v_full[st], Ly::kVBytes);
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tma_load_3d(sV + st * Ly::kVBytes + c * Ly::kVBox, &tmV, &v_full[st], j * kFaKeys + c * 64, 0, head,
                      shared_kv);
        ++issued;
      }
      // Let this thread's copies land before the CTA's shared memory goes away (they have,
      // unless another role gave up early): Q and the last two stages.
      mbar_wait_drain(q_full, 0);
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) {
        mbar_wait_drain(&k_full[j & 1], (j >> 1) & 1);
        mbar_wait_drain(&v_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_make(kFmtBF16, kFaRows, kFaKeys);
      constexpr uint32_t idesc_o = idesc_make(kFmtBF16, kFaRows, D);
      bool ok = mbar_wait(q_full, 0, p.err, kErrWaitMma);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1, sb = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, p.err, kErrWaitMma)) return false;
        if (!mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1u, p.err, kErrWaitMma)) return false;
        tc_fence_after();
        const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK + st * Ly::kKBytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + sb * kFaKeys, smem_desc_k_sw128(q0 + c * kFaBox + k * 32),
                     smem_desc_k_sw128(k0 + c * kFaBox + k * 32), idesc_s, (c | k) != 0 ? 1u : 0u);
        umma_commit(&s_full[sb]);
        return true;
      };
      if (ok) {
        tc_fence_after();
        ok = issue_s(0);
      }
      for (int j = 0; j < nkb && ok; ++j) {
        if (j + 1 < nkb && !(ok = issue_s(j + 1))) break;
        const int pb = j & 1, st = j & 1;
        if (!(ok = mbar_wait(&p_full[pb], (j >> 1) & 1, p.err, kErrWaitMma))) break;
        if (!(ok = mbar_wait(&v_full[st], (j >> 1) & 1, p.err, kErrWaitMma))) break;
        tc_fence_after();
        const uint32_t p0 = smem_u32(sP + pb * Ly::kPBytes), v0 = smem_u32(sV + st * Ly::kVBytes);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + 2 * kFaKeys, smem_desc_k_sw128(p0 + c * kFaBox + k * 32),
                     smem_desc_k_sw128(v0 + c * Ly::kVBox + k * 32), idesc_o, (j | c | k) != 0 ? 1u : 0u);
        umma_commit(&kv_empty[st]);
        umma_commit(&p_empty[pb]);
      }
      if (!ok) {
        umma_commit(drain_bar);  // MMAs already issued retire before TMEM is released
        mbar_wait_drain(drain_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax (warps 2..5)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    float m_used = -INFINITY, l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int sb = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (j >> 1) & 1, p.err, kErrWaitEpilogue));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(lane_base + sb * kFaKeys + c * 32, r[c]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);  // the MMA warp may overwrite this S buffer

      const float* bias = p.bias_log2 + j * kFaKeys;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 b = __ldg(reinterpret_cast<const float4*>(bias + c * 32 + i));
          const float t0 = fmaf(__uint_as_float(r[c][i]), p.scale_log2, b.x);
          const float t1 = fmaf(__uint_as_float(r[c][i + 1]), p.scale_log2, b.y);
          const float t2 = fmaf(__uint_as_float(r[c][i + 2]), p.scale_log2, b.z);
          const float t3 = fmaf(__uint_as_float(r[c][i + 3]), p.scale_log2, b.w);
          r[c][i] = __float_as_uint(t0);
          r[c][i + 1] = __float_as_uint(t1);
          r[c][i + 2] = __float_as_uint(t2);
          r[c][i + 3] = __float_as_uint(t3);
          mx = fmaxf(mx, fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)));
        }
      }
      // Raise the running max only when this block exceeds it by more than a factor 2^8.
      const bool raise = mx > m_used + kFaRescaleLog2;
      const float alpha = raise ? fast_exp2(m_used - mx) : 1.f;  // 2^-inf = 0 on the first raise
      if (raise) m_used = mx;
      if (__any_sync(0xffffffffu, raise && j > 0)) {
        // O holds blocks < j: wait for P_{j-1}.Vt_{j-1}, then scale this row of O by alpha.
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&p_empty[(j - 1) & 1], ((j - 1) >> 1) & 1, p.err, kErrWaitEpilogue));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(lane_base + 2 * kFaKeys + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_32x32b_x32(lane_base + 2 * kFaKeys + c * 32, o);
        }
        tmem_wait_st();
      }
      l_sum *= alpha;
      const float m_ref = m_used == -INFINITY ? 0.f : m_used;

      // P_j into shared-memory buffer pb once P_{j-2}.Vt_{j-2} has read it.
      const int pb = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[pb], ((j >> 1) & 1) ^ 1u, p.err, kErrWaitEpilogue));
      if (!ok) break;
      uint8_t* prow = sP + pb * Ly::kPBytes + row * 128;
#pragma unroll
      for (int g = 0; g < 16; ++g) {  // 16-byte groups of 8 keys; box g/8, swizzled chunk g%8
        const int c = g >> 2, i0 = (g & 3) * 8;
        float e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          e[i] = fast_exp2(__uint_as_float(r[c][i0 + i]) - m_ref);
          l_sum += e[i];
        }
        uint4 v;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(e[0], e[1]), h1 = __floats2bfloat162_rn(e[2], e[3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(e[4], e[5]), h3 = __floats2bfloat162_rn(e[6], e[7]);
        v.x = *reinterpret_cast<uint32_t*>(&h0);
        v.y = *reinterpret_cast<uint32_t*>(&h1);
        v.z = *reinterpret_cast<uint32_t*>(&h2);
        v.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(prow + (g >> 3) * kFaBox + (((g & 7) ^ (row & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core's reads
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[pb]);
    }
    if (ok && nkb > 0) {
      const int jl = nkb - 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[jl & 1], (jl >> 1) & 1, p.err, kErrWaitEpilogue));
      if (ok) {
        tc_fence_after();
        const int q = qtile * kFaRows + row;
        const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
        const long long col0 = static_cast<long long>(head) * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(lane_base + 2 * kFaKeys + c * 32, o);
          tmem_wait_ld();
          if (q < p.L) {
            if (p.out_bf16) {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + q * p.ldo + col0 + c * 32);
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
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + q * p.ldo + col0 + c * 32);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                     __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
            }
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
}

template <int D>
b2g_status launch_flash(const __nv_bfloat16* qb, const __nv_bfloat16* kb, const __nv_bfloat16* vt, const FaParams& fp,
                        int64_t L, int64_t H, cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  b2g_status s;
  const int64_t HD = H * D;
  if ((s = make_operand_map(&tq, qb, B2G_BF16, D, L, HD, H, D, kFaRows)) != B2G_OK) return s;
  if ((s = make_operand_map(&tk, kb, B2G_BF16, D, L, HD, H, D, kFaKeys)) != B2G_OK) return s;
  if ((s = make_operand_map(&tv, vt, B2G_BF16, L, D, L, H, D * L, D)) != B2G_OK) return s;
  constexpr uint32_t smem = FaLayout<D>::kSmem;
  static_assert(smem <= 227 * 1024, "shared memory budget");
  if ((s = check_cuda(cudaFuncSetAttribute(flash_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem)),
                      "cudaFuncSetAttribute(flash_attn)")) != B2G_OK)
    return s;
  const dim3 grid(static_cast<unsigned>((L + kFaRows - 1) / kFaRows), static_cast<unsigned>(H));
  flash_attn_kernel<D><<<grid, kFaThreads, smem, st>>>(tq, tk, tv, fp);
  note_launch();
  return check_cuda(cudaGetLastError(), "flash_attn launch");
}


}  // namespace

b2g_status attention_rope_ex(const AttnArgs& a, cudaStream_t st) {
  const int64_t L = a.L, H = a.H, D = a.D;
  if (L <= 0 || H <= 0) return B2G_OK;
  if (D != 64 && D != 128) return set_error(B2G_ERR_UNSUPPORTED, "attention: head dim must be 64 or 128");
  // 16-byte TMA row strides for Vt (rows are L long); 16-byte row loads of Q, K and V.
  if (L % 8 != 0) return set_error(B2G_ERR_UNSUPPORTED, "attention: sequence length must be a multiple of 8");
  const uintptr_t qkv_bits = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                             reinterpret_cast<uintptr_t>(a.v);
  if ((qkv_bits & 15u) != 0 || (a.ldq | a.ldk | a.ldv) % 4 != 0 || (a.pe && (reinterpret_cast<uintptr_t>(a.pe) & 15u)))
    return set_error(B2G_ERR_UNSUPPORTED, "attention: q, k, v and pe must be 16-byte aligned with row strides % 4 == 0");
  if (L > (1ll << 30) || H > 65535) return set_error(B2G_ERR_UNSUPPORTED, "attention: size");
  if (a.out_dtype != B2G_F32 && a.out_dtype != B2G_BF16)
    return set_error(B2G_ERR_UNSUPPORTED, "attention: output must be F32 or BF16");
  const size_t ob = a.out_dtype == B2G_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(a.out) & 15u) != 0 || (a.ldo * ob) % 16 != 0)
    return set_error(B2G_ERR_UNSUPPORTED, "attention: output base and row stride must be 16-byte aligned");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const int64_t HD = H * D;
  const int64_t nkb = (L + kFaKeys - 1) / kFaKeys;
  const size_t qk_bytes = static_cast<size_t>(round_up(L * HD * 2, 256));
  const size_t vt_bytes = static_cast<size_t>(round_up(HD * L * 2, 256));
  const size_t bias_bytes = static_cast<size_t>(round_up(nkb * kFaKeys * 4, 256));
  void* ws = nullptr;
  if ((s = workspace_get(2 * qk_bytes + vt_bytes + bias_bytes, &ws, kWsAttention)) != B2G_OK) return s;
  char* base = static_cast<char*>(ws);
  __nv_bfloat16* qb = reinterpret_cast<__nv_bfloat16*>(base);
  __nv_bfloat16* kb = reinterpret_cast<__nv_bfloat16*>(base + qk_bytes);
  __nv_bfloat16* vt = reinterpret_cast<__nv_bfloat16*>(base + 2 * qk_bytes);
  float* bias_log2 = reinterpret_cast<float*>(base + 2 * qk_bytes + vt_bytes);

  // The V tiles write 4 tokens (8 bytes) per thread and read float4 rows.
  PrepArgs pa{};
  pa.x[0] = a.q; pa.x[1] = a.k;
  pa.ldx[0] = a.ldq; pa.ldx[1] = a.ldk;
  pa.norm1[0] = a.q_norm; pa.norm1[1] = a.k_norm;
  pa.norm2[0] = a.q_norm2 ? a.q_norm2 : a.q_norm;
  pa.norm2[1] = a.k_norm2 ? a.k_norm2 : a.k_norm;
  pa.out[0] = qb; pa.out[1] = kb;
  pa.norm_split = a.norm_split >= 0 && a.norm_split < L ? static_cast<int>(a.norm_split) : static_cast<int>(L);
  pa.eps = a.eps;
  pa.pe = a.pe;
  pa.v = a.v; pa.ldv = a.ldv; pa.vt = vt;
  pa.bias = a.key_bias; pa.bias_log2 = bias_log2;
  pa.L = static_cast<int>(L); pa.H = static_cast<int>(H);
  pa.padded = static_cast<int>(nkb * kFaKeys);
  pa.rows_blocks = static_cast<int>((2 * L * H + 7) / 8);
  pa.vt_cols_tiles = static_cast<int>((HD + 63) / 64);
  pa.vt_blocks = static_cast<int>((L + 63) / 64) * pa.vt_cols_tiles;
  const unsigned blocks = static_cast<unsigned>(pa.rows_blocks + pa.vt_blocks + 1);
  if (D == 128) attn_prep_kernel<128><<<blocks, 256, 0, st>>>(pa);
  else attn_prep_kernel<64><<<blocks, 256, 0, st>>>(pa);
  note_launch();
  if ((s = check_cuda(cudaGetLastError(), "attention prologue kernel")) != B2G_OK) return s;

  FaParams fp{};
  fp.L = static_cast<int>(L);
  fp.num_kb = static_cast<int>(nkb);
  fp.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  fp.bias_log2 = bias_log2;
  fp.out = a.out;
  fp.ldo = a.ldo;
  fp.out_bf16 = a.out_dtype == B2G_BF16 ? 1 : 0;
  fp.err = dev->err_word;
  if (D == 128) return launch_flash<128>(qb, kb, vt, fp, L, H, st);
  return launch_flash<64>(qb, kb, vt, fp, L, H, st);
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
