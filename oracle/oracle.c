/*
 * oracle.c — TEST INFRASTRUCTURE ONLY.  A plain-C, fp32 CPU restatement of the reference's
 * GEMM path (cublas_ops.cuh) and of the elementwise kernels that bracket it (kernels.cu),
 * used as the checker by tests/, __graft_entry__.smoke() and bench.py's CPU baseline.
 * Nothing in the engine links or calls this file.
 *
 * Parity of this restatement is pinned against the reference itself: tests/golden/ holds
 * vectors produced by the reference's own linear_lt / linear / batched_matmul_Bt /
 * gelu_to_bf16 / gated_residual, compiled from its sources by oracle/Makefile and run on a
 * B200 (tests/golden/make_golden.py); tests/test_oracle_golden.py checks this file against
 * them.
 *
 * dtype codes follow the reference's DType enum order (tensor.cuh:116): 0 F32, 1 FP16, 2 BF16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { O_F32 = 0, O_F16 = 1, O_BF16 = 2 };

/* ------------------------------------------------------------------ number formats */

static inline float bits_to_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint32_t f32_to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

float oracle_bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

/* Round-to-nearest-even fp32 -> bf16, NaN kept quiet (what __float2bfloat16 does). */
uint16_t oracle_f32_to_bf16(float f) {
  uint32_t u = f32_to_bits(f);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* IEEE binary16 -> fp32 (exact). */
float oracle_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  const uint32_t man = h & 0x3FFu;
  if (exp == 0) {
    if (man == 0) return bits_to_f32(sign);
    float v = (float)man * (1.0f / 16777216.0f); /* man * 2^-24 */
    return sign ? -v : v;
  }
  if (exp == 31) return bits_to_f32(sign | 0x7F800000u | (man << 13));
  return bits_to_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

/* fp32 -> IEEE binary16, round-to-nearest-even, overflow to inf (what __float2half does). */
uint16_t oracle_f32_to_f16(float f) {
  const uint32_t u = f32_to_bits(f);
  const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  const uint32_t aexp = (u >> 23) & 0xFFu;
  uint32_t man = u & 0x7FFFFFu;
  if (aexp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
  const int e = (int)aexp - 127;
  if (e > 15) return (uint16_t)(sign | 0x7C00u);
  if (e >= -14) {
    /* normal half: 10 mantissa bits, drop 13 with RNE */
    uint32_t v = ((uint32_t)(e + 15) << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (v & 1u))) v += 1u; /* may carry into exponent: fine */
    return (uint16_t)(sign | v);
  }
  if (e < -25) return sign; /* below half of the smallest subnormal */
  /* subnormal half: value = m * 2^-24 with m = round(|f| * 2^24) */
  man |= 0x800000u;                  /* 24-bit significand, value = man * 2^(e-23) */
  const int shift = -e - 1;          /* bits to drop so that the unit is 2^-24: (e-23) -> -24 */
  uint32_t v = man >> shift;
  const uint32_t rem = man & ((1u << shift) - 1u);
  const uint32_t half = 1u << (shift - 1);
  if (rem > half || (rem == half && (v & 1u))) v += 1u;
  return (uint16_t)(sign | v);
}

static inline float load_as_f32(const void* base, int dt, int64_t i) {
  if (dt == O_F32) return ((const float*)base)[i];
  if (dt == O_BF16) return oracle_bf16_to_f32(((const uint16_t*)base)[i]);
  return oracle_f16_to_f32(((const uint16_t*)base)[i]);
}

/* dst[i] = value of src[i] as fp32 (src in dtype dt). */
void oracle_to_f32(const void* src, int dt, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = load_as_f32(src, dt, i);
}

/* fp32 rounded to TF32 precision (10 explicit mantissa bits), round to nearest even. */
float oracle_round_tf32(float f) {
  uint32_t u = f32_to_bits(f);
  if ((u & 0x7F800000u) == 0x7F800000u) return f;
  u += 0xFFFu + ((u >> 13) & 1u);
  return bits_to_f32(u & 0xFFFFE000u);
}

enum { O_TF32 = 3 }; /* rounding target only (storage stays fp32) */

/* Round fp32 values to bf16 (dt=2), fp16 (dt=1) or tf32 (dt=3) precision, kept as fp32. */
void oracle_round(const float* src, int dt, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    if (dt == O_BF16) dst[i] = oracle_bf16_to_f32(oracle_f32_to_bf16(src[i]));
    else if (dt == O_F16) dst[i] = oracle_f16_to_f32(oracle_f32_to_f16(src[i]));
    else if (dt == O_TF32) dst[i] = oracle_round_tf32(src[i]);
    else dst[i] = src[i];
  }
}

void oracle_f32_to_bf16_array(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f32_to_bf16(src[i]);
}
void oracle_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f32_to_f16(src[i]);
}

/* ------------------------------------------------------------------ FP8 E4M3
 * E4M3 ("fn" variant): 1 sign, 4 exponent (bias 7), 3 mantissa bits; no infinities;
 * S.1111.111 is NaN; largest finite 448 = 1.75 * 2^8; smallest normal 2^-6; subnormals
 * m/8 * 2^-6.  This restates the format definition (the FP8 formats paper, Micikevicius et
 * al. 2022) with round-to-nearest-even and saturation to +-448, the conversion
 * cvt.rn.satfinite.e4m3x2.f32 performs.  The reference has no FP8 path: the format and the
 * per-row absmax/448 scaling are the engine's FP8 variant as BASELINE's config 5 defines it. */
uint8_t oracle_f32_to_e4m3(float x) {
  const uint32_t u = f32_to_bits(x);
  const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  if (isnan(x)) return 0x7F;
  float a = fabsf(x);
  if (a >= 448.0f) return (uint8_t)(sign | 0x7E); /* saturate (also +-inf) */
  if (a < ldexpf(1.0f, -6)) {
    /* subnormal range: multiples of 2^-9 (q = 8 rounds up into the smallest normal) */
    const float q = rintf(a * 512.0f); /* exact scaling by a power of two, then RNE */
    return (uint8_t)(sign | (uint8_t)q);
  }
  int e;
  frexpf(a, &e); /* a = f * 2^e, f in [0.5, 1): unbiased exponent of a is e - 1 */
  const int ex = e - 1;
  float q = rintf(ldexpf(a, 3 - ex)); /* mantissa with the implicit bit, in [8, 16] */
  int ee = ex;
  if (q >= 16.0f) {
    q = 8.0f;
    ee += 1;
  }
  if (ee > 8 || (ee == 8 && q > 14.0f)) return (uint8_t)(sign | 0x7E);
  return (uint8_t)(sign | (uint8_t)(((ee + 7) << 3) | ((int)q - 8)));
}

float oracle_e4m3_to_f32(uint8_t b) {
  const float sign = (b & 0x80) ? -1.0f : 1.0f;
  const int ex = (b >> 3) & 0xF, m = b & 7;
  if (ex == 0xF && m == 7) return NAN;
  if (ex == 0) return sign * ldexpf((float)m, -9);
  return sign * ldexpf((float)(8 + m), ex - 10);
}

void oracle_f32_to_e4m3_array(const float* src, uint8_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f32_to_e4m3(src[i]);
}
void oracle_e4m3_to_f32_array(const uint8_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_e4m3_to_f32(src[i]);
}

/* Per-row quantisation as the engine defines it: scale_r = absmax_r / 448 (1 when the row is
 * zero), q = E4M3(x * (448 / absmax_r)), all arithmetic in fp32. */
void oracle_quantize_rows_e4m3(const float* src, int64_t rows, int64_t cols, uint8_t* dst, float* scales) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* x = src + r * cols;
    float amax = 0.0f;
    for (int64_t c = 0; c < cols; ++c) amax = fmaxf(amax, fabsf(x[c]));
    const float inv = amax > 0.0f ? 448.0f / amax : 1.0f;
    scales[r] = amax > 0.0f ? amax / 448.0f : 1.0f;
    for (int64_t c = 0; c < cols; ++c) dst[r * cols + c] = oracle_f32_to_e4m3(x[c] * inv);
  }
}

/* ------------------------------------------------------------------ GEMM */

/* out[m, n] = sum_k X[m, k] * W[n, k] over fp32 operands, 16 interleaved fp32 partial sums
 * per dot product (added in a fixed order), 4 rows of X per W row for cache reuse. */
static void gemm_rows_f32(const float* X, int64_t ldx, const float* W, int64_t ldw, float* O, int64_t ldo,
                          int64_t m0, int64_t m1, int64_t n0, int64_t n1, int64_t K) {
  const int64_t K16 = K & ~(int64_t)15;
  int64_t m = m0;
  for (; m + 4 <= m1; m += 4) {
    const float* x0 = X + m * ldx;
    const float* x1 = x0 + ldx;
    const float* x2 = x1 + ldx;
    const float* x3 = x2 + ldx;
    for (int64_t n = n0; n < n1; ++n) {
      const float* w = W + n * ldw;
      float a0[16] = {0}, a1[16] = {0}, a2[16] = {0}, a3[16] = {0};
      for (int64_t k = 0; k < K16; k += 16) {
        for (int l = 0; l < 16; ++l) {
          const float wv = w[k + l];
          a0[l] += x0[k + l] * wv;
          a1[l] += x1[k + l] * wv;
          a2[l] += x2[k + l] * wv;
          a3[l] += x3[k + l] * wv;
        }
      }
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
      for (int l = 0; l < 16; ++l) {
        s0 += a0[l];
        s1 += a1[l];
        s2 += a2[l];
        s3 += a3[l];
      }
      for (int64_t k = K16; k < K; ++k) {
        s0 += x0[k] * w[k];
        s1 += x1[k] * w[k];
        s2 += x2[k] * w[k];
        s3 += x3[k] * w[k];
      }
      O[(m + 0) * ldo + n] = s0;
      O[(m + 1) * ldo + n] = s1;
      O[(m + 2) * ldo + n] = s2;
      O[(m + 3) * ldo + n] = s3;
    }
  }
  for (; m < m1; ++m) {
    const float* x0 = X + m * ldx;
    for (int64_t n = n0; n < n1; ++n) {
      const float* w = W + n * ldw;
      float a0[16] = {0};
      for (int64_t k = 0; k < K16; k += 16)
        for (int l = 0; l < 16; ++l) a0[l] += x0[k + l] * w[k + l];
      float s0 = 0.f;
      for (int l = 0; l < 16; ++l) s0 += a0[l];
      for (int64_t k = K16; k < K; ++k) s0 += x0[k] * w[k];
      O[m * ldo + n] = s0;
    }
  }
}

/*
 * out[M, N] (fp32, row stride ldo) = x[M, K] . w[N, K]^T + bias[N]
 * The arithmetic of the reference's linear_lt (cublas_ops.cuh:214-288): operands of one
 * dtype (F32, FP16 or BF16) read exactly, products and sums in fp32 (CUBLAS_COMPUTE_32F),
 * optional fp32 bias added once per output (CUBLASLT_EPILOGUE_BIAS), fp32 output.
 * nthreads <= 0 uses every core OpenMP offers.  Returns 0, or -1 if memory ran out.
 */
int oracle_linear(int64_t M, int64_t K, int64_t N, const void* x, int xdt, int64_t ldx, const void* w, int wdt,
                  int64_t ldw, const float* bias, float* out, int64_t ldo, int nthreads) {
  if (M <= 0 || N <= 0) return 0;
  float* xf = (float*)malloc(sizeof(float) * (size_t)(M * (K > 0 ? K : 1)));
  float* wf = (float*)malloc(sizeof(float) * (size_t)(N * (K > 0 ? K : 1)));
  if (!xf || !wf) {
    free(xf);
    free(wf);
    return -1;
  }
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
  nthreads = 1;
#endif
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t r = 0; r < M; ++r)
    for (int64_t k = 0; k < K; ++k) xf[r * K + k] = load_as_f32(x, xdt, r * ldx + k);
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t r = 0; r < N; ++r)
    for (int64_t k = 0; k < K; ++k) wf[r * K + k] = load_as_f32(w, wdt, r * ldw + k);

  const int64_t NB = 64; /* W rows per task: 64 x K fp32 stays in L2 */
  const int64_t MB = 256;
  const int64_t n_tasks = (N + NB - 1) / NB;
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1)
  for (int64_t t = 0; t < n_tasks; ++t) {
    const int64_t n0 = t * NB, n1 = (n0 + NB < N) ? n0 + NB : N;
    for (int64_t m0 = 0; m0 < M; m0 += MB) {
      const int64_t m1 = (m0 + MB < M) ? m0 + MB : M;
      gemm_rows_f32(xf, K, wf, K, out, ldo, m0, m1, n0, n1, K);
    }
    if (bias)
      for (int64_t m = 0; m < M; ++m)
        for (int64_t n = n0; n < n1; ++n) out[m * ldo + n] += bias[n];
  }
  free(xf);
  free(wf);
  return 0;
}

/*
 * C[b] = A[b] . B[b]^T, all fp32 [batch, M, K] x [batch, N, K] -> [batch, M, N].
 * The reference's batched_matmul_Bt (cublas_ops.cuh:558-585) runs cuBLAS with
 * CUBLAS_COMPUTE_32F_FAST_16BF.  On B200 that executes as TF32: operands rounded to nearest
 * TF32, products summed in fp32 (tests/golden/batched_matmul_Bt.npz matches that to 2e-7).
 * rounding: 0 exact fp32 operands, 2 (O_BF16) bf16 operands, 3 (O_TF32) tf32 operands.
 */
int oracle_batched_matmul_bt(const float* A, const float* B, float* C, int64_t batch, int64_t M, int64_t K,
                             int64_t N, int rounding, int nthreads) {
  float* ar = (float*)malloc(sizeof(float) * (size_t)(M * K > 0 ? M * K : 1));
  float* br = (float*)malloc(sizeof(float) * (size_t)(N * K > 0 ? N * K : 1));
  if (!ar || !br) {
    free(ar);
    free(br);
    return -1;
  }
  for (int64_t b = 0; b < batch; ++b) {
    const float* a = A + b * M * K;
    const float* bb = B + b * N * K;
    if (rounding) {
      oracle_round(a, rounding, ar, M * K);
      oracle_round(bb, rounding, br, N * K);
    } else {
      memcpy(ar, a, sizeof(float) * (size_t)(M * K));
      memcpy(br, bb, sizeof(float) * (size_t)(N * K));
    }
    oracle_linear(M, K, N, ar, O_F32, K, br, O_F32, K, NULL, C + b * M * N, N, nthreads);
  }
  free(ar);
  free(br);
  return 0;
}

/* ------------------------------------------------------------------ elementwise kernels */

/* tanh GELU, the formula of gelu_val (kernels.cu:266-269). */
static inline float gelu_tanh(float v) {
  const float inner = 0.7978845608f * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner));
}

void oracle_gelu(const float* x, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = gelu_tanh(x[i]);
}

/* gelu_to_bf16 (kernels.cu:297-310): GELU in fp32, then round to bf16. */
void oracle_gelu_to_bf16(const float* x, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f32_to_bf16(gelu_tanh(x[i]));
}

/* gated_residual (kernels.cu:942-968): out[m, c] = x[m, c] + gate[c] * y[m, c]. */
void oracle_gated_residual(const float* x, const float* y, const float* gate, float* out, int64_t M, int64_t C) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t c = 0; c < C; ++c) out[m * C + c] = x[m * C + c] + gate[c] * y[m * C + c];
}

/* modulate (kernels.cu:498-538 / modulate_to_bf16 :552-599): per row, LayerNorm without
 * affine (mean, biased variance, eps), then * (1 + scale[c]) + shift[c]. fp32 out. */
void oracle_modulate(const float* x, const float* shift, const float* scale, float* out, int64_t M, int64_t C,
                     float eps) {
  for (int64_t m = 0; m < M; ++m) {
    const float* xr = x + m * C;
    double s = 0.0;
    for (int64_t c = 0; c < C; ++c) s += xr[c];
    const float mean = (float)(s / (double)C);
    double v = 0.0;
    for (int64_t c = 0; c < C; ++c) {
      const float d = xr[c] - mean;
      v += (double)d * d;
    }
    const float inv = 1.0f / sqrtf((float)(v / (double)C) + eps);
    for (int64_t c = 0; c < C; ++c) out[m * C + c] = (xr[c] - mean) * inv * (1.0f + scale[c]) + shift[c];
  }
}

/* rms_norm (kernels.cu:174-207): out = x / sqrt(mean(x^2) + eps) * scale, per row of C. */
void oracle_rms_norm(const float* x, const float* scale, float* out, int64_t rows, int64_t C, float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    double s = 0.0;
    for (int64_t c = 0; c < C; ++c) s += (double)x[r * C + c] * x[r * C + c];
    const float inv = 1.0f / sqrtf((float)(s / (double)C) + eps);
    for (int64_t c = 0; c < C; ++c) out[r * C + c] = x[r * C + c] * inv * scale[c];
  }
}

/* RoPE on rows of heads, the rotation of apply_rope_fused_bf16 (rope.cuh:180-221) kept in
 * fp32: x [L, H*D], pair j of a head -> (x_e*p0 + x_o*p1, x_e*p2 + x_o*p3) with p = pe[l][j]
 * ([L, D/2, 4]: cos, -sin, sin, cos). */
void oracle_rope(const float* x, const float* pe, float* out, int64_t L, int64_t H, int64_t D) {
  const int64_t half = D / 2;
  for (int64_t l = 0; l < L; ++l)
    for (int64_t h = 0; h < H; ++h)
      for (int64_t j = 0; j < half; ++j) {
        const float* p = pe + (l * half + j) * 4;
        const int64_t i = l * H * D + h * D + 2 * j;
        const float e = x[i], o = x[i + 1];
        out[i] = e * p[0] + o * p[1];
        out[i + 1] = e * p[2] + o * p[3];
      }
}

/*
 * Attention with RoPE, restating cudnn_attention_with_rope (cudnn_attention.cuh:449-476):
 *   Qr, Kr = RoPE(Q), RoPE(K) rounded to bf16 (apply_rope_fused_bf16, rope.cuh:180-221:
 *            out_even = x_e*cos + x_o*(-sin), out_odd = x_e*sin + x_o*cos from pe [L, D/2, 4]);
 *   V rounded to bf16 (permute_and_convert_to_bf16, kernels.cu:3197);
 *   S = Qr.Kr^T / sqrt(D) + mask[key]   (fp32; mask 0 or -inf);
 *   P = softmax(S) rounded to bf16 (flash attention feeds bf16 probabilities to the PV
 *   product); O = P.V in fp32, rounded to bf16 (SDPA writes bf16 O), returned as fp32
 *   [L, H*D] (unpermute_bf16_to_f32, cudnn_attention.cuh:52-77).
 * Q, K, V: [L, H, D] fp32.  Single-threaded over heads (small sizes only).
 */
int oracle_attention_rope(const float* Q, const float* K, const float* V, const float* pe, const float* mask,
                          float* out, int64_t L, int64_t H, int64_t D) {
  const int64_t HD = H * D, half = D / 2;
  float* qr = (float*)malloc(sizeof(float) * (size_t)(L * D));
  float* kr = (float*)malloc(sizeof(float) * (size_t)(L * D));
  float* vr = (float*)malloc(sizeof(float) * (size_t)(L * D));
  float* srow = (float*)malloc(sizeof(float) * (size_t)L);
  if (!qr || !kr || !vr || !srow) {
    free(qr); free(kr); free(vr); free(srow);
    return -1;
  }
  const float scale = 1.0f / sqrtf((float)D);
  for (int64_t h = 0; h < H; ++h) {
    for (int64_t l = 0; l < L; ++l) {
      for (int64_t j = 0; j < half; ++j) {
        const float* p = pe + (l * half + j) * 4;
        const int64_t i = l * HD + h * D + 2 * j;
        const float qe = Q[i], qo = Q[i + 1], ke = K[i], ko = K[i + 1];
        qr[l * D + 2 * j] = oracle_bf16_to_f32(oracle_f32_to_bf16(qe * p[0] + qo * p[1]));
        qr[l * D + 2 * j + 1] = oracle_bf16_to_f32(oracle_f32_to_bf16(qe * p[2] + qo * p[3]));
        kr[l * D + 2 * j] = oracle_bf16_to_f32(oracle_f32_to_bf16(ke * p[0] + ko * p[1]));
        kr[l * D + 2 * j + 1] = oracle_bf16_to_f32(oracle_f32_to_bf16(ke * p[2] + ko * p[3]));
      }
      for (int64_t d = 0; d < D; ++d) vr[l * D + d] = oracle_bf16_to_f32(oracle_f32_to_bf16(V[l * HD + h * D + d]));
    }
    for (int64_t i = 0; i < L; ++i) {
      float mx = -INFINITY;
      for (int64_t j = 0; j < L; ++j) {
        float acc = 0.f;
        for (int64_t d = 0; d < D; ++d) acc += qr[i * D + d] * kr[j * D + d];
        const float sv = acc * scale + (mask ? mask[j] : 0.f);
        srow[j] = sv;
        if (sv > mx) mx = sv;
      }
      double sum = 0.0;
      for (int64_t j = 0; j < L; ++j) {
        srow[j] = (mx == -INFINITY) ? 0.f : expf(srow[j] - mx);
        sum += srow[j];
      }
      const float inv = sum > 0 ? (float)(1.0 / sum) : 0.f;
      for (int64_t j = 0; j < L; ++j) srow[j] = oracle_bf16_to_f32(oracle_f32_to_bf16(srow[j] * inv));
      for (int64_t d = 0; d < D; ++d) {
        float acc = 0.f;
        for (int64_t j = 0; j < L; ++j) acc += srow[j] * vr[j * D + d];
        out[i * HD + h * D + d] = oracle_bf16_to_f32(oracle_f32_to_bf16(acc));
      }
    }
  }
  free(qr); free(kr); free(vr); free(srow);
  return 0;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
