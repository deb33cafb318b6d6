// capi.cu — the extern "C" entry points of libb2g.so (declared in include/b2g.h), plus the
// library state they share: last-error message, per-device info, the device error word
// and the cast workspace.
#include <cuda_runtime.h>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <string>
#include "engine.cuh"

namespace b2g {

namespace {

// Kernels OR a role code in here when a pipeline wait exceeds its limit (ptx_sm100.cuh).
__device__ int g_device_error_word = 0;

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];

struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
  int device = -1;
};
Workspace g_ws[kMaxDevices][kWsSlots];

b2g_dtype from_cuda_type(cudaDataType_t t, bool* ok) {
  *ok = true;
  switch (t) {
    case CUDA_R_32F: return B2G_F32;
    case CUDA_R_16F: return B2G_F16;
    case CUDA_R_16BF: return B2G_BF16;
    default: *ok = false; return B2G_F32;
  }
}


int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace

b2g_status set_error(b2g_status st, const std::string& msg) {
  g_last_error = msg;
  return st;
}

b2g_status check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return B2G_OK;
  return set_error(B2G_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

void note_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("B2G_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

b2g_status device_info(DeviceInfo** out) {
  int dev = -1;
  b2g_status s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (s != B2G_OK) return s;
  if (dev < 0 || dev >= kMaxDevices) return set_error(B2G_ERR_NO_DEVICE, "device ordinal out of range");
  DeviceInfo& d = g_devices[dev];
  if (d.device != dev) {
    cudaDeviceProp prop;
    if ((s = check_cuda(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties")) != B2G_OK) return s;
    if (prop.major != 10 || prop.minor != 0)
      return set_error(B2G_ERR_NO_DEVICE, "device " + std::to_string(dev) + " is sm_" + std::to_string(prop.major) +
                                              std::to_string(prop.minor) + "; this library is built for sm_100a only");
    void* ew = nullptr;
    if ((s = check_cuda(cudaGetSymbolAddress(&ew, g_device_error_word), "cudaGetSymbolAddress(error word)")) != B2G_OK)
      return s;
    d.num_sms = prop.multiProcessorCount;
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    d.err_word = static_cast<int*>(ew);
    d.device = dev;
  }
  *out = &d;
  return B2G_OK;
}

b2g_status workspace_get(size_t bytes, void** ptr, int slot) {
  int dev = -1;
  b2g_status s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (s != B2G_OK) return s;
  Workspace& w = g_ws[dev][slot];
  if (w.bytes < bytes) {
    if (w.ptr) {
      // The old buffer may still be read by queued kernels.
      if ((s = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize (workspace grow)")) != B2G_OK) return s;
      cudaFree(w.ptr);
      w.ptr = nullptr;
      w.bytes = 0;
    }
    const size_t want = static_cast<size_t>(round_up(static_cast<int64_t>(bytes), 1 << 20));
    if ((s = check_cuda(cudaMalloc(&w.ptr, want), "cudaMalloc (workspace)")) != B2G_OK) return s;
    if (slot == kWsCounters && (s = check_cuda(cudaMemset(w.ptr, 0, want), "cudaMemset (counters)")) != B2G_OK)
      return s;
    w.bytes = want;
    w.device = dev;
  }
  *ptr = w.ptr;
  return B2G_OK;
}

void workspace_release() {
  for (auto& per_dev : g_ws) {
    for (auto& w : per_dev) {
      if (w.ptr) {
        int cur = -1;
        cudaGetDevice(&cur);
        cudaSetDevice(w.device);
        cudaDeviceSynchronize();
        cudaFree(w.ptr);
        cudaSetDevice(cur);
      }
      w = Workspace{};
    }
  }
}

// Runs one (possibly batched) GEMM, converting F32 activations to the weight dtype first
// when the weights are 16-bit, exactly as linear() does before calling cuBLASLt.
b2g_status run_gemm(GemmProblem p, cudaStream_t st) {
  if (p.M == 0 || p.N == 0 || p.batch == 0) return B2G_OK;
  if (p.a_dtype == B2G_F32 && (p.b_dtype == B2G_BF16 || p.b_dtype == B2G_F16) && p.K > 0) {
    const int64_t kp = round_up(p.K, 8);  // TMA row stride must be a multiple of 16 bytes
    void* ws = nullptr;
    b2g_status s = workspace_get(static_cast<size_t>(p.batch * p.M * kp) * 2, &ws);
    if (s != B2G_OK) return s;
    s = cast_f32_to_16(static_cast<const float*>(p.a), ws, p.b_dtype, p.batch, p.M, p.K, p.lda,
                       p.batch > 1 ? p.a_bstride : 0, kp, p.M * kp, st);
    if (s != B2G_OK) return s;
    p.a = ws;
    p.a_dtype = p.b_dtype;
    p.lda = kp;
    p.a_bstride = p.M * kp;
  }
  if (p.K > 0 && tc_gemm_supported(p, nullptr)) return tc_gemm_launch(p, st);
  return simt_gemm_launch(p, st);
}

}  // namespace b2g

using namespace b2g;

extern "C" {

b2g_status b2g_init(void) {
  DeviceInfo* d = nullptr;
  return device_info(&d);
}

b2g_status b2g_shutdown(void) {
  workspace_release();
  noalloc_forget();
  return B2G_OK;
}

const char* b2g_last_error(void) { return g_last_error.c_str(); }

const char* b2g_version(void) { return "b2g 0.1 (sm_100a tcgen05)"; }

uint64_t b2g_launch_count(void) { return g_launches.load(); }

b2g_status b2g_set_attention_splits(int splits) {
  if (splits < -1 || splits > 16) return set_error(B2G_ERR_INVALID, "b2g_set_attention_splits: splits in [-1, 16]");
  g_attn_splits = splits;
  return B2G_OK;
}

b2g_status b2g_set_gemm_variant(int variant, int splits) {
  if (variant < -1 || variant > 2) return set_error(B2G_ERR_INVALID, "b2g_set_gemm_variant: variant in [-1, 2]");
  if (splits < -16 || splits > 16) return set_error(B2G_ERR_INVALID, "b2g_set_gemm_variant: splits in [-16, 16]");
  tc_gemm_set_variant(variant, 1, splits);
  return B2G_OK;
}

}  // extern "C"

namespace b2g {

// Checks one descriptor (the rules of b2g_gemm) and fills the internal problem.
// *empty = true for an M == 0 or N == 0 problem (nothing to do).
b2g_status desc_to_problem(const b2g_gemm_desc* d, const char* who, GemmProblem* p, bool* empty) {
  const std::string w(who);
  *empty = false;
  if (!d) return set_error(B2G_ERR_INVALID, w + ": null descriptor");
  if (d->M < 0 || d->N < 0 || d->K < 0) return set_error(B2G_ERR_INVALID, w + ": negative size");
  if (d->M == 0 || d->N == 0) {
    *empty = true;
    return B2G_OK;
  }
  if (!d->d || (d->K > 0 && (!d->a || !d->b))) return set_error(B2G_ERR_INVALID, w + ": null operand");
  if (d->K > 0 && (d->lda < d->K || d->ldb < d->K)) return set_error(B2G_ERR_INVALID, w + ": lda/ldb < K");
  if (d->ldd < d->N) return set_error(B2G_ERR_INVALID, w + ": ldd < N");
  if (d->epilogue == B2G_EPI_GATED_RESIDUAL && (!d->gate || d->d_dtype != B2G_F32))
    return set_error(B2G_ERR_INVALID, w + ": gated residual needs a gate and an F32 output");
  if (d->epilogue < B2G_EPI_NONE || d->epilogue > B2G_EPI_SILU)
    return set_error(B2G_ERR_UNSUPPORTED, w + ": unknown epilogue");
  if (d->a_dtype == B2G_E4M3 || d->b_dtype == B2G_E4M3 || d->d_dtype == B2G_E4M3)
    return set_error(B2G_ERR_UNSUPPORTED, w + ": E4M3 operands are not implemented");
  const bool ab16 = d->b_dtype == B2G_BF16 || d->b_dtype == B2G_F16;
  if (!(d->a_dtype == d->b_dtype || (d->a_dtype == B2G_F32 && ab16)))
    return set_error(B2G_ERR_UNSUPPORTED, w + ": unsupported operand dtype combination");
  p->M = d->M; p->N = d->N; p->K = d->K;
  p->a = d->a; p->a_dtype = d->a_dtype; p->lda = d->lda;
  p->b = d->b; p->b_dtype = d->b_dtype; p->ldb = d->ldb;
  p->bias = d->bias; p->bias_dtype = d->bias_dtype;
  p->d = d->d; p->d_dtype = d->d_dtype; p->ldd = d->ldd;
  p->epilogue = d->epilogue;
  p->gate = d->gate;
  return B2G_OK;
}

namespace {

// desc_to_problem for a problem on E4M3 operands: both a and b E4M3 (activations already
// quantised per row) with their per-row (a_scale) and per-output-channel (b_scale) scales.
b2g_status fp8_desc_to_problem(const b2g_gemm_desc* d, const float* a_scale, const float* b_scale, const char* who,
                               GemmProblem* p, bool* empty) {
  const std::string w(who);
  if (!d) return set_error(B2G_ERR_INVALID, w + ": null descriptor");
  if (d->a_dtype != B2G_E4M3 || d->b_dtype != B2G_E4M3)
    return set_error(B2G_ERR_UNSUPPORTED, w + ": E4M3 activations and weights expected");
  if (!a_scale || !b_scale) return set_error(B2G_ERR_INVALID, w + ": E4M3 operands need row and column scales");
  if (d->d_dtype == B2G_E4M3) return set_error(B2G_ERR_UNSUPPORTED, w + ": E4M3 output is not implemented");
  b2g_gemm_desc dd = *d;  // the checks of the 16-bit path, on a descriptor with bf16 operand tags
  dd.a_dtype = dd.b_dtype = B2G_BF16;
  b2g_status s = desc_to_problem(&dd, who, p, empty);
  if (s != B2G_OK || *empty) return s;
  if (p->K == 0) return set_error(B2G_ERR_INVALID, w + ": K must be positive");
  p->a_dtype = p->b_dtype = B2G_E4M3;
  p->a_scale = a_scale;
  p->b_scale = b_scale;
  return B2G_OK;
}

}  // namespace
}  // namespace b2g

extern "C" {

b2g_status b2g_gemm(const b2g_gemm_desc* d, void* stream) {
  GemmProblem p;
  bool empty = false;
  b2g_status s = desc_to_problem(d, "b2g_gemm", &p, &empty);
  if (s != B2G_OK || empty) return s;
  DeviceInfo* dev = nullptr;
  if ((s = device_info(&dev)) != B2G_OK) return s;
  return run_gemm(p, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_gemm_group(const b2g_gemm_desc* descs, int count, void* stream) {
  if (count < 0 || (count > 0 && !descs)) return set_error(B2G_ERR_INVALID, "b2g_gemm_group: bad descriptor array");
  GemmProblem ps[kMaxGemmGroups];
  int n = 0;
  bool all_empty = true;
  for (int i = 0; i < count; ++i) {
    GemmProblem p;
    bool empty = false;
    b2g_status s = desc_to_problem(descs + i, "b2g_gemm_group", &p, &empty);
    if (s != B2G_OK) return s;
    if (!empty) {
      all_empty = false;
      if (n < kMaxGemmGroups) ps[n] = p;
      ++n;
    }
  }
  if (all_empty) return B2G_OK;
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Problems that read the same F32 activations against 16-bit weights (the T5 layer's q, k,
  // v and its wi_0, wi_1 linears, t5.cuh:233-275, each of which linear() casts on its own) share
  // one cast into the workspace, then run as 16-bit problems.
  bool shared_cast = n >= 2 && n <= kMaxGemmGroups && ps[0].a_dtype == B2G_F32 && ps[0].K > 0 &&
                     (ps[0].b_dtype == B2G_BF16 || ps[0].b_dtype == B2G_F16) && ps[0].batch == 1;
  for (int i = 1; shared_cast && i < n; ++i)
    shared_cast = ps[i].a == ps[0].a && ps[i].a_dtype == B2G_F32 && ps[i].lda == ps[0].lda && ps[i].M == ps[0].M &&
                  ps[i].K == ps[0].K && ps[i].b_dtype == ps[0].b_dtype && ps[i].batch == 1;
  if (shared_cast) {
    const int64_t kp = round_up(ps[0].K, 8);
    void* ws = nullptr;
    if ((s = workspace_get(static_cast<size_t>(ps[0].M * kp) * 2, &ws)) != B2G_OK) return s;
    if ((s = cast_f32_to_16(static_cast<const float*>(ps[0].a), ws, ps[0].b_dtype, 1, ps[0].M, ps[0].K, ps[0].lda,
                            0, kp, ps[0].M * kp, st)) != B2G_OK)
      return s;
    for (int i = 0; i < n; ++i) {
      ps[i].a = ws;
      ps[i].a_dtype = ps[0].b_dtype;
      ps[i].lda = kp;
    }
    bool one = true;
    for (int i = 0; one && i < n; ++i) one = tc_gemm_supported(ps[i], nullptr) && tc_gemm_groupable(ps[0], ps[i]);
    if (one) return tc_gemm_launch_group(ps, n, st);
    for (int i = 0; i < n; ++i)
      if ((s = run_gemm(ps[i], st)) != B2G_OK) return s;
    return B2G_OK;
  }
  // One launch when the (two to four) non-empty problems run on the tensor cores without an
  // activation cast and agree on everything but M and their pointers; otherwise one GEMM
  // after the other on the stream.
  bool one_launch = n >= 2 && n <= kMaxGemmGroups && ps[0].K > 0;
  for (int i = 0; one_launch && i < n; ++i)
    one_launch = tc_gemm_supported(ps[i], nullptr) && tc_gemm_groupable(ps[0], ps[i]);
  if (one_launch) return tc_gemm_launch_group(ps, n, st);
  for (int i = 0; i < count; ++i) {
    GemmProblem p;
    bool empty = false;
    if ((s = desc_to_problem(descs + i, "b2g_gemm_group", &p, &empty)) != B2G_OK) return s;
    if (!empty && (s = run_gemm(p, st)) != B2G_OK) return s;
  }
  return B2G_OK;
}

b2g_status b2g_gemm_tp_reduce(const b2g_gemm_desc* descs, const int64_t* row0, int count,
                              const b2g_tp_reduce_desc* tp, void* stream) {
  if (!descs || !row0 || !tp || count < 1 || count > 2)
    return set_error(B2G_ERR_INVALID, "b2g_gemm_tp_reduce: 1 or 2 descriptors, row offsets and a tp descriptor");
  GemmProblem ps[2];
  TpReduce t;
  t.world = tp->world; t.rank = tp->rank;
  t.part_ptrs = tp->part_ptrs; t.res_ptrs = tp->res_ptrs;
  t.ld_part = tp->ld_part; t.ld_res = tp->ld_res;
  t.counters = tp->counters; t.counter_slots = tp->counter_slots;
  for (int i = 0; i < count; ++i) {
    const b2g_gemm_desc* d = descs + i;
    if (d->M < 0 || d->N <= 0 || d->K <= 0) return set_error(B2G_ERR_INVALID, "b2g_gemm_tp_reduce: sizes");
    if (!d->a || !d->b || !d->gate) return set_error(B2G_ERR_INVALID, "b2g_gemm_tp_reduce: null operand or gate");
    if (d->lda < d->K || d->ldb < d->K) return set_error(B2G_ERR_INVALID, "b2g_gemm_tp_reduce: lda/ldb < K");
    if (d->a_dtype != d->b_dtype || (d->a_dtype != B2G_BF16 && d->a_dtype != B2G_F16))
      return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_tp_reduce: bf16 or fp16 operands of one type");
    if (d->bias && d->bias_dtype != B2G_F32) return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_tp_reduce: F32 bias");
    GemmProblem& p = ps[i];
    p.M = d->M; p.N = d->N; p.K = d->K;
    p.a = d->a; p.a_dtype = d->a_dtype; p.lda = d->lda;
    p.b = d->b; p.b_dtype = d->b_dtype; p.ldb = d->ldb;
    p.bias = d->bias; p.bias_dtype = B2G_F32;
    p.d = nullptr; p.d_dtype = B2G_F32; p.ldd = d->N;
    p.epilogue = static_cast<b2g_epilogue>(kEpiTpReduce);
    p.gate = d->gate;
    p.tp = &t;
    p.tp_row0 = row0[i];
  }
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  for (int i = 0; i < count; ++i)
    if (!tc_gemm_supported(ps[i], nullptr))
      return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_tp_reduce: operands not supported by the tensor-core path");
  return tc_gemm_launch_group(ps, count, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_tp_push_rows(const void* part, void* const* recv_ptrs, int64_t rows, int64_t N, int world, int rank,
                            void* stream) {
  return tp_push_rows(part, recv_ptrs, rows, N, world, rank, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_tp_push_sums(void* const* sum_ptrs, int64_t rows, int64_t N, int world, int rank, void* stream) {
  return tp_push_sums(sum_ptrs, rows, N, world, rank, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_tp_scatter_rows(const void* part, void* const* recv_ptrs, int64_t rows, int64_t N, int world,
                               int rank, void* stream) {
  return tp_scatter_rows(part, recv_ptrs, rows, N, world, rank, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_tp_reduce_slots_bcast(const void* recv, void* const* sum_ptrs, int64_t rows, int64_t N, int world,
                                     int rank, void* stream) {
  return tp_reduce_slots_bcast(recv, sum_ptrs, rows, N, world, rank, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_tp_reduce_slots(const void* recv, void* sum, int64_t rows, int64_t N, int world, int rank,
                               void* stream) {
  return tp_reduce_slots(recv, sum, rows, N, world, rank, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_tp_barrier(int* const* flag_ptrs, int* own_flags, int world, int rank, int epoch, void* stream) {
  return tp_barrier(flag_ptrs, own_flags, world, rank, epoch, nullptr, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_tp_barrier_next(int* const* flag_ptrs, int* own_flags, int* epoch_counter, int world, int rank,
                               void* stream) {
  if (!epoch_counter) return set_error(B2G_ERR_INVALID, "tp_barrier_next: epoch_counter is NULL");
  return tp_barrier(flag_ptrs, own_flags, world, rank, 0, epoch_counter, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_tp_reduce_shard(const void* const* part_ptrs, void* sum, int64_t ld, int64_t rows, int64_t N,
                               int world, int rank, void* stream) {
  return tp_reduce_shard(part_ptrs, sum, ld, rows, N, world, rank, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_tp_gather_residual(const void* const* sum_ptrs, int64_t ld, int64_t rows, int64_t N, int world,
                                  const b2g_tp_residual_seg* segs, int nsegs, void* stream) {
  return tp_gather_residual(sum_ptrs, ld, rows, N, world, segs, nsegs, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_t5_attention(const float* Q, const float* K, const float* V, const float* rel_bias, int n_head,
                            int d_head, int64_t L, float scale, const float* attn_mask, float* out, void* stream) {
  return t5_attention(Q, K, V, rel_bias, n_head, d_head, L, scale, attn_mask, out, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_quantize_e4m3(const void* src, b2g_dtype src_dtype, int64_t rows, int64_t cols, int64_t ld,
                             uint8_t* dst, int64_t dst_ld, float* scales, void* stream) {
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  return quantize_rows_e4m3(src, src_dtype, rows, cols, ld, dst, dst_ld, scales, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_gemm_fp8(const b2g_gemm_desc* d, const float* a_scale, const float* b_scale, void* stream) {
  if (!d) return set_error(B2G_ERR_INVALID, "b2g_gemm_fp8: null descriptor");
  if (d->M < 0 || d->N < 0 || d->K < 0) return set_error(B2G_ERR_INVALID, "b2g_gemm_fp8: negative size");
  if (d->M == 0 || d->N == 0) return B2G_OK;
  if (d->K == 0) return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_fp8: K must be positive");
  if (!d->a || !d->b || !d->d) return set_error(B2G_ERR_INVALID, "b2g_gemm_fp8: null operand");
  if (d->lda < d->K || d->ldb < d->K || d->ldd < d->N) return set_error(B2G_ERR_INVALID, "b2g_gemm_fp8: lda/ldb/ldd");
  if (d->b_dtype != B2G_E4M3 || !b_scale)
    return set_error(B2G_ERR_INVALID, "b2g_gemm_fp8: weights must be E4M3 with per-row scales");
  if (d->a_dtype == B2G_E4M3 && !a_scale)
    return set_error(B2G_ERR_INVALID, "b2g_gemm_fp8: E4M3 activations need per-row scales");
  if (d->a_dtype != B2G_E4M3 && d->a_dtype != B2G_BF16 && d->a_dtype != B2G_F16 && d->a_dtype != B2G_F32)
    return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_fp8: activations must be E4M3, BF16, F16 or F32");
  if (d->epilogue < B2G_EPI_NONE || d->epilogue > B2G_EPI_GATED_RESIDUAL)
    return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_fp8: unknown epilogue");
  if (d->epilogue == B2G_EPI_GATED_RESIDUAL && (!d->gate || d->d_dtype != B2G_F32))
    return set_error(B2G_ERR_INVALID, "b2g_gemm_fp8: gated residual needs a gate and an F32 output");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  GemmProblem p;
  p.M = d->M; p.N = d->N; p.K = d->K;
  p.a = d->a; p.a_dtype = d->a_dtype; p.lda = d->lda;
  p.b = d->b; p.b_dtype = B2G_E4M3; p.ldb = d->ldb;
  p.bias = d->bias; p.bias_dtype = d->bias_dtype;
  p.d = d->d; p.d_dtype = d->d_dtype; p.ldd = d->ldd;
  p.epilogue = d->epilogue;
  p.gate = d->gate;
  p.a_scale = a_scale;
  p.b_scale = b_scale;
  if (p.a_dtype != B2G_E4M3) {
    // Per-token quantisation of the activations into the workspace: [M, round_up(K, 16)]
    // E4M3 rows (16-byte TMA rows) followed by M fp32 scales.
    const int64_t kp = round_up(p.K, 16);
    const size_t q_bytes = static_cast<size_t>(round_up(p.M * kp, 256));
    void* ws = nullptr;
    if ((s = workspace_get(q_bytes + static_cast<size_t>(p.M) * 4, &ws)) != B2G_OK) return s;
    uint8_t* q = static_cast<uint8_t*>(ws);
    float* qs = reinterpret_cast<float*>(q + q_bytes);
    if ((s = quantize_rows_e4m3(p.a, p.a_dtype, p.M, p.K, p.lda, q, kp, qs, st)) != B2G_OK) return s;
    p.a = q;
    p.a_dtype = B2G_E4M3;
    p.lda = kp;
    p.a_scale = qs;
  }
  std::string why;
  if (!tc_gemm_supported(p, &why)) return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_fp8: " + why);
  return tc_gemm_launch(p, st);
}

b2g_status b2g_gemm_fp8_group(const b2g_gemm_desc* descs, const float* const* a_scales,
                              const float* const* b_scales, int count, void* stream) {
  if (count < 0 || (count > 0 && (!descs || !a_scales || !b_scales)))
    return set_error(B2G_ERR_INVALID, "b2g_gemm_fp8_group: bad descriptor or scale arrays");
  GemmProblem ps[kMaxGemmGroups];
  int n = 0;
  for (int i = 0; i < count; ++i) {
    GemmProblem p;
    bool empty = false;
    b2g_status s = fp8_desc_to_problem(descs + i, a_scales[i], b_scales[i], "b2g_gemm_fp8_group", &p, &empty);
    if (s != B2G_OK) return s;
    std::string why;
    if (!empty && !tc_gemm_supported(p, &why)) return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_fp8_group: " + why);
    if (!empty && n < kMaxGemmGroups) ps[n] = p;
    if (!empty) ++n;
  }
  if (n == 0) return B2G_OK;
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  bool one_launch = n >= 2 && n <= kMaxGemmGroups;
  for (int i = 1; one_launch && i < n; ++i) one_launch = tc_gemm_groupable(ps[0], ps[i]);
  if (one_launch) return tc_gemm_launch_group(ps, n, st);
  for (int i = 0; i < count; ++i) {
    GemmProblem p;
    bool empty = false;
    if ((s = fp8_desc_to_problem(descs + i, a_scales[i], b_scales[i], "b2g_gemm_fp8_group", &p, &empty)) != B2G_OK)
      return s;
    if (!empty && (s = tc_gemm_launch(p, st)) != B2G_OK) return s;
  }
  return B2G_OK;
}

b2g_status b2g_bias_gated_residual(const void* y, b2g_dtype y_dtype, int64_t ldy, const float* bias,
                                   const float* gate, float* residual, int64_t ldr, int64_t M, int64_t N,
                                   void* stream) {
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  return bias_gated_residual(y, y_dtype, ldy, bias, gate, residual, ldr, M, N, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_linear_lt_stream(int64_t M, int64_t K, int64_t N, const void* x_data, cudaDataType_t x_type,
                                const void* w_data, cudaDataType_t w_type, const void* bias_data, void* out_data,
                                void* stream) {
  bool okx = false, okw = false;
  const b2g_dtype xt = from_cuda_type(x_type, &okx), wt = from_cuda_type(w_type, &okw);
  if (!okx || !okw || xt != wt) return set_error(B2G_ERR_UNSUPPORTED, "b2g_linear_lt: x_type and w_type must be equal "
                                                                     "and one of CUDA_R_32F, CUDA_R_16F, CUDA_R_16BF");
  b2g_gemm_desc d{};
  d.M = M; d.N = N; d.K = K;
  d.a = x_data; d.a_dtype = xt; d.lda = K;
  d.b = w_data; d.b_dtype = wt; d.ldb = K;
  d.bias = bias_data; d.bias_dtype = B2G_F32;
  d.d = out_data; d.d_dtype = B2G_F32; d.ldd = N;
  d.epilogue = B2G_EPI_NONE;
  return b2g_gemm(&d, stream);
}

b2g_status b2g_linear_lt(int64_t M, int64_t K, int64_t N, const void* x_data, cudaDataType_t x_type,
                         const void* w_data, cudaDataType_t w_type, const void* bias_data, void* out_data) {
  return b2g_linear_lt_stream(M, K, N, x_data, x_type, w_data, w_type, bias_data, out_data, nullptr);
}

b2g_status b2g_linear_gated_residual(const void* x, cudaDataType_t x_type, const void* w, cudaDataType_t w_type,
                                     const float* bias, float* residual_inout, const float* gate, int64_t M, int64_t K,
                                     int64_t N_out) {
  bool okx = false, okw = false;
  const b2g_dtype xt = from_cuda_type(x_type, &okx), wt = from_cuda_type(w_type, &okw);
  if (!okx || !okw || (wt != B2G_BF16 && wt != B2G_F16) || !(xt == wt || xt == B2G_F32))
    return set_error(B2G_ERR_UNSUPPORTED, "b2g_linear_gated_residual: w must be BF16/F16 and x F32 or w's dtype");
  b2g_gemm_desc d{};
  d.M = M; d.N = N_out; d.K = K;
  d.a = x; d.a_dtype = xt; d.lda = K;
  d.b = w; d.b_dtype = wt; d.ldb = K;
  d.bias = bias; d.bias_dtype = B2G_F32;
  d.d = residual_inout; d.d_dtype = B2G_F32; d.ldd = N_out;
  d.epilogue = B2G_EPI_GATED_RESIDUAL;
  d.gate = gate;
  return b2g_gemm(&d, nullptr);
}

b2g_status b2g_convert_f32(const float* src, int64_t lds, int64_t rows, int64_t cols, void* dst, b2g_dtype dst_dtype,
                           int64_t ldd, void* stream) {
  if (rows <= 0 || cols <= 0) return B2G_OK;
  if (!src || !dst || lds < cols || ldd < cols || (dst_dtype != B2G_BF16 && dst_dtype != B2G_F16))
    return set_error(B2G_ERR_INVALID, "b2g_convert_f32: arguments");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  return cast_f32_to_16(src, dst, dst_dtype, 1, rows, cols, lds, 0, ldd, 0, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_batched_matmul_Bt(const float* A, const float* B, float* C, int64_t batch, int64_t M, int64_t K,
                                 int64_t N) {
  return b2g_batched_matmul_Bt_stream(A, B, C, batch, M, K, N, nullptr);
}

b2g_status b2g_batched_matmul_Bt_stream(const float* A, const float* B, float* C, int64_t batch, int64_t M, int64_t K,
                                        int64_t N, void* stream) {
  if (batch < 0 || M < 0 || K < 0 || N < 0) return set_error(B2G_ERR_INVALID, "b2g_batched_matmul_Bt: negative size");
  if (batch == 0 || M == 0 || N == 0) return B2G_OK;
  if (!A || !B || !C) return set_error(B2G_ERR_INVALID, "b2g_batched_matmul_Bt: null operand");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  // CUBLAS_COMPUTE_32F_FAST_16BF as cuBLAS runs it on B200: operands rounded to TF32 (round
  // to nearest even), TF32 products, fp32 accumulation -> kind::tf32 tensor-core MMAs.  With
  // 16-byte operand rows (K % 4 == 0, aligned bases) the operands go to the kernel as they are
  // and it rounds each shared-memory stage; otherwise a pass rounds them into padded copies.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GemmProblem p;
  p.M = M; p.N = N; p.K = K; p.batch = batch;
  p.d = C; p.d_dtype = B2G_F32; p.ldd = N; p.d_bstride = M * N;
  p.allow_tf32 = true;
  p.a_dtype = p.b_dtype = B2G_F32;
  if (K > 0 && K % 4 == 0 && (reinterpret_cast<uintptr_t>(A) & 15u) == 0 && (reinterpret_cast<uintptr_t>(B) & 15u) == 0) {
    p.a = A; p.lda = K; p.a_bstride = M * K;
    p.b = B; p.ldb = K; p.b_bstride = N * K;
    p.round_tf32 = true;
    return run_gemm(p, st);
  }
  const int64_t kp = round_up(K > 0 ? K : 1, 4);  // 16-byte rows for TMA
  const size_t a_bytes = static_cast<size_t>(round_up(batch * M * kp * 4, 256));
  const size_t b_bytes = static_cast<size_t>(batch * N * kp * 4);
  void* ws = nullptr;
  if ((s = workspace_get(a_bytes + b_bytes, &ws)) != B2G_OK) return s;
  void* wa = ws;
  void* wb = static_cast<char*>(ws) + a_bytes;
  if ((s = cast_f32_to_16(A, wa, B2G_F32, batch, M, K, K, M * K, kp, M * kp, st)) != B2G_OK) return s;
  if ((s = cast_f32_to_16(B, wb, B2G_F32, batch, N, K, K, N * K, kp, N * kp, st)) != B2G_OK) return s;
  p.a = wa; p.lda = kp; p.a_bstride = M * kp;
  p.b = wb; p.ldb = kp; p.b_bstride = N * kp;
  return run_gemm(p, st);
}

b2g_status b2g_attention_with_rope(const float* Q, const float* K, const float* V, const float* pe, int n_head,
                                   int d_head, int64_t L, const float* attn_mask, float* out, void* stream) {
  if (n_head < 0 || d_head < 0 || L < 0) return set_error(B2G_ERR_INVALID, "b2g_attention_with_rope: negative size");
  if (L == 0 || n_head == 0) return B2G_OK;
  if (!Q || !K || !V || !pe || !out) return set_error(B2G_ERR_INVALID, "b2g_attention_with_rope: null operand");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  return attention_rope(Q, K, V, pe, attn_mask, out, L, n_head, d_head, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_attention_qknorm_rope(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                                     int64_t ldv, const float* q_norm, const float* k_norm, const float* q_norm2,
                                     const float* k_norm2, int64_t norm_split, float eps, const float* pe,
                                     const float* attn_mask, void* out, b2g_dtype out_dtype, int64_t ldo, int64_t L,
                                     int n_head, int d_head, void* stream) {
  if (n_head < 0 || d_head < 0 || L < 0) return set_error(B2G_ERR_INVALID, "b2g_attention_qknorm_rope: negative size");
  if (L == 0 || n_head == 0) return B2G_OK;
  if (!q || !k || !v || !pe || !out) return set_error(B2G_ERR_INVALID, "b2g_attention_qknorm_rope: null operand");
  const int64_t hd = static_cast<int64_t>(n_head) * d_head;
  if (ldq < hd || ldk < hd || ldv < hd || ldo < hd)
    return set_error(B2G_ERR_INVALID, "b2g_attention_qknorm_rope: row stride below n_head*d_head");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  AttnArgs a;
  a.q = q; a.ldq = ldq; a.k = k; a.ldk = ldk; a.v = v; a.ldv = ldv;
  a.q_norm = q_norm; a.k_norm = k_norm; a.eps = eps;
  a.q_norm2 = q_norm2; a.k_norm2 = k_norm2; a.norm_split = norm_split;
  a.pe = pe; a.key_bias = attn_mask;
  a.out = out; a.out_dtype = out_dtype; a.ldo = ldo;
  a.L = L; a.H = n_head; a.D = d_head;
  return attention_rope_ex(a, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_gemm_qkv_rope(const b2g_gemm_desc* descs, const b2g_qkv_rope_desc* rope, int count, int n_head,
                             float eps, void* stream) {
  if (!descs || !rope || count < 1 || count > kMaxGemmGroups || n_head < 1)
    return set_error(B2G_ERR_INVALID, "b2g_gemm_qkv_rope: 1 to 4 descriptors with rope descriptors, n_head >= 1");
  GemmProblem ps[kMaxGemmGroups];
  QkvRope rs[kMaxGemmGroups];
  int n = 0;
  for (int i = 0; i < count; ++i) {
    const b2g_gemm_desc* d = descs + i;
    if (d->epilogue != B2G_EPI_NONE) return set_error(B2G_ERR_INVALID, "b2g_gemm_qkv_rope: epilogue must be NONE");
    if (d->d_dtype != B2G_BF16) return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_qkv_rope: bf16 output");
    const int64_t qkv_cols = 3ll * n_head * 128;
    const bool tail = rope[i].gelu_out != nullptr;
    if (tail ? (count != 1 || d->N <= qkv_cols) : d->N != qkv_cols)
      return set_error(B2G_ERR_INVALID, "b2g_gemm_qkv_rope: N must be 3 * n_head * 128 (more, with one problem, for "
                                        "a GELU tail)");
    const bool fp8 = d->a_dtype == B2G_E4M3;
    if (d->a_dtype != d->b_dtype || (d->a_dtype != B2G_BF16 && d->a_dtype != B2G_F16 && !fp8))
      return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_qkv_rope: bf16, fp16 or E4M3 operands of one type");
    if (!rope[i].pe) return set_error(B2G_ERR_INVALID, "b2g_gemm_qkv_rope: pe is required");
    if (rope[i].pe_period < 0 || rope[i].pe_period > (1ll << 30))
      return set_error(B2G_ERR_INVALID, "b2g_gemm_qkv_rope: pe_period must be 0 or a positive row count");
    GemmProblem p;
    bool empty = false;
    b2g_gemm_desc dq = *d;  // d holds the [q | k | v] columns only; the tail goes to gelu_out
    dq.N = qkv_cols;
    b2g_status s = fp8 ? fp8_desc_to_problem(&dq, rope[i].a_scale, rope[i].b_scale, "b2g_gemm_qkv_rope", &p, &empty)
                       : desc_to_problem(&dq, "b2g_gemm_qkv_rope", &p, &empty);
    if (s != B2G_OK) return s;
    if (empty) continue;
    p.N = d->N;
    if (p.K == 0) return set_error(B2G_ERR_INVALID, "b2g_gemm_qkv_rope: K must be positive");
    rs[n].heads = n_head;
    rs[n].eps = eps;
    rs[n].pe = rope[i].pe;
    rs[n].q_norm = rope[i].q_norm;
    rs[n].k_norm = rope[i].k_norm;
    rs[n].gelu_out = rope[i].gelu_out;
    rs[n].gelu_ld = rope[i].gelu_ld;
    rs[n].pe_period = rope[i].pe_period;
    if (rope[i].pe_compact != 0 && rope[i].pe_compact != 1)
      return set_error(B2G_ERR_INVALID, "b2g_gemm_qkv_rope: pe_compact must be 0 or 1");
    rs[n].pe_compact = rope[i].pe_compact == 1;
    p.rope = &rs[n];
    p.epilogue = static_cast<b2g_epilogue>(kEpiQkvRope);
    std::string why;
    if (!tc_gemm_supported(p, &why)) return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_qkv_rope: " + why);
    ps[n++] = p;
  }
  if (n == 0) return B2G_OK;
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  bool one_launch = n >= 2;
  for (int i = 1; one_launch && i < n; ++i) one_launch = tc_gemm_groupable(ps[0], ps[i]);
  if (one_launch) return tc_gemm_launch_group(ps, n, st);
  for (int i = 0; i < n; ++i)
    if ((s = tc_gemm_launch_group(ps + i, 1, st)) != B2G_OK) return s;
  return B2G_OK;
}

b2g_status b2g_attention_bf16(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                              int64_t L, int n_head, int d_head, const float* key_bias, void* out,
                              b2g_dtype out_dtype, int64_t ldo, void* stream) {
  if (n_head < 0 || d_head < 0 || L < 0) return set_error(B2G_ERR_INVALID, "b2g_attention_bf16: negative size");
  if (L == 0 || n_head == 0) return B2G_OK;
  AttnBf16Args a;
  a.q = static_cast<const __nv_bfloat16*>(q); a.ldq = ldq;
  a.k = static_cast<const __nv_bfloat16*>(k); a.ldk = ldk;
  a.v = static_cast<const __nv_bfloat16*>(v); a.ldv = ldv;
  a.key_bias = key_bias;
  a.out = out; a.out_dtype = out_dtype; a.ldo = ldo;
  a.L = L; a.H = n_head; a.D = d_head;
  return attention_bf16(a, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_attention_bf16_batched(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                      int64_t ldv, int64_t L, int64_t batch, int n_head, int d_head,
                                      const float* key_bias, int64_t bias_stride, void* out, b2g_dtype out_dtype,
                                      int64_t ldo, void* stream) {
  if (n_head < 0 || d_head < 0 || L < 0 || batch < 0)
    return set_error(B2G_ERR_INVALID, "b2g_attention_bf16_batched: negative size");
  if (L == 0 || n_head == 0 || batch == 0) return B2G_OK;
  AttnBf16Args a;
  a.q = static_cast<const __nv_bfloat16*>(q); a.ldq = ldq;
  a.k = static_cast<const __nv_bfloat16*>(k); a.ldk = ldk;
  a.v = static_cast<const __nv_bfloat16*>(v); a.ldv = ldv;
  a.key_bias = key_bias; a.bias_stride = bias_stride;
  a.out = out; a.out_dtype = out_dtype; a.ldo = ldo;
  a.L = L; a.H = n_head; a.D = d_head; a.batch = batch;
  return attention_bf16(a, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_modulate_to_bf16(const float* x, const float* shift, const float* scale, void* out, int64_t M,
                                int64_t C, float eps, void* stream) {
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  return modulate_rows(x, shift, scale, out, B2G_BF16, nullptr, M, C, eps, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_modulate_to_e4m3(const float* x, const float* shift, const float* scale, uint8_t* out,
                                float* row_scale, int64_t M, int64_t C, float eps, void* stream) {
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  return modulate_rows(x, shift, scale, out, B2G_E4M3, row_scale, M, C, eps, static_cast<cudaStream_t>(stream));
}

b2g_status b2g_modulate_streams(const float* x, const float* txt_shift, const float* txt_scale,
                                const float* img_shift, const float* img_scale, int64_t seq, int64_t txt_rows,
                                void* out, b2g_dtype out_dtype, float* row_scale, int64_t M, int64_t C, float eps,
                                void* stream) {
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  if (seq <= 0 || txt_rows < 0 || txt_rows > seq || M % seq != 0)
    return set_error(B2G_ERR_INVALID, "b2g_modulate_streams: M must be whole sequences of seq >= txt_rows rows");
  return modulate_rows(x, txt_shift, txt_scale, out, out_dtype, row_scale, M, C, eps,
                       static_cast<cudaStream_t>(stream), img_shift, img_scale, seq, txt_rows);
}

b2g_status b2g_check_device_error(int* code) {
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  if ((s = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize")) != B2G_OK) return s;
  int v = 0;
  if ((s = check_cuda(cudaMemcpy(&v, dev->err_word, sizeof(int), cudaMemcpyDeviceToHost), "read error word")) != B2G_OK)
    return s;
  if (code) *code = v;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpy(dev->err_word, &zero, sizeof(int), cudaMemcpyHostToDevice);
    std::string who;
    const char* names[] = {"TMA producer", "MMA issuer", "epilogue", "tensor-parallel barrier (another rank)"};
    for (int b = 0; b < 4; ++b)
      if (v & (1 << b)) who += (who.empty() ? "" : ", ") + std::string(names[b]);
    return set_error(B2G_ERR_DEVICE_TIMEOUT, "a kernel gave up on a bounded wait (code " + std::to_string(v) +
                                                 ": " + (who.empty() ? "unknown" : who) + ")");
  }
  return B2G_OK;
}

}  // extern "C"
