// noalloc.cu — b2g_gemm_noalloc: b2g_gemm for callers that must not see the library allocate.
//
// b2g_gemm needs device scratch in one case: F32 activations with 16-bit weights are first
// cast to the weight dtype (as the reference's linear() does before cuBLASLt), and the cast
// lands in a workspace that grows with cudaMalloc (and a device-wide sync + cudaFree when it
// grows).  This variant casts into a fixed array compiled into the library instead, and keeps
// the tensor-core GEMM from splitting K (split-K partials are the GEMM's only other scratch).
//
// Limits: batch*M*round_up(K,8)*2 bytes of cast activations must fit kNoAllocScratchBytes
// (8 MiB, e.g. 1024 x 4096 or 512 x 8192 activations); larger requests return
// B2G_ERR_INVALID with the size in b2g_last_error().  16-bit activations need no scratch.
// The array is shared by every call on a device: calls whose kernels may overlap (other
// streams, other host threads) race on it and must be serialised by the caller.  The first
// call on each device resolves the array's address (cudaGetSymbolAddress) with that device
// current; make that first call before capturing any stream on the device.
#include <cuda_runtime.h>
#include <string>
#include "engine.cuh"

namespace b2g {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of this device's copy of g_noalloc_scratch, resolved once per device.
b2g_status scratch_address(void** out) {
  int dev = -1;
  b2g_status s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (s != B2G_OK) return s;
  if (dev < 0 || dev >= kMaxDevices) return set_error(B2G_ERR_NO_DEVICE, "device ordinal out of range");
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if ((s = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)")) !=
        B2G_OK)
      return s;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return B2G_OK;
}

int64_t round_up8(int64_t v) { return (v + 7) / 8 * 8; }

}  // namespace
}  // namespace b2g

using namespace b2g;

extern "C" b2g_status b2g_gemm_noalloc(const b2g_gemm_desc* d, void* stream) {
  if (!d) return set_error(B2G_ERR_INVALID, "b2g_gemm_noalloc: null descriptor");
  if (d->M < 0 || d->N < 0 || d->K < 0) return set_error(B2G_ERR_INVALID, "b2g_gemm_noalloc: negative size");
  if (d->M == 0 || d->N == 0) return B2G_OK;
  if (!d->d || (d->K > 0 && (!d->a || !d->b))) return set_error(B2G_ERR_INVALID, "b2g_gemm_noalloc: null operand");
  if (d->K > 0 && (d->lda < d->K || d->ldb < d->K))
    return set_error(B2G_ERR_INVALID, "b2g_gemm_noalloc: lda/ldb < K");
  if (d->ldd < d->N) return set_error(B2G_ERR_INVALID, "b2g_gemm_noalloc: ldd < N");
  if (d->epilogue < B2G_EPI_NONE || d->epilogue > B2G_EPI_GATED_RESIDUAL)
    return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_noalloc: unknown epilogue");
  if (d->epilogue == B2G_EPI_GATED_RESIDUAL && (!d->gate || d->d_dtype != B2G_F32))
    return set_error(B2G_ERR_INVALID, "b2g_gemm_noalloc: gated residual needs a gate and an F32 output");
  if (d->a_dtype == B2G_E4M3 || d->b_dtype == B2G_E4M3 || d->d_dtype == B2G_E4M3)
    return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_noalloc: E4M3 operands are not implemented");
  const bool w16 = d->b_dtype == B2G_BF16 || d->b_dtype == B2G_F16;
  if (!(d->a_dtype == d->b_dtype || (d->a_dtype == B2G_F32 && w16)))
    return set_error(B2G_ERR_UNSUPPORTED, "b2g_gemm_noalloc: unsupported operand dtype combination");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);

  GemmProblem p;
  p.M = d->M; p.N = d->N; p.K = d->K;
  p.a = d->a; p.a_dtype = d->a_dtype; p.lda = d->lda;
  p.b = d->b; p.b_dtype = d->b_dtype; p.ldb = d->ldb;
  p.bias = d->bias; p.bias_dtype = d->bias_dtype;
  p.d = d->d; p.d_dtype = d->d_dtype; p.ldd = d->ldd;
  p.epilogue = d->epilogue;
  p.gate = d->gate;
  p.allow_split = false;
  if (p.a_dtype == B2G_F32 && w16 && p.K > 0) {
    const int64_t kp = round_up8(p.K);  // 16-byte rows for TMA
    const double need = static_cast<double>(p.M) * static_cast<double>(kp) * 2.0;
    if (need > static_cast<double>(kNoAllocScratchBytes))
      return set_error(B2G_ERR_INVALID, "b2g_gemm_noalloc: F32 activations need M*round_up(K,8)*2 = " +
                                            std::to_string(static_cast<long long>(need)) +
                                            " bytes of cast scratch; the static scratch holds " +
                                            std::to_string(kNoAllocScratchBytes) + " bytes");
    void* scratch = nullptr;
    if ((s = scratch_address(&scratch)) != B2G_OK) return s;
    // Every element the GEMM reads (rows < M, columns < K) is written by the cast; the tensor
    // map's K extent stops reads at column K, so no part of the scratch needs clearing.
    s = cast_f32_to_16(static_cast<const float*>(p.a), scratch, p.b_dtype, 1, p.M, p.K, p.lda, 0, kp, p.M * kp, st);
    if (s != B2G_OK) return s;
    p.a = scratch;
    p.a_dtype = p.b_dtype;
    p.lda = kp;
    p.a_bstride = p.M * kp;
  }
  if (p.K > 0 && tc_gemm_supported(p, nullptr)) return tc_gemm_launch(p, st);
  return simt_gemm_launch(p, st);
}
