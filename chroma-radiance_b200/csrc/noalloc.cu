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
// current; make that first call before capturing any stream on the device.  b2g_shutdown
// forgets the resolved addresses, so after a device reset (a new primary context) call
// b2g_shutdown before the next call.
#include <cuda_runtime.h>
#include <atomic>
#include <string>
#include "engine.cuh"

namespace b2g {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
// Device address of each device's copy of the array, resolved on first use.  Two host threads
// resolving the same device at once store the same value, so plain atomics suffice.
std::atomic<void*> g_scratch_addr[kMaxDevices];

// Device address of this device's copy of g_noalloc_scratch, resolved once per device.
b2g_status scratch_address(void** out) {
  int dev = -1;
  b2g_status s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (s != B2G_OK) return s;
  if (dev < 0 || dev >= kMaxDevices) return set_error(B2G_ERR_NO_DEVICE, "device ordinal out of range");
  void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (!p) {
    if ((s = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)")) !=
        B2G_OK)
      return s;
    g_scratch_addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return B2G_OK;
}

int64_t round_up8(int64_t v) { return (v + 7) / 8 * 8; }

}  // namespace

void noalloc_forget() {
  for (auto& a : g_scratch_addr) a.store(nullptr, std::memory_order_release);
}

}  // namespace b2g

using namespace b2g;

extern "C" b2g_status b2g_gemm_noalloc(const b2g_gemm_desc* d, void* stream) {
  GemmProblem p;
  bool empty = false;
  // The same checks as b2g_gemm, so the two entry points accept exactly the same descriptors.
  b2g_status s = desc_to_problem(d, "b2g_gemm_noalloc", &p, &empty);
  if (s != B2G_OK || empty) return s;
  DeviceInfo* dev = nullptr;
  if ((s = device_info(&dev)) != B2G_OK) return s;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  p.allow_split = false;
  const bool w16 = p.b_dtype == B2G_BF16 || p.b_dtype == B2G_F16;
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
