// tp_comm.cu — the cross-rank barrier of the fused tensor-parallel layers.
//
// After a row-split layer whose reduction is fused into its GEMM (b2g_gemm_tp_reduce), every
// rank's residual copy is written by other ranks' CTAs; no rank may read its copy, or reuse its
// partial buffer, until all ranks' GEMMs have finished.  This kernel is that barrier: rank r
// stores `epoch` into slot r of every rank's flag array (peer-mapped, system-scope release) and
// then waits until every slot of its own array has reached `epoch` (acquire).  The wait is
// bounded (2 s); on timeout it records kErrWaitTpBarrier in the device error word and returns,
// so a missing rank surfaces through b2g_check_device_error instead of a hung GPU.
#include <cstdint>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

namespace {

__global__ void tp_barrier_kernel(int* const* flag_ptrs, int* own_flags, int world, int rank, int epoch, int* err) {
  const int q = threadIdx.x;
  if (q >= world) return;
  __threadfence_system();
  int* slot = flag_ptrs[q] + rank;
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(slot), "r"(epoch) : "memory");
  const int* mine = own_flags + q;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if (static_cast<int>(static_cast<unsigned>(v) - static_cast<unsigned>(epoch)) >= 0) break;
    if ((it & 255u) == 255u && global_timer_ns() - t0 > kWaitLimitNs) {
      atomicOr(err, kErrWaitTpBarrier);
      return;
    }
  }
}

}  // namespace

b2g_status tp_barrier(int* const* flag_ptrs, int* own_flags, int world, int rank, int epoch, cudaStream_t st) {
  if (world < 1 || world > 1024 || rank < 0 || rank >= world || !flag_ptrs || !own_flags)
    return set_error(B2G_ERR_INVALID, "tp_barrier: world/rank/pointers");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  tp_barrier_kernel<<<1, 32 * ((world + 31) / 32), 0, st>>>(flag_ptrs, own_flags, world, rank, epoch, dev->err_word);
  note_launch();
  return check_cuda(cudaGetLastError(), "tp_barrier launch");
}

}  // namespace b2g
