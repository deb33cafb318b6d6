// tp_comm.cu — the cross-rank barrier of the fused tensor-parallel layers.
//
// After a row-split layer whose reduction is fused into its GEMM (b2g_gemm_tp_reduce), every
// rank's residual copy is written by other ranks' CTAs; no rank may read its copy, or reuse its
// partial buffer, until all ranks' GEMMs have finished.  This kernel is that barrier: rank r
// stores `epoch` into slot r of every rank's flag array (peer-mapped, system-scope release) and
// then waits until every slot of its own array has reached `epoch` (acquire).  The wait is
// bounded (2 s); on timeout it records kErrWaitTpBarrier in the device error word and returns,
// so a missing rank surfaces through b2g_check_device_error instead of a hung GPU.
#include <cuda_bf16.h>
#include <cstdint>
#include "engine.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

namespace {

__global__ void tp_barrier_kernel(int* const* flag_ptrs, int* own_flags, int world, int rank, int epoch,
                                  int* epoch_ctr, int* err) {
  const int q = threadIdx.x;
  // Device-held epoch (epoch_ctr != nullptr): this barrier's epoch is the previous one + 1,
  // read by every thread before thread 0 stores it back, so a CUDA graph that captured the
  // launch waits on a fresh epoch at every replay.
  if (epoch_ctr) epoch = *epoch_ctr + 1;
  __syncthreads();
  if (epoch_ctr && q == 0) *epoch_ctr = epoch;
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

// ---------------------------------------------------------------------------- two-phase reduction
// The all-reduce of a row-split layer's bf16 partial [rows, N] over NVLink peer memory, with the
// bias + gated residual update folded into its second phase.  Rows are split into `world`
// shards of ceil(rows / world); rank q owns shard q.
//   phase 1 (tp_reduce_shard_kernel): each rank sums, in rank order, the world partials of its
//     own shard (world - 1 of them read from the peers' buffers), rounds to bf16 (as a bf16
//     all-reduce rounds) and stores the shard in its own sum buffer;
//   phase 2 (tp_gather_residual_kernel): each rank reads every row's sums from the owner's sum
//     buffer and applies residual += gate * (sum + bias) to its own replicated residual.
// A cross-rank barrier (tp_barrier) goes before each phase; the kernels themselves never wait.
// A thread covers 8 columns (16 bytes of bf16) of one row; peer loads bypass L1 (__ldcg).
constexpr int kTpMaxWorld = 8;

__device__ __forceinline__ void bf16x8_to_f32(const uint4 u, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__global__ void __launch_bounds__(256) tp_reduce_shard_kernel(const __nv_bfloat16* const* parts, int world,
                                                               __nv_bfloat16* __restrict__ sum, long long ld,
                                                               long long r0, long long r1, int N) {
  const int groups = N / 8;
  const long long total = (r1 - r0) * groups;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long m = r0 + i / groups;
    const int n = static_cast<int>(i % groups) * 8;
    const long long off = m * ld + n;
    uint4 u[kTpMaxWorld];
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q)
      if (q < world) u[q] = __ldcg(reinterpret_cast<const uint4*>(parts[q] + off));
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q) {
      if (q >= world) break;
      float v[8];
      bf16x8_to_f32(u[q], v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
    uint4 o;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    *reinterpret_cast<uint4*>(sum + off) = o;
  }
}

// Phase 1 of the reduce-scatter form: the row-split GEMMs have stored every rank's partial of
// this rank's rows into this rank's receive buffer [world slots][shard rows][N]; sum the slots in
// rank order (local reads only) into this rank's rows of `sum`.
__global__ void __launch_bounds__(256) tp_reduce_slots_kernel(const __nv_bfloat16* __restrict__ recv, int world,
                                                               long long shard, __nv_bfloat16* __restrict__ sum,
                                                               long long ld, long long r0, long long nrows, int N) {
  const int groups = N / 8;
  const long long total = nrows * groups;
  const long long slot = shard * ld;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / groups;
    const int n = static_cast<int>(i % groups) * 8;
    uint4 u[kTpMaxWorld];
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q)
      if (q < world) u[q] = __ldcg(reinterpret_cast<const uint4*>(recv + q * slot + r * ld + n));
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q) {
      if (q >= world) break;
      float v[8];
      bf16x8_to_f32(u[q], v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
    uint4 o;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    *reinterpret_cast<uint4*>(sum + (r0 + r) * ld + n) = o;
  }
}

// The store form: every NVLink transfer is an SM store (16 bytes a thread, consecutive threads on
// consecutive bytes of a row), none a load and none a copy-engine copy.
//   tp_scatter_rows_kernel: row m of this rank's bf16 partial goes to its owner q = m / shard,
//     slot `rank`, row m - q * shard of q's receive buffer [world][shard][N].
//   tp_reduce_slots_bcast_kernel: this rank sums its receive slots in rank order (local reads,
//     bf16 rounding as a bf16 all-reduce rounds) and stores each sum row into every rank's sum
//     buffer (its own included) at the same row.
__global__ void __launch_bounds__(256) tp_scatter_rows_kernel(const __nv_bfloat16* __restrict__ part,
                                                               __nv_bfloat16* const* recv, int rank,
                                                               long long rows, long long shard, int N) {
  const int groups = N / 8;
  const long long total = rows * groups;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long m = i / groups;
    const int n = static_cast<int>(i % groups) * 8;
    const long long q = m / shard;
    const uint4 u = __ldcs(reinterpret_cast<const uint4*>(part + m * N + n));
    *reinterpret_cast<uint4*>(recv[q] + (rank * shard + (m - q * shard)) * N + n) = u;
  }
}

__global__ void __launch_bounds__(256) tp_reduce_slots_bcast_kernel(const __nv_bfloat16* __restrict__ recv,
                                                                     __nv_bfloat16* const* sums, int world,
                                                                     long long shard, long long r0,
                                                                     long long nrows, int N) {
  const int groups = N / 8;
  const long long total = nrows * groups;
  const long long slot = shard * N;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / groups;
    const int n = static_cast<int>(i % groups) * 8;
    uint4 u[kTpMaxWorld];
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q)
      if (q < world) u[q] = __ldcs(reinterpret_cast<const uint4*>(recv + q * slot + r * N + n));
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q) {
      if (q >= world) break;
      float v[8];
      bf16x8_to_f32(u[q], v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
    uint4 o;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    const long long off = (r0 + r) * N + n;
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q)
      if (q < world) *reinterpret_cast<uint4*>(sums[q] + off) = o;
  }
}

struct TpSegs {
  int count;
  long long row0[2], rows[2], ldr[2];
  const float* bias[2];
  const float* gate[2];
  float* res[2];
};

__global__ void __launch_bounds__(256) tp_gather_residual_kernel(const __nv_bfloat16* const* sums, long long ld,
                                                                  long long shard, int N, TpSegs sg) {
  const int groups = N / 8;
  for (int k = 0; k < sg.count; ++k) {
    const long long total = sg.rows[k] * groups;
    const float* bias = sg.bias[k];
    const float* gate = sg.gate[k];
    float* res = sg.res[k];
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
      const long long r = i / groups;
      const int n = static_cast<int>(i % groups) * 8;
      const long long m = sg.row0[k] + r;  // row of the partial / sum buffers
      const uint4 u = __ldcg(reinterpret_cast<const uint4*>(sums[m / shard] + m * ld + n));
      float4* rp = reinterpret_cast<float4*>(res + r * sg.ldr[k] + n);
      float4 a = rp[0], c = rp[1];
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(gate + n)), g1 = __ldg(reinterpret_cast<const float4*>(gate + n) + 1);
      float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
      if (bias) {
        b0 = __ldg(reinterpret_cast<const float4*>(bias + n));
        b1 = __ldg(reinterpret_cast<const float4*>(bias + n) + 1);
      }
      float v[8];
      bf16x8_to_f32(u, v);
      a.x += g0.x * (v[0] + b0.x); a.y += g0.y * (v[1] + b0.y); a.z += g0.z * (v[2] + b0.z); a.w += g0.w * (v[3] + b0.w);
      c.x += g1.x * (v[4] + b1.x); c.y += g1.y * (v[5] + b1.y); c.z += g1.z * (v[6] + b1.z); c.w += g1.w * (v[7] + b1.w);
      rp[0] = a;
      rp[1] = c;
    }
  }
}

}  // namespace

b2g_status tp_reduce_shard(const void* const* part_ptrs, void* sum, int64_t ld, int64_t rows, int64_t N, int world,
                           int rank, cudaStream_t st) {
  if (world < 1 || world > kTpMaxWorld || rank < 0 || rank >= world || !part_ptrs || !sum || rows < 0 || N <= 0 ||
      N % 8 || ld < N || ld % 8 || (reinterpret_cast<uintptr_t>(sum) & 15u))
    return set_error(B2G_ERR_INVALID, "tp_reduce_shard: world in [1, 8], N % 8 == 0, 16-byte rows");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const int64_t shard = (rows + world - 1) / world;
  const int64_t r0 = rank * shard < rows ? rank * shard : rows;
  const int64_t r1 = r0 + shard < rows ? r0 + shard : rows;
  if (r1 <= r0) return B2G_OK;
  const int64_t work = (r1 - r0) * (N / 8);
  const int64_t blocks = (work + 255) / 256 < 8 * dev->num_sms ? (work + 255) / 256 : 8 * dev->num_sms;
  tp_reduce_shard_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16* const*>(part_ptrs), world, static_cast<__nv_bfloat16*>(sum), ld, r0, r1,
      static_cast<int>(N));
  note_launch();
  return check_cuda(cudaGetLastError(), "tp_reduce_shard launch");
}

b2g_status tp_reduce_slots(const void* recv, void* sum, int64_t rows, int64_t N, int world, int rank,
                           cudaStream_t st) {
  if (world < 1 || world > kTpMaxWorld || rank < 0 || rank >= world || !recv || !sum || rows < 0 || N <= 0 || N % 8 ||
      (reinterpret_cast<uintptr_t>(recv) & 15u) || (reinterpret_cast<uintptr_t>(sum) & 15u))
    return set_error(B2G_ERR_INVALID, "tp_reduce_slots: world in [1, 8], N % 8 == 0, 16-byte aligned buffers");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const int64_t shard = (rows + world - 1) / world;
  const int64_t r0 = rank * shard < rows ? rank * shard : rows;
  const int64_t r1 = r0 + shard < rows ? r0 + shard : rows;
  if (r1 <= r0) return B2G_OK;
  const int64_t work = (r1 - r0) * (N / 8);
  const int64_t blocks = (work + 255) / 256 < 8 * dev->num_sms ? (work + 255) / 256 : 8 * dev->num_sms;
  tp_reduce_slots_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(recv), world, shard, static_cast<__nv_bfloat16*>(sum), N, r0, r1 - r0,
      static_cast<int>(N));
  note_launch();
  return check_cuda(cudaGetLastError(), "tp_reduce_slots launch");
}

b2g_status tp_scatter_rows(const void* part, void* const* recv_ptrs, int64_t rows, int64_t N, int world, int rank,
                           cudaStream_t st) {
  if (world < 1 || world > kTpMaxWorld || rank < 0 || rank >= world || !part || !recv_ptrs || rows <= 0 || N <= 0 ||
      N % 8 || (reinterpret_cast<uintptr_t>(part) & 15u))
    return set_error(B2G_ERR_INVALID, "tp_scatter_rows: world in [1, 8], N % 8 == 0, 16-byte aligned partial");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const int64_t shard = (rows + world - 1) / world;
  const int64_t work = rows * (N / 8);
  const int64_t blocks = (work + 255) / 256 < 8 * dev->num_sms ? (work + 255) / 256 : 8 * dev->num_sms;
  tp_scatter_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(part), reinterpret_cast<__nv_bfloat16* const*>(recv_ptrs), rank, rows, shard,
      static_cast<int>(N));
  note_launch();
  return check_cuda(cudaGetLastError(), "tp_scatter_rows launch");
}

b2g_status tp_reduce_slots_bcast(const void* recv, void* const* sum_ptrs, int64_t rows, int64_t N, int world,
                                 int rank, cudaStream_t st) {
  if (world < 1 || world > kTpMaxWorld || rank < 0 || rank >= world || !recv || !sum_ptrs || rows <= 0 || N <= 0 ||
      N % 8 || (reinterpret_cast<uintptr_t>(recv) & 15u))
    return set_error(B2G_ERR_INVALID, "tp_reduce_slots_bcast: world in [1, 8], N % 8 == 0, 16-byte aligned buffers");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const int64_t shard = (rows + world - 1) / world;
  const int64_t r0 = rank * shard < rows ? rank * shard : rows;
  const int64_t r1 = r0 + shard < rows ? r0 + shard : rows;
  if (r1 <= r0) return B2G_OK;
  const int64_t work = (r1 - r0) * (N / 8);
  const int64_t blocks = (work + 255) / 256 < 8 * dev->num_sms ? (work + 255) / 256 : 8 * dev->num_sms;
  tp_reduce_slots_bcast_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(recv), reinterpret_cast<__nv_bfloat16* const*>(sum_ptrs), world, shard, r0,
      r1 - r0, static_cast<int>(N));
  note_launch();
  return check_cuda(cudaGetLastError(), "tp_reduce_slots_bcast launch");
}

// Push form with the copy engines: each transfer is one cudaMemcpyAsync of whole rows between
// this device and a peer's mapped buffer (peer addresses given in host arrays), so the moves run
// on the DMA engines, not the SMs.  Stream-ordered: the barrier kernel that follows starts after
// they have completed.
b2g_status tp_push_rows(const void* part, void* const* recv_ptrs, int64_t rows, int64_t N, int world, int rank,
                        cudaStream_t st) {
  if (world < 1 || world > kTpMaxWorld || rank < 0 || rank >= world || !part || !recv_ptrs || rows <= 0 || N <= 0)
    return set_error(B2G_ERR_INVALID, "tp_push_rows: world in [1, 8], rows and N positive");
  const int64_t shard = (rows + world - 1) / world;
  for (int k = 0; k < world; ++k) {
    const int q = (rank + k) % world;  // each rank starts on a different peer
    const int64_t r0 = q * shard < rows ? q * shard : rows;
    const int64_t r1 = r0 + shard < rows ? r0 + shard : rows;
    if (r1 <= r0) continue;
    char* dst = static_cast<char*>(recv_ptrs[q]) + rank * shard * N * 2;
    const char* src = static_cast<const char*>(part) + r0 * N * 2;
    b2g_status s = check_cuda(cudaMemcpyAsync(dst, src, static_cast<size_t>((r1 - r0) * N * 2),
                                              cudaMemcpyDeviceToDevice, st), "tp_push_rows copy");
    if (s != B2G_OK) return s;
  }
  return B2G_OK;
}

b2g_status tp_push_sums(void* const* sum_ptrs, int64_t rows, int64_t N, int world, int rank, cudaStream_t st) {
  if (world < 1 || world > kTpMaxWorld || rank < 0 || rank >= world || !sum_ptrs || rows <= 0 || N <= 0)
    return set_error(B2G_ERR_INVALID, "tp_push_sums: world in [1, 8], rows and N positive");
  const int64_t shard = (rows + world - 1) / world;
  const int64_t r0 = rank * shard < rows ? rank * shard : rows;
  const int64_t r1 = r0 + shard < rows ? r0 + shard : rows;
  if (r1 <= r0) return B2G_OK;
  const char* src = static_cast<const char*>(sum_ptrs[rank]) + r0 * N * 2;
  for (int k = 1; k < world; ++k) {
    const int q = (rank + k) % world;
    b2g_status s = check_cuda(cudaMemcpyAsync(static_cast<char*>(sum_ptrs[q]) + r0 * N * 2, src,
                                              static_cast<size_t>((r1 - r0) * N * 2), cudaMemcpyDeviceToDevice, st),
                              "tp_push_sums copy");
    if (s != B2G_OK) return s;
  }
  return B2G_OK;
}

b2g_status tp_gather_residual(const void* const* sum_ptrs, int64_t ld, int64_t rows, int64_t N, int world,
                              const b2g_tp_residual_seg* segs, int nsegs, cudaStream_t st) {
  if (world < 1 || world > kTpMaxWorld || !sum_ptrs || !segs || nsegs < 1 || nsegs > 2 || rows <= 0 || N <= 0 ||
      N % 8 || ld < N || ld % 8)
    return set_error(B2G_ERR_INVALID, "tp_gather_residual: world in [1, 8], 1 or 2 segments, N % 8 == 0");
  TpSegs sg{};
  sg.count = nsegs;
  int64_t work = 0;
  for (int k = 0; k < nsegs; ++k) {
    const b2g_tp_residual_seg& g = segs[k];
    if (g.row0 < 0 || g.rows < 0 || g.row0 + g.rows > rows || !g.gate || !g.residual || g.ldr < N || g.ldr % 4 ||
        (reinterpret_cast<uintptr_t>(g.residual) & 15u) || (reinterpret_cast<uintptr_t>(g.gate) & 15u) ||
        (g.bias && (reinterpret_cast<uintptr_t>(g.bias) & 15u)))
      return set_error(B2G_ERR_INVALID, "tp_gather_residual: segment rows, 16-byte aligned gate/bias/residual rows");
    sg.row0[k] = g.row0;
    sg.rows[k] = g.rows;
    sg.ldr[k] = g.ldr;
    sg.bias[k] = g.bias;
    sg.gate[k] = g.gate;
    sg.res[k] = g.residual;
    work += g.rows * (N / 8);
  }
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  const int64_t shard = (rows + world - 1) / world;
  const int64_t blocks = (work + 255) / 256 < 8 * dev->num_sms ? (work + 255) / 256 : 8 * dev->num_sms;
  tp_gather_residual_kernel<<<static_cast<unsigned>(blocks > 0 ? blocks : 1), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16* const*>(sum_ptrs), ld, shard, static_cast<int>(N), sg);
  note_launch();
  return check_cuda(cudaGetLastError(), "tp_gather_residual launch");
}

b2g_status tp_barrier(int* const* flag_ptrs, int* own_flags, int world, int rank, int epoch, int* epoch_ctr,
                      cudaStream_t st) {
  if (world < 1 || world > 1024 || rank < 0 || rank >= world || !flag_ptrs || !own_flags)
    return set_error(B2G_ERR_INVALID, "tp_barrier: world/rank/pointers");
  if (!epoch_ctr && epoch < 1) return set_error(B2G_ERR_INVALID, "tp_barrier: epoch must be >= 1");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  tp_barrier_kernel<<<1, 32 * ((world + 31) / 32), 0, st>>>(flag_ptrs, own_flags, world, rank, epoch, epoch_ctr,
                                                                    dev->err_word);
  note_launch();
  return check_cuda(cudaGetLastError(), "tp_barrier launch");
}

}  // namespace b2g
