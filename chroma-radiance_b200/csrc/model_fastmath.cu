// model_fastmath.cu — the approximator's input vector (compute_modulation, chroma.cuh:467-505),
// compiled with --use_fast_math like the reference (its CMakeLists.txt builds kernels.cu so).
//
// The reference's timestep_embedding (kernels.cu:608-631) evaluates cos/sin of t * 1000 * freq
// with the fast hardware approximations; for the mod-index rows the argument reaches 344000
// rad, where one ulp of the argument moves the result by far more than any tolerance.  To give
// the same values, this file states the same expression and is built with the same flags, and
// the period and time factor reach the kernel as run-time arguments (as in the reference) so
// that nothing is folded at compile time.
#include <cuda_runtime.h>
#include "engine.cuh"

namespace b2g {
namespace {

// Sinusoidal embedding: dims [0, dim/2) cos(t * f_d), [dim/2, dim) sin(t * f_d), with
// f_d = exp(-ln(max_period) * d / (dim/2)) and t = input * time_factor.
__device__ __forceinline__ float embed(float input, int d, int dim, float time_factor, float max_period) {
  const int half_dim = dim / 2;
  const float t = input * time_factor;
  if (d < half_dim) {
    const float freq = expf(-logf(max_period) * (float)d / (float)half_dim);
    return cosf(t * freq);
  }
  const int d2 = d - half_dim;
  const float freq = expf(-logf(max_period) * (float)d2 / (float)half_dim);
  return sinf(t * freq);
}

// vec[i] = [embed(timestep, 16 dims) | embed(guidance, 16) | embed(i, 32)] for row i < rows
// (the concatenation compute_modulation builds, [344, 64]).
__global__ void timestep_vec_kernel(const float* timestep, float guidance, float time_factor, float max_period,
                                    float* out, int rows) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * 64) return;
  const int i = idx / 64, c = idx % 64;
  float v;
  if (c < 16) v = embed(timestep[0], c, 16, time_factor, max_period);
  else if (c < 32) v = embed(guidance, c - 16, 16, time_factor, max_period);
  else v = embed(static_cast<float>(i), c - 32, 32, time_factor, max_period);
  out[idx] = v;
}

}  // namespace
}  // namespace b2g

using namespace b2g;

extern "C" b2g_status b2g_timestep_vec(const float* timestep, float guidance, float* out, int rows, void* stream) {
  if (!timestep || !out || rows <= 0 || rows > (1 << 24)) return set_error(B2G_ERR_INVALID, "b2g_timestep_vec");
  DeviceInfo* dev = nullptr;
  b2g_status s = device_info(&dev);
  if (s != B2G_OK) return s;
  timestep_vec_kernel<<<(rows * 64 + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      timestep, guidance, 1000.0f, 10000.0f, out, rows);
  note_launch();
  return check_cuda(cudaGetLastError(), "timestep_vec launch");
}
