// Self-check of the sampler's fixed-divisor division on the running device.
//
// The spec sampler divides every logit by its row's temperature with
// div_fixed (common.cuh), Markstein's refinement of a * RN(1/T), which is
// correctly rounded only within stated operand ranges. Bit-exact top-k sets
// rest on it, so this entry point lets a caller (and the GPU tests) check it
// against IEEE division, __fdiv_rn, bit for bit on the device that runs the
// sampler.
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

namespace {

constexpr int kSelfThreads = 256;

// mismatch[j] counts the a[i] for which div_by(a[i], T[j]) differs in any bit
// from __fdiv_rn(a[i], T[j]); fast[j] is 1 when the fixed-divisor path is in
// use for T[j]. Grid: x over a (grid-stride), y over T.
__global__ void __launch_bounds__(kSelfThreads) selfcheck_div_kernel(const float* a, int n, const float* T, int nT,
                                                                    uint32_t* mismatch, uint32_t* fast) {
  const int j = blockIdx.y;
  if (j >= nT) return;
  const float b = T[j];
  const float yb = __frcp_rn(b);
  const bool f = rl::fixed_div_ok(b);
  uint32_t bad = 0u;
  for (int i = blockIdx.x * kSelfThreads + threadIdx.x; i < n; i += gridDim.x * kSelfThreads) {
    const float x = a[i];
    const float q = rl::div_by(x, b, yb, f);
    const float r = __fdiv_rn(x, b);
    bad += (__float_as_uint(q) != __float_as_uint(r)) ? 1u : 0u;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) bad += __shfl_xor_sync(0xffffffffu, bad, o);
  if ((threadIdx.x & 31) == 0 && bad) atomicAdd(&mismatch[j], bad);
  if (blockIdx.x == 0 && threadIdx.x == 0) fast[j] = f ? 1u : 0u;
}

}  // namespace

extern "C" {
#pragma GCC visibility push(default)

rl_status rl_selfcheck_div(const float* a, int n, const float* T, int nT, uint32_t* mismatch, uint32_t* fast,
                           void* stream) {
  rl::clear_error();
  if (n < 0 || nT < 0) return rl::set_error(RL_ERR_INVALID_ARG, "rl_selfcheck_div: negative size");
  if (n == 0 || nT == 0) return RL_OK;
  if (!a || !T || !mismatch || !fast) return rl::set_error(RL_ERR_INVALID_ARG, "rl_selfcheck_div: NULL pointer");
  if (nT > 65535) return rl::set_error(RL_ERR_SHAPE, "rl_selfcheck_div: nT > 65535");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(mismatch, 0, sizeof(uint32_t) * static_cast<size_t>(nT), s);
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, "rl_selfcheck_div: cudaMemsetAsync failed");
  const int gx = (n + kSelfThreads - 1) / kSelfThreads < 64 ? (n + kSelfThreads - 1) / kSelfThreads : 64;
  selfcheck_div_kernel<<<dim3(gx, nT), kSelfThreads, 0, s>>>(a, n, T, nT, mismatch, fast);
  e = cudaGetLastError();
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, "rl_selfcheck_div: kernel launch failed");
  return RL_OK;
}

#pragma GCC visibility pop
}  // extern "C"
