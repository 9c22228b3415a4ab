// Per-row temperature arithmetic shared by the spec samplers (the streaming
// kernels and the short-row kernel): the exact logit scale l = (x - m) / T and
// its exponential, as the CPU restatement computes them.
#pragma once

#include "common.cuh"
#include "spec_kernel.cuh"

namespace rl {

constexpr double kLog2e = 1.4426950408889634074;

struct RowT {
  float T, rT;         // temperature, RN(1/T)
  int fast_div;        // Markstein division valid for T
  float c;             // log2(e)/T (bulk sums)
  float cb_hi, cb_lo;  // kRbin / T split in two floats
  float dlt;           // log2(e) / kRbin
};

__device__ __forceinline__ RowT make_rowt(float T) {
  RowT r;
  r.T = T;
  r.rT = __frcp_rn(T);
  r.fast_div = fixed_div_ok(T);
  r.c = static_cast<float>(kLog2e / static_cast<double>(T));
  const double cb = static_cast<double>(kRbin) / static_cast<double>(T);
  r.cb_hi = static_cast<float>(cb);
  r.cb_lo = static_cast<float>(cb - static_cast<double>(r.cb_hi));
  r.dlt = static_cast<float>(kLog2e / static_cast<double>(kRbin));
  return r;
}
// l = (x - m) / T with IEEE rounding, as the CPU restatement computes it.
__device__ __forceinline__ float exact_l(float x, float m, const RowT& r) {
  return div_by(sub_rn(x, m), r.T, r.rT, r.fast_div != 0);
}
__device__ __forceinline__ float exact_e(float x, float m, const RowT& r) { return expf(exact_l(x, m, r)); }

}  // namespace rl
