// Device helpers shared by the sampler kernels (sm_100a).
#pragma once

#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "rl_sampler.h"

namespace rl {

namespace cg = cooperative_groups;

#define RL_NEG_INF (-__builtin_huge_valf())
#define RL_POS_INF (__builtin_huge_valf())

// ---------------------------------------------------------------------------
// Exact f32 arithmetic (never contracted into FMA): the penalties and the
// temperature division must round exactly like the CPU restatement.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }

// Correctly rounded a / b for a divisor b fixed per row, by Markstein's
// FMA-based refinement (P. Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990):
// y = RN(1/b), q = RN(a*y), r = a - b*q (exact with one FMA), RN(q + r*y).
// The caller keeps the operands where that holds and the quotient is a
// finite normal number: 2^-90 <= |a| < 2^100 and 2^-20 <= b <= 2^20 (an
// overflowing quotient would come out NaN, a zero numerator without its
// sign); elsewhere it uses IEEE division. Checked bit for bit against
// __fdiv_rn on the device by rl_selfcheck_div (the library's self-check
// entry point, run by the GPU tests).
__device__ __forceinline__ float div_fixed(float a, float b, float y) {
  float q = __fmul_rn(a, y);
  float r = __fmaf_rn(-q, b, a);
  return __fmaf_rn(r, y, q);
}
// The divisor range in which div_fixed is used (2^-20 <= b <= 2^20).
__device__ __forceinline__ bool fixed_div_ok(float b) { return b >= 9.5367431640625e-07f && b <= 1048576.0f; }
// a / b correctly rounded, by div_fixed where its preconditions hold
// (fast: fixed_div_ok(b); yb = RN(1/b)), else by IEEE division.
__device__ __forceinline__ float div_by(float a, float b, float yb, bool fast) {
  const float m = fabsf(a);
  if (fast && m >= 8.077935669e-28f && m < 1.2676506002282294e30f) return div_fixed(a, b, yb);
  return __fdiv_rn(a, b);
}

// Order-preserving map float -> uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t ord_key(float x) {
  uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord_key_inv(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}
// 64-bit sort key: larger key = earlier in (value desc, id asc) order.
// -0.0 and +0.0 compare equal (IEEE, and the reference's partial_cmp), so
// the value part is taken from x + 0 (which turns -0.0 into +0.0): equal
// values then order by id alone.
__device__ __forceinline__ uint64_t cand_key(float x, uint32_t id) {
  return (static_cast<uint64_t>(ord_key(__fadd_rn(x, 0.0f))) << 32) | static_cast<uint64_t>(0xffffffffu - id);
}
__device__ __forceinline__ float key_val(uint64_t k) { return ord_key_inv(static_cast<uint32_t>(k >> 32)); }
__device__ __forceinline__ uint32_t key_id(uint64_t k) {
  return 0xffffffffu - static_cast<uint32_t>(k & 0xffffffffu);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h16) { return __uint_as_float(h16 << 16); }

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA, non-tensor form): each copy lands in the issuing CTA only.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// Bounded wait on phase `parity`. Returns false when the budget expires.
// Each try suspends the thread until the phase completes or a 20 us hint
// runs out, so a waiting warp takes no issue slots from the working ones.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, long long budget_cycles) {
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > budget_cycles) return false;
  }
}
// global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned), completing on `bar` by transaction count.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// Warp / block reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Device-side wait budget: ~2 s at 2 GHz. A wait that runs out records
// RL_ERR_TIMEOUT for its row and returns; it never traps.
constexpr long long kWaitBudget = 4000000000LL;

}  // namespace rl
