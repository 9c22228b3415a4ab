// LM head feeding the sampler: logits[b, v] = sum_h hidden[b, h] * W[v, h]
// (src/model.rs:236-262, Model::forward's last step, and its matmul_vec),
// on the tensor cores, with the greedy argmax fused into the epilogue.
//
//   rl_lmhead_logits   the logits only (f32 or bf16 out)
//   rl_lmhead_greedy   Decoder::greedy_sample (src/decoder.rs:160-167) of the
//                      logits, LAST maximum on ties; the logits need not be
//                      written at all
//   rl_lmhead_sample   logits into the handle's staging buffer, then the
//                      batched sampler (rl_sample_batch) on them
//
// Operands are bf16 (the reference dequantizes its weights to f32; here the
// weight stays bf16 in HBM, 2 bytes per element), accumulation is f32. One
// persistent CTA per SM walks vocabulary tiles of 128 rows:
//   warp 0      TMA producer: W tile [128 x 64] and hidden tile [N x 64] per
//               stage, both K-major with the 128-byte swizzle
//   warp 1      TMEM allocation and the MMA issuer: tcgen05.mma kind::f16,
//               M = 128 (vocabulary rows), N = batch padded to 16, K = 16 per
//               instruction, accumulators double-buffered in TMEM so the
//               epilogue of tile i overlaps the MMAs of tile i + 1
//   warps 2-5   epilogue: tcgen05.ld of 16 columns (batch rows) at a time,
//               logits stores (coalesced along the vocabulary), and the
//               per-row running maximum (value, id) in shared memory
// A second tiny kernel merges the per-CTA maxima into tokens.
//
// Every wait is bounded (kWaitBudget); a wait that runs out sets the error
// flag, its role stops, and the CTA drains its copies in flight and frees its
// TMEM before returning. The rows then report RL_ERR_TIMEOUT.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <climits>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace rl {

constexpr int kLmThreads = 192;            // 6 warps
constexpr int kLmBM = 128;                 // vocabulary rows per tile (MMA M)
constexpr int kLmBK = 64;                  // K elements per stage (128 bytes of bf16)
constexpr int kLmATile = kLmBM * kLmBK * 2;  // 16 KB
constexpr int kLmMaxN = 256;               // batch rows per launch (MMA N limit)
constexpr int kLmStageCap = 200 * 1024;    // shared memory for the stages
constexpr int kLmMaxStages = 12;

struct LmArgs {
  int B, H, V, N;        // N: batch padded to a multiple of 16
  int ntiles, kblocks, stages;
  uint32_t stage_bytes;  // A tile + B tile
  uint32_t tmem_cols;    // 2 * N rounded up to a power of two (>= 32)
  float* out_f32;        // [B, ldo] or null
  uint16_t* out_bf16;    // [B, ldo] or null
  int64_t ldo;
  uint64_t* part;        // [B, gridDim.x] packed (value, id) maxima, or null
  int* err;              // set to 1 when a wait runs out
};

namespace {

__device__ __forceinline__ uint64_t lm_policy_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t lm_policy_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tiled TMA load into this CTA's shared memory (no multicast); x is the
// K coordinate, always a multiple of 64 elements (128 bytes).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major operand with the 128-byte swizzle
// (8-row groups of 1024 bytes: stride byte offset 1024; the leading byte
// offset is unused for this layout and set to 16 bytes), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3fffu) | (static_cast<uint64_t>(1u) << 16) |
         (static_cast<uint64_t>(1024u >> 4) << 32) | (static_cast<uint64_t>(1u) << 46) |
         (static_cast<uint64_t>(2u) << 61);
}

// Instruction descriptor of kind::f16: bf16 A and B (both K-major), f32
// accumulator, M = 128, N = n.
__device__ __forceinline__ uint32_t lm_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
  const uint32_t z = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

// Arrives on `bar` once every tcgen05 operation this thread issued before it
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 TMEM lanes (this warp's quadrant) x 16 columns: register j of lane l is
// column col + j of lane (quadrant base + l).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// (value, id) packed so that the larger u64 is the later maximum: the
// greedy_sample order (last maximum; -0.0 and +0.0 tie).
__device__ __forceinline__ uint64_t lm_key(float v, int id) {
  return (static_cast<uint64_t>(ord_key(__fadd_rn(v, 0.0f))) << 32) | static_cast<uint32_t>(id);
}
__device__ __forceinline__ uint64_t umax64(uint64_t a, uint64_t b) { return a > b ? a : b; }
__device__ __forceinline__ uint64_t shfl_xor64(uint64_t v, int o) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v), o);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v >> 32), o);
  return (static_cast<uint64_t>(hi) << 32) | lo;
}

// Per-column maximum over the warp's 32 lanes for 16 columns, by a
// transposing butterfly (31 exchanges instead of 16 x 5): afterwards lane l
// holds column (l & 15).
__device__ __forceinline__ uint64_t warp_colmax16(uint64_t (&k)[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 16; ++j) k[j] = umax64(k[j], shfl_xor64(k[j], 16));
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const bool up = (lane & 8) != 0;
    const uint64_t send = up ? k[j] : k[j + 8];
    const uint64_t keep = up ? k[j + 8] : k[j];
    k[j] = umax64(keep, shfl_xor64(send, 8));
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const bool up = (lane & 4) != 0;
    const uint64_t send = up ? k[j] : k[j + 4];
    const uint64_t keep = up ? k[j + 4] : k[j];
    k[j] = umax64(keep, shfl_xor64(send, 4));
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const bool up = (lane & 2) != 0;
    const uint64_t send = up ? k[j] : k[j + 2];
    const uint64_t keep = up ? k[j + 2] : k[j];
    k[j] = umax64(keep, shfl_xor64(send, 2));
  }
  const bool up = (lane & 1) != 0;
  const uint64_t send = up ? k[0] : k[1];
  const uint64_t keep = up ? k[1] : k[0];
  return umax64(keep, shfl_xor64(send, 1));
}

}  // namespace

__global__ void __launch_bounds__(kLmThreads, 1)
    lmhead_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                  const __grid_constant__ LmArgs a) {
  extern __shared__ uint8_t lm_smem_raw[];
  uint8_t* base = lm_smem_raw + ((1024u - (smem_u32(lm_smem_raw) & 1023u)) & 1023u);
  const int S = a.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + static_cast<size_t>(S) * a.stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;   // [2]
  uint64_t* tempty = tfull + 2;  // [2]
  uint64_t* done = tempty + 2;
  uint64_t* best = done + 1;     // [N]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(best + a.N);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&tfull[j], 1);
      mbar_init(&tempty[j], 4);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < a.N; i += kLmThreads) best[i] = 0ull;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- producer ----
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
    const uint64_t pol_w = lm_policy_first();  // the weight streams once
    const uint64_t pol_x = lm_policy_last();   // the hidden rows are read by every CTA
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < a.kblocks; ++kb) {
        const int s = static_cast<int>(it % S);
        const uint32_t ph = (it / S) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, kWaitBudget)) {
          ok = false;
          break;
        }
        uint8_t* st = base + static_cast<size_t>(s) * a.stage_bytes;
        mbar_expect_tx(&full[s], a.stage_bytes);
        tma_load_2d(st, &tmW, kb * kLmBK, tile * kLmBM, &full[s], pol_w);
        tma_load_2d(st + kLmATile, &tmX, kb * kLmBK, 0, &full[s], pol_x);
        ++it;
      }
    }
    if (!ok) atomicExch(a.err, 1);
    // every issued copy lands before the CTA may return
    for (int s = 0; s < S; ++s) {
      const uint32_t n = it / S + (static_cast<uint32_t>(s) < it % S ? 1u : 0u);
      if (n > 0 && !mbar_wait(&full[s], (n - 1u) & 1u, kWaitBudget)) atomicExch(a.err, 1);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    const uint32_t idesc = lm_idesc(a.N);
    uint32_t it = 0;
    int local = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x, ++local) {
      const int j = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&tempty[j], (use & 1u) ^ 1u, kWaitBudget)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + static_cast<uint32_t>(j * a.N);
      for (int kb = 0; kb < a.kblocks; ++kb) {
        const int s = static_cast<int>(it % S);
        if (!mbar_wait(&full[s], (it / S) & 1u, kWaitBudget)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(base + static_cast<size_t>(s) * a.stage_bytes);
        const uint64_t ad = sw128_desc(sa), bd = sw128_desc(sa + kLmATile);
#pragma unroll
        for (int k = 0; k < kLmBK / 16; ++k)  // 32 bytes of K per instruction: +2 in the address field
          umma_bf16(d, ad + 2u * k, bd + 2u * k, idesc, (kb | k) != 0);
        umma_commit(&empty[s]);
        ++it;
      }
      if (!ok) break;
      umma_commit(&tfull[j]);
    }
    if (!ok) atomicExch(a.err, 1);
    // every MMA of this CTA completes before its TMEM is freed
    umma_commit(done);
    if (!mbar_wait(done, 0u, kWaitBudget)) atomicExch(a.err, 1);
  } else if (warp >= 2) {
    // ---- epilogue ----
    const int q = warp & 3;  // TMEM lane quadrant this warp may read
    int local = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x, ++local) {
      const int j = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&tfull[j], use & 1u, kWaitBudget)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int v = tile * kLmBM + q * 32 + lane;
      const bool vin = v < a.V;
      const uint32_t tcol = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(j * a.N);
      for (int c0 = 0; c0 < a.N; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tcol + static_cast<uint32_t>(c0), r);
        if (c0 + 16 >= a.N) {
          // the accumulator buffer is free for the MMAs of a later tile
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive1(&tempty[j]);
        }
        if (vin) {
          if (a.out_f32) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
              if (c0 + jj < a.B) a.out_f32[static_cast<int64_t>(c0 + jj) * a.ldo + v] = __uint_as_float(r[jj]);
          }
          if (a.out_bf16) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
              if (c0 + jj < a.B)
                a.out_bf16[static_cast<int64_t>(c0 + jj) * a.ldo + v] =
                    __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(r[jj])));
          }
        }
        if (a.part) {
          uint64_t k[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) k[jj] = vin ? lm_key(__uint_as_float(r[jj]), v) : 0ull;
          const uint64_t m = warp_colmax16(k);
          if (lane < 16 && c0 + lane < a.B) atomicMax(reinterpret_cast<unsigned long long*>(&best[c0 + lane]),
                                                     static_cast<unsigned long long>(m));
        }
      }
    }
    if (!ok) atomicExch(a.err, 1);
  }
  __syncthreads();
  if (a.part)
    for (int b = threadIdx.x; b < a.B; b += kLmThreads) a.part[static_cast<int64_t>(b) * gridDim.x + blockIdx.x] = best[b];
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
  }
}

// Row b's token: the largest packed key over the G CTA maxima (last maximum).
__global__ void lmhead_argmax_kernel(const uint64_t* __restrict__ part, int B, int G, const int* err,
                                     int32_t* __restrict__ out_tok, int32_t* __restrict__ row_status) {
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= B) return;
  uint64_t m = 0ull;
  for (int g = lane; g < G; g += 32) m = umax64(m, part[static_cast<int64_t>(b) * G + g]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = umax64(m, shfl_xor64(m, o));
  if (lane == 0) {
    const bool bad = *err != 0;
    out_tok[b] = bad ? -1 : static_cast<int32_t>(m & 0xffffffffu);
    if (row_status) row_status[b] = bad ? RL_ERR_TIMEOUT : RL_OK;
  }
}

// Marks every row RL_ERR_TIMEOUT (token -1) when the GEMM reported a wait
// that ran out.
__global__ void lmhead_flag_kernel(const int* err, int B, int32_t* out_tok, int32_t* row_status) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B || *err == 0) return;
  out_tok[b] = -1;
  if (row_status) row_status[b] = RL_ERR_TIMEOUT;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::atomic<EncodeTiledFn> fn{nullptr};
  EncodeTiledFn f = fn.load(std::memory_order_acquire);
  if (!f) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess && p) {
      f = reinterpret_cast<EncodeTiledFn>(p);
      fn.store(f, std::memory_order_release);
    }
  }
  return f;
}

// A [rows, H] bf16 matrix (row stride ld elements) as 64 x box_rows tiles
// with the 128-byte swizzle; rows past the end read as zeros.
bool make_map(CUtensorMap* m, const void* ptr, int H, int rows, int64_t ld, int box_rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2u};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kLmBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1u, 1u};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

uint32_t pow2_cols(int n) {
  uint32_t c = 32u;
  while (c < static_cast<uint32_t>(n)) c <<= 1;
  return c;
}

}  // namespace

// The launch geometry of one batch chunk (B <= 256): exposed for the tests
// of the host checks.
void lmhead_plan(int B, int H, int V, int num_sms, LmArgs* a, int* grid, size_t* smem) {
  a->B = B;
  a->H = H;
  a->V = V;
  a->N = (B + 15) / 16 * 16;
  a->ntiles = (V + kLmBM - 1) / kLmBM;
  a->kblocks = H / kLmBK;
  a->stage_bytes = static_cast<uint32_t>(kLmATile + a->N * kLmBK * 2);
  a->stages = kLmStageCap / static_cast<int>(a->stage_bytes);
  if (a->stages > kLmMaxStages) a->stages = kLmMaxStages;
  a->tmem_cols = pow2_cols(2 * a->N);
  *grid = a->ntiles < num_sms ? a->ntiles : num_sms;
  *smem = 1024 + static_cast<size_t>(a->stages) * a->stage_bytes + (2 * a->stages + 5) * 8 + a->N * 8 + 16;
}

// Launches the GEMM (and, with out_tok, the argmax merge) for rows [0, B) of
// hidden; B may exceed 256 (chunks of 256 rows, the weight streamed once per
// chunk).
rl_status lmhead_launch(rl_sampler* h, const uint16_t* hidden, int64_t ldh, const uint16_t* weight, int64_t ldw,
                        int B, int H, int V, float* out_f32, uint16_t* out_bf16, int64_t ldo, int32_t* out_tok,
                        int32_t* row_status, cudaStream_t stream) {
  static std::atomic<int> configured[64];
  int dev = h->device;
  if (dev >= 0 && dev < 64 && !configured[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(lmhead_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
      return set_error(RL_ERR_CUDA, "rl_lmhead: cudaFuncSetAttribute failed");
    configured[dev].store(1, std::memory_order_release);
  }
  if (cudaMemsetAsync(h->lm_err, 0, sizeof(int), stream) != cudaSuccess)
    return set_error(RL_ERR_CUDA, "rl_lmhead: cudaMemsetAsync failed");
  CUtensorMap mw;
  if (!make_map(&mw, weight, H, V, ldw, kLmBM))
    return set_error(RL_ERR_INVALID_ARG, "rl_lmhead: weight tensor map rejected (alignment or stride)");
  for (int b0 = 0; b0 < B; b0 += kLmMaxN) {
    const int Bc = B - b0 < kLmMaxN ? B - b0 : kLmMaxN;
    LmArgs a = {};
    int grid = 0;
    size_t smem = 0;
    lmhead_plan(Bc, H, V, h->num_sms, &a, &grid, &smem);
    CUtensorMap mx;
    if (!make_map(&mx, hidden + static_cast<int64_t>(b0) * ldh, H, Bc, ldh, a.N))
      return set_error(RL_ERR_INVALID_ARG, "rl_lmhead: hidden tensor map rejected (alignment or stride)");
    a.out_f32 = out_f32 ? out_f32 + static_cast<int64_t>(b0) * ldo : nullptr;
    a.out_bf16 = out_bf16 ? out_bf16 + static_cast<int64_t>(b0) * ldo : nullptr;
    a.ldo = ldo;
    a.part = out_tok ? h->lm_part : nullptr;
    a.err = h->lm_err;
    lmhead_kernel<<<grid, kLmThreads, smem, stream>>>(mw, mx, a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(RL_ERR_CUDA, cudaGetErrorString(e));
    if (out_tok) {
      lmhead_argmax_kernel<<<(Bc + 7) / 8, 256, 0, stream>>>(h->lm_part, Bc, grid, h->lm_err, out_tok + b0,
                                                             row_status ? row_status + b0 : nullptr);
      e = cudaGetLastError();
      if (e != cudaSuccess) return set_error(RL_ERR_CUDA, cudaGetErrorString(e));
    }
  }
  return RL_OK;
}

}  // namespace rl

namespace {

struct LmDeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit LmDeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~LmDeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

rl_status lm_check(rl_sampler* h, const uint16_t* hidden, int64_t ldh, const uint16_t* weight, int64_t ldw, int B,
                   int H, int V, const char* who) {
  if (!h) return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead: handle is NULL");
  if (B < 0 || H <= 0 || V <= 0 || ldh < H || ldw < H)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead: bad B / H / V / ld");
  if (B > 0 && (!hidden || !weight)) return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead: hidden and weight are required");
  if (H % rl::kLmBK != 0) return rl::set_error(RL_ERR_UNSUPPORTED, "rl_lmhead: H must be a multiple of 64");
  if ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(weight)) & 15u)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead: hidden and weight must be 16-byte aligned");
  if ((ldh % 8) || (ldw % 8)) return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead: row strides must be multiples of 8 elements");
  if (B > h->max_batch) return rl::set_error(RL_ERR_SHAPE, "rl_lmhead: B beyond the handle's max_batch");
  (void)who;
  return RL_OK;
}

}  // namespace

extern "C" {
#pragma GCC visibility push(default)

rl_status rl_lmhead_logits(rl_sampler* h, const uint16_t* hidden, int64_t ldh, const uint16_t* weight, int64_t ldw,
                           int B, int H, int V, void* out_logits, rl_dtype out_dtype, int64_t ldo, void* stream) {
  rl_status st = lm_check(h, hidden, ldh, weight, ldw, B, H, V, "rl_lmhead_logits");
  if (st != RL_OK) return st;
  if (B > 0 && !out_logits) return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead_logits: out_logits is required");
  if (out_dtype != RL_F32 && out_dtype != RL_BF16) return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead_logits: bad dtype");
  if (ldo < V) return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead_logits: ldo < V");
  if (B == 0) return RL_OK;
  LmDeviceGuard g(h->device);
  if (!g.ok) return rl::set_error(RL_ERR_CUDA, "rl_lmhead_logits: cudaSetDevice failed");
  return rl::lmhead_launch(h, hidden, ldh, weight, ldw, B, H, V,
                           out_dtype == RL_F32 ? static_cast<float*>(out_logits) : nullptr,
                           out_dtype == RL_BF16 ? static_cast<uint16_t*>(out_logits) : nullptr, ldo, nullptr, nullptr,
                           static_cast<cudaStream_t>(stream));
}

rl_status rl_lmhead_greedy(rl_sampler* h, const uint16_t* hidden, int64_t ldh, const uint16_t* weight, int64_t ldw,
                           int B, int H, int V, int32_t* out_tok, int32_t* row_status, float* out_logits, int64_t ldo,
                           void* stream) {
  rl_status st = lm_check(h, hidden, ldh, weight, ldw, B, H, V, "rl_lmhead_greedy");
  if (st != RL_OK) return st;
  if (B > 0 && !out_tok) return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead_greedy: out_tok is required");
  if (out_logits && ldo < V) return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead_greedy: ldo < V");
  if (B == 0) return RL_OK;
  LmDeviceGuard g(h->device);
  if (!g.ok) return rl::set_error(RL_ERR_CUDA, "rl_lmhead_greedy: cudaSetDevice failed");
  return rl::lmhead_launch(h, hidden, ldh, weight, ldw, B, H, V, out_logits, nullptr, ldo, out_tok, row_status,
                           static_cast<cudaStream_t>(stream));
}

rl_status rl_lmhead_sample(rl_sampler* h, const uint16_t* hidden, int64_t ldh, const uint16_t* weight, int64_t ldw,
                           int B, int H, int V, const int32_t* hist, const int32_t* hist_len, int hist_stride,
                           const rl_row_params* params, const float* uniforms, int32_t* out_tok, float* out_prob,
                           int32_t* row_status, void* stream) {
  rl_status st = lm_check(h, hidden, ldh, weight, ldw, B, H, V, "rl_lmhead_sample");
  if (st != RL_OK) return st;
  if (V > h->max_vocab) return rl::set_error(RL_ERR_SHAPE, "rl_lmhead_sample: V beyond the handle's max_vocab");
  if (B > 0 && (!params || !uniforms || !out_tok))
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_lmhead_sample: params, uniforms and out_tok are required");
  if (!h->stage_logits) return rl::set_error(RL_ERR_UNSUPPORTED, "rl_lmhead_sample: handle without staging buffers");
  if (B == 0) return RL_OK;
  LmDeviceGuard g(h->device);
  if (!g.ok) return rl::set_error(RL_ERR_CUDA, "rl_lmhead_sample: cudaSetDevice failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = rl::lmhead_launch(h, hidden, ldh, weight, ldw, B, H, V, h->stage_logits, nullptr, V, nullptr, nullptr, s);
  if (st != RL_OK) return st;
  st = rl_sample_batch(h, h->stage_logits, RL_F32, B, V, V, hist, hist_len, hist_stride, nullptr, 0, params, uniforms,
                       out_tok, out_prob, row_status, stream);
  if (st != RL_OK) return st;
  // a GEMM whose wait ran out leaves its rows' logits undefined
  rl::lmhead_flag_kernel<<<(B + 255) / 256, 256, 0, s>>>(h->lm_err, B, out_tok, row_status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, cudaGetErrorString(e));
  return RL_OK;
}

#pragma GCC visibility pop
}  // extern "C"
