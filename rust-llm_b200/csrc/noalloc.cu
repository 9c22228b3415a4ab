// rl_sample_batch_static: spec sampling with no handle and no allocation.
//
// Some callers cannot allocate device memory at the point where they sample:
// code running inside a CUDA-graph capture (cudaMalloc is not capturable and
// synchronises the device), latency-critical decode loops that must not hit
// the allocator, and foreign-function callers that have nowhere to keep a
// handle's lifetime. This entry point serves them with the same kernel as
// rl_sample_batch, run with one segment per row so that its only scratch is
// the per-warp candidate overflow, which lives in a fixed file-scope device
// array instead of a handle's workspace.
//
// Limits: the scratch holds kStaticCtas CTAs' overflow areas (the grid is
// capped there; the persistent CTAs loop over the rows), 9.7 MB of device
// memory reserved when the library's module loads. Rows, vocabulary and
// history are limited as for rl_sample_batch (V <= 2^21 - 4096, history
// <= 1024 entries per row); larger sizes are rejected with RL_ERR_SHAPE.
//
// Nothing in the scratch must start at zero: every overflow slot is written
// before it is read within a launch. Two calls that overlap in time on the
// same device (different streams, or host threads) share the scratch and
// race; serialise them.
#include <cuda_runtime.h>

#include <mutex>

#include "internal.h"

namespace {

constexpr int kStaticCtas = 296;  // 2 CTAs per SM on a 148-SM B200
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned long long g_static_ovf[static_cast<size_t>(kStaticCtas) * rl::kCW * rl::kWovf];

struct DevState {
  int ready = 0;
  int num_sms = 0;
  void* ovf = nullptr;
};
DevState g_dev[kMaxDevices];
std::mutex g_mu;

// Per-device set-up on the first call (the SM count; both dtypes' kernels
// configured, so that no later call does it inside a capture), and the
// scratch's device address with that device current. The address is looked
// up again on every call made outside a stream capture -- a reset device
// reloads the module, and the address may move -- and taken from the cache
// inside a capture. Nothing here allocates.
rl_status device_state(cudaStream_t stream, DevState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, "rl_sample_batch_static: cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return rl::set_error(RL_ERR_UNSUPPORTED, "rl_sample_batch_static: device index too large");
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(stream, &cap);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return rl::set_error(RL_ERR_CUDA, "rl_sample_batch_static: cudaStreamIsCapturing failed");
  }
  std::lock_guard<std::mutex> lock(g_mu);
  DevState& d = g_dev[dev];
  if (!d.ready) {
    if (cap != cudaStreamCaptureStatusNone)
      return rl::set_error(RL_ERR_UNSUPPORTED,
                           "rl_sample_batch_static: the first call on a device must come before any stream capture");
    int major = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, "rl_sample_batch_static: device query failed");
    if (major < 10) return rl::set_error(RL_ERR_UNSUPPORTED, "rl_sample_batch_static: this library is built for sm_100a");
    e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, "rl_sample_batch_static: device query failed");
    e = rl::spec_configure_single();
    if (e != cudaSuccess) {
      cudaGetLastError();
      return rl::set_error(RL_ERR_CUDA, "rl_sample_batch_static: kernel configuration failed");
    }
  }
  if (!d.ready || cap == cudaStreamCaptureStatusNone) {
    e = cudaGetSymbolAddress(&d.ovf, g_static_ovf);
    if (e != cudaSuccess) {
      cudaGetLastError();
      d.ready = 0;
      return rl::set_error(RL_ERR_CUDA, "rl_sample_batch_static: cudaGetSymbolAddress of the scratch failed");
    }
    d.ready = 1;
  }
  *out = &d;
  return RL_OK;
}

// Whether device pointer p lives on device dev (or is managed memory that
// dev can use); queried without allocating.
bool on_device(const void* p, int dev) {
  if (!p) return true;
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (at.type == cudaMemoryTypeManaged) return true;
  return at.type == cudaMemoryTypeDevice && at.device == dev;
}

}  // namespace

extern "C" {
#pragma GCC visibility push(default)

rl_status rl_sample_batch_static(const void* logits, rl_dtype dtype, int B, int V, int64_t ld, const int32_t* hist,
                                 const int32_t* hist_len, int hist_stride, const uint32_t* mask, int64_t mask_stride,
                                 const rl_row_params* params, const float* uniforms, int32_t* out_tok,
                                 float* out_prob, int32_t* row_status, void* stream) {
  rl::clear_error();
  if (B < 0 || V <= 0) return rl::set_error(RL_ERR_INVALID_ARG, "rl_sample_batch_static: bad B or V");
  if (B == 0) return RL_OK;
  if (!logits || !params || !uniforms || !out_tok)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_sample_batch_static: logits, params, uniforms and out_tok are required");
  if (dtype != RL_F32 && dtype != RL_BF16) return rl::set_error(RL_ERR_INVALID_ARG, "rl_sample_batch_static: bad dtype");
  if (ld < V) return rl::set_error(RL_ERR_INVALID_ARG, "rl_sample_batch_static: ld < V");
  if (B > 65535) return rl::set_error(RL_ERR_SHAPE, "rl_sample_batch_static: B > 65535");
  if (V > (1 << 21) - rl::kCE) return rl::set_error(RL_ERR_SHAPE, "rl_sample_batch_static: V > 2093056");
  if (hist) {
    if (!hist_len) return rl::set_error(RL_ERR_INVALID_ARG, "rl_sample_batch_static: hist without hist_len");
    if (hist_stride < 0 || hist_stride > rl::kHmax)
      return rl::set_error(RL_ERR_SHAPE, "rl_sample_batch_static: hist_stride beyond 1024");
  }
  if (mask && mask_stride < (V + 31) / 32)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_sample_batch_static: mask_stride < ceil(V/32)");
  DevState* d = nullptr;
  rl_status st = device_state(static_cast<cudaStream_t>(stream), &d);
  if (st != RL_OK) return st;
  // the kernel runs on the current device with that device's scratch: its
  // buffers must be there too (a peer's memory would fault without peer access)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return rl::set_error(RL_ERR_CUDA, "rl_sample_batch_static: cudaGetDevice failed");
  if (!on_device(logits, dev) || !on_device(out_tok, dev) || !on_device(params, dev) || !on_device(uniforms, dev) ||
      !on_device(out_prob, dev) || !on_device(row_status, dev) || !on_device(hist, dev) || !on_device(hist_len, dev) ||
      !on_device(mask, dev))
    return rl::set_error(RL_ERR_INVALID_ARG,
                         "rl_sample_batch_static: every buffer must be device memory of the current device");
  rl::SpecArgs a = {};
  a.logits = logits;
  a.ld = ld;
  a.B = B;
  a.V = V;
  a.hist = hist;
  a.hist_len = hist_len;
  a.hist_stride = hist ? hist_stride : 0;
  a.mask = mask;
  a.mask_stride = mask_stride;
  a.params = params;
  a.uniforms = uniforms;
  a.out_tok = out_tok;
  a.out_prob = out_prob;
  a.row_status = row_status;
  a.ws.wovf = static_cast<uint64_t*>(d->ovf);
  const cudaError_t e =
      rl::launch_spec_single(a, dtype, d->num_sms, kStaticCtas, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, "rl_sample_batch_static: kernel launch failed");
  return RL_OK;
}

#pragma GCC visibility pop
}  // extern "C"
