// Entry points whose kernels are not built yet: they report RL_ERR_UNSUPPORTED.
#include "internal.h"
#include "rl_sampler.h"

extern "C" {
#pragma GCC visibility push(default)

rl_status rl_decoder_sample(rl_sampler*, const float*, int, int, int64_t, const float*, const float*,
                            const float*, int32_t*, float*, void*) {
  return rl::set_error(RL_ERR_UNSUPPORTED, "rl_decoder_sample: not built yet");
}

}  // extern "C"
