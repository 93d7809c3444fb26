// Asymmetric 2-bit group quantization arithmetic, bit-exact with the
// reference's Triton quantizers (quant_kernel.py:77-98 for K, :166-183 for V):
// IEEE float32 in the reference's order, written with explicit
// round-to-nearest intrinsics so that no contraction or fast-math path can
// change a bit:
//   scale = (max - min) / 3, scale == 0 -> 1,
//   zero  = floor(-min / scale + 0.5),
//   code  = clamp(floor(x / scale + 0.5) + zero, 0, 3),
// scale and zero stored as float16 (round to nearest even), codes computed
// with the float32 scale.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace nsa {

struct GroupParams {
  float scale, zero;
};

__device__ __forceinline__ GroupParams group_params(float mn, float mx) {
  float scale = __fdiv_rn(__fsub_rn(mx, mn), 3.0f);
  if (scale == 0.0f) scale = 1.0f;
  const float zero = floorf(__fadd_rn(__fdiv_rn(-mn, scale), 0.5f));
  return {scale, zero};
}

__device__ __forceinline__ uint32_t code_of(float x, const GroupParams& g) {
  float q = __fadd_rn(floorf(__fadd_rn(__fdiv_rn(x, g.scale), 0.5f)), g.zero);
  q = fminf(fmaxf(q, 0.0f), 3.0f);
  return static_cast<uint32_t>(q);
}

}  // namespace nsa
