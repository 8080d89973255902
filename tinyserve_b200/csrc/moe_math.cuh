// Expert activation shared by the decode and prefill kernels.
#pragma once
#include "../../include/tsb_moe.h"

namespace tsb {

// TSB_ACT_SWIGLU_OAI: g = min(gate, limit); u = clamp(up, -limit, limit);
// (u + 1) * g * sigmoid(alpha * g)   (tinyserve/expert_forward.py:185-187)
// TSB_ACT_SILU: silu(gate) * up      (tinyserve/ggml_forward.py:112)
// The sigmoid uses the fast exponential and division intrinsics (a few ulp,
// far inside the layer tolerance); exp overflow gives a zero reciprocal.
__device__ __forceinline__ float act_fn(int act, float gate, float up, float limit, float alpha) {
  if (act == TSB_ACT_SWIGLU_OAI) {
    const float g = fminf(gate, limit);
    const float u = fminf(fmaxf(up, -limit), limit);
    return (u + 1.f) * g * __fdividef(1.f, 1.f + __expf(-alpha * g));
  }
  return __fdividef(gate, 1.f + __expf(-gate)) * up;
}

}  // namespace tsb
