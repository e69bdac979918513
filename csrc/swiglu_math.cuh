// SwiGLU activation math shared by the fused GEMM epilogues (gemm.cu) and the standalone
// SwiGLU kernels (elementwise.cu), so that both paths give bit-identical results.
//
//   silu(g) = g * sigmoid(g),  d silu / dg = sigmoid(g) * (1 + g * (1 - sigmoid(g)))
//
// The sigmoid uses the fast single-precision division: its error (a few fp32 ulp) is far below
// the bf16 rounding of every output.  exp overflow (g < -88) gives 1 / inf = 0, the right limit.
#pragma once

#include <cuda_runtime.h>

namespace mimir {

__device__ __forceinline__ float swiglu_sigmoid(float g) { return __fdividef(1.f, 1.f + __expf(-g)); }
__device__ __forceinline__ float swiglu_silu(float g) { return g * swiglu_sigmoid(g); }

// (d gate, d up) of silu(gate) * up for the incoming gradient d.
__device__ __forceinline__ void swiglu_backward(float d, float g, float u, float& dg, float& du) {
  const float s = swiglu_sigmoid(g);
  du = d * g * s;
  dg = d * u * s * (1.f + g * (1.f - s));
}

}  // namespace mimir
