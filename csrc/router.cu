// MoE router selection and routing-balance statistics in one pass.
//
// For every token t: chosen[t, 0..k) = the k experts with the largest selection value sel[t, e]
// (the router's scores, or its sigmoid affinities plus the balancing bias, computed by the
// caller), ordered by value, ties going to the lower expert index (the order of a stable
// descending argsort), and load[e] += the number of tokens that chose expert e (the
// routing-balance counts of one forward).
//
// One warp per token; each lane holds experts lane, lane + 32, ... (up to kMaxExperts); k rounds
// of a warp arg-max with index tie-break.  Loads are accumulated in a shared-memory histogram per
// CTA and added to the global counts with one atomic per expert and CTA.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

namespace {

constexpr int kWarps = 8;
constexpr int kPerLane = 8;
constexpr int kMaxExperts = 32 * kPerLane;

// (value, index) pair comparison: larger value wins, equal values go to the smaller index.
__device__ __forceinline__ bool better(float v, int i, float w, int j) { return v > w || (v == w && i < j); }

__global__ void __launch_bounds__(kWarps * 32) router_topk_kernel(const float* __restrict__ sel, int64_t T, int E,
                                                                   int k, int64_t* __restrict__ chosen,
                                                                   int64_t* __restrict__ load) {
  __shared__ int hist[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t t = int64_t(blockIdx.x) * kWarps + threadIdx.x / 32;
  if (t < T) {
    float v[kPerLane];
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int e = lane + 32 * j;
      v[j] = e < E ? sel[t * E + e] : -INFINITY;
    }
    for (int r = 0; r < k; ++r) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < kPerLane; ++j) {
        const int e = lane + 32 * j;
        if (e < E && better(v[j], e, bv, bi)) bv = v[j], bi = e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
      }
      if (lane == 0) {
        chosen[t * k + r] = bi;
        atomicAdd(&hist[bi], 1);
      }
      if ((bi & 31) == lane) v[bi >> 5] = -INFINITY;  // remove the winner (its owner lane)
    }
  }
  __syncthreads();
  if (load != nullptr)
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      if (hist[e]) atomicAdd(reinterpret_cast<unsigned long long*>(load + e), static_cast<unsigned long long>(hist[e]));
}

}  // namespace

// sel: fp32 [T, E] selection values; load: optional int64 [E] accumulated in place.
// Returns chosen int64 [T, k].
at::Tensor router_topk(at::Tensor scores, int64_t k, c10::optional<at::Tensor> load) {
  TORCH_CHECK(scores.is_cuda() && scores.dtype() == at::kFloat && scores.dim() == 2 && scores.is_contiguous(),
              "scores: contiguous fp32 [T, E]");
  const int64_t T = scores.size(0);
  const int E = static_cast<int>(scores.size(1));
  TORCH_CHECK(E >= 1 && E <= kMaxExperts && k >= 1 && k <= E, "1 <= k <= E <= ", kMaxExperts);
  if (load) TORCH_CHECK(load->is_cuda() && load->dtype() == at::kLong && load->numel() == E && load->is_contiguous(),
                        "load: int64 [E]");
  const c10::cuda::CUDAGuard guard(scores.device());
  at::Tensor chosen = at::empty({T, k}, scores.options().dtype(at::kLong));
  if (T == 0) return chosen;
  router_topk_kernel<<<static_cast<unsigned>((T + kWarps - 1) / kWarps), kWarps * 32, 0,
                       at::cuda::getCurrentCUDAStream()>>>(
      scores.data_ptr<float>(), T, E, static_cast<int>(k), chosen.data_ptr<int64_t>(),
      load ? load->data_ptr<int64_t>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return chosen;
}
