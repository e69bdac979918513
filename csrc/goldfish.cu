// Goldfish label-drop mask on the GPU, one CTA per packed sequence, no host synchronisation.
//
// For token p of a sequence (0-based position) the hash XORs, over offsets o = 1..min(w, n), a
// splitmix64 finaliser of  ctx(p, o) + seed * c2 + o * c3,  where ctx = tok[p - o] * c0 + p * c1
// when p >= o and 0 otherwise; the label is dropped when it is supervised and |hash| mod k == 0.
// All arithmetic is two's-complement int64 as in PyTorch's integer tensors: products and sums
// wrap (computed in uint64), shifts are arithmetic, |INT64_MIN| stays INT64_MIN, and mod is the
// floor modulus (PyTorch's remainder), so the mask equals the PyTorch formulation bit for bit.
// cu_seqlens may be padded with zeros after the last bound: pairs with end <= start are skipped.
//
// Reference: `src/mimir/model/goldfish_loss.py:34-124` (hash strategy).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

namespace {

__device__ __forceinline__ int64_t wrap_mul(int64_t a, int64_t b) {
  return static_cast<int64_t>(static_cast<uint64_t>(a) * static_cast<uint64_t>(b));
}
__device__ __forceinline__ int64_t wrap_add(int64_t a, int64_t b) {
  return static_cast<int64_t>(static_cast<uint64_t>(a) + static_cast<uint64_t>(b));
}

struct Mix {
  int64_t c_tok, c_pos, c_seed, c_off, s0, s1;
};

__device__ __forceinline__ int64_t splitmix(int64_t x, const Mix& m) {
  x ^= x >> 30;  // arithmetic shift of a signed value, as PyTorch's >> on int64
  x = wrap_mul(x, m.s0);
  x ^= x >> 27;
  x = wrap_mul(x, m.s1);
  return x ^ (x >> 31);
}

template <typename TI>
__global__ void goldfish_kernel(const TI* __restrict__ tok, const bool* __restrict__ supervised,
                                const int32_t* __restrict__ cu, bool* __restrict__ drop, Mix m, int64_t k, int w,
                                int64_t seed) {
  const int64_t start = cu[blockIdx.x], end = cu[blockIdx.x + 1];
  if (end <= start) return;
  const int64_t n = end - start;
  const int64_t seed_term = wrap_mul(seed, m.c_seed);
  const int64_t width = n < w ? n : static_cast<int64_t>(w);
  for (int64_t p = threadIdx.x; p < n; p += blockDim.x) {
    const int64_t t = start + p;
    if (!supervised[t]) continue;
    int64_t h = 0;
    for (int64_t o = 1; o <= width; ++o) {
      const int64_t ctx = p >= o ? wrap_add(wrap_mul(static_cast<int64_t>(tok[t - o]), m.c_tok), wrap_mul(p, m.c_pos))
                                 : 0;
      h ^= splitmix(wrap_add(wrap_add(ctx, seed_term), wrap_mul(o, m.c_off)), m);
    }
    const int64_t a = h < 0 ? static_cast<int64_t>(0ull - static_cast<uint64_t>(h)) : h;  // |INT64_MIN| wraps
    int64_t r = a % k;
    if (r < 0) r += k;  // floor modulus for the one negative case
    drop[t] = r == 0;
  }
}

}  // namespace

// drop[T] (bool): supervised tokens whose context hash is divisible by k.  inputs: int32/int64 [T];
// supervised: bool [T]; cu_seqlens: int32 (padded bounds allowed); mix: the six constants
// (c_tok, c_pos, c_seed, c_off, splitmix0, splitmix1) as signed int64.
at::Tensor goldfish_mask(at::Tensor inputs, at::Tensor supervised, at::Tensor cu_seqlens, int64_t k,
                         int64_t context_width, int64_t seed, std::vector<int64_t> mix) {
  TORCH_CHECK(inputs.is_cuda() && inputs.dim() == 1 && inputs.is_contiguous(), "inputs: contiguous 1-D CUDA tensor");
  TORCH_CHECK(inputs.scalar_type() == at::kInt || inputs.scalar_type() == at::kLong, "inputs: int32 or int64");
  TORCH_CHECK(supervised.scalar_type() == at::kBool && supervised.is_contiguous() &&
                  supervised.numel() == inputs.numel(), "supervised: bool, one per token");
  TORCH_CHECK(cu_seqlens.scalar_type() == at::kInt && cu_seqlens.is_contiguous() && cu_seqlens.dim() == 1,
              "cu_seqlens: int32");
  TORCH_CHECK(k >= 2 && context_width >= 1 && mix.size() == 6, "goldfish: k >= 2, width >= 1, six constants");
  const c10::cuda::CUDAGuard guard(inputs.device());
  auto drop = at::zeros_like(supervised);
  const int64_t pairs = cu_seqlens.numel() - 1;
  if (pairs <= 0 || inputs.numel() == 0) return drop;
  Mix m{mix[0], mix[1], mix[2], mix[3], mix[4], mix[5]};
  auto st = at::cuda::getCurrentCUDAStream();
  const dim3 grid(static_cast<unsigned>(pairs));
  if (inputs.scalar_type() == at::kInt)
    goldfish_kernel<int32_t><<<grid, 256, 0, st>>>(inputs.data_ptr<int32_t>(), supervised.data_ptr<bool>(),
                                                   cu_seqlens.data_ptr<int32_t>(), drop.data_ptr<bool>(), m, k,
                                                   static_cast<int>(context_width), seed);
  else
    goldfish_kernel<int64_t><<<grid, 256, 0, st>>>(inputs.data_ptr<int64_t>(), supervised.data_ptr<bool>(),
                                                   cu_seqlens.data_ptr<int32_t>(), drop.data_ptr<bool>(), m, k,
                                                   static_cast<int>(context_width), seed);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return drop;
}
