// Scaled token embedding: out[t, :] = scale * E[ids[t], :] and its gradient
//   dE[v, :] += scale * sum_{t : ids[t] = v} dout[t, :].
//
// Forward: one warp per token row, 16-byte vector loads and stores, the scale applied in fp32 and
// rounded once (what `scale * F.embedding(ids, E)` computes for bf16 and fp32).
//
// Backward without atomics, deterministic: the caller passes the token ids sorted stably (so the
// positions of one id are in increasing order).  One warp per sorted position; the warp that
// starts a run of equal ids sums the run's dout rows in fp32, in position order, and adds
// scale * sum to the gradient row once (read-modify-write in the gradient's dtype).  Every other
// warp exits.  Reference: `src/mimir/model/layers.py:103-104` (ScaledEmbeddingInit.forward).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

namespace {

template <typename T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {  // 8 bf16 = 16 bytes
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float* v) {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  __device__ static void store(__nv_bfloat16* p, const float* v) {
    uint4 w;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = w;
  }
};
template <>
struct Vec8<float> {  // 4 fp32 = 16 bytes
  static constexpr int N = 4;
  __device__ static void load(const float* p, float* v) {
    const float4 w = *reinterpret_cast<const float4*>(p);
    v[0] = w.x, v[1] = w.y, v[2] = w.z, v[3] = w.w;
  }
  __device__ static void store(float* p, const float* v) { *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]); }
};

template <typename TW, typename TI>
__global__ void embed_fwd_kernel(const TI* __restrict__ ids, const TW* __restrict__ weight, TW* __restrict__ out,
                                 int64_t tokens, int d, int64_t vocab, float scale, int* bad) {
  constexpr int N = Vec8<TW>::N;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t t = warp; t < tokens; t += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t id = static_cast<int64_t>(ids[t]);
    const bool ok = id >= 0 && id < vocab;
    if (!ok && lane == 0) atomicExch(bad, 1);
    const TW* src = weight + (ok ? id : 0) * d;
    TW* dst = out + t * d;
    for (int c = lane * N; c < d; c += 32 * N) {
      float v[N];
      Vec8<TW>::load(src + c, v);
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = ok ? v[i] * scale : 0.f;
      Vec8<TW>::store(dst + c, v);
    }
  }
}

template <typename TD, typename TG>
__global__ void embed_bwd_kernel(const TD* __restrict__ dout, const int64_t* __restrict__ sorted_ids,
                                 const int64_t* __restrict__ order, TG* __restrict__ grad, int64_t tokens, int d,
                                 int64_t vocab, float scale) {
  constexpr int N = 8;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t i = warp; i < tokens; i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t id = sorted_ids[i];
    if ((i > 0 && sorted_ids[i - 1] == id) || id < 0 || id >= vocab) continue;  // not a run head
    int64_t end = i + 1;
    while (end < tokens && sorted_ids[end] == id) ++end;
    TG* row = grad + id * d;
    for (int c = lane * N; c < d; c += 32 * N) {
      float acc[N] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int64_t k = i; k < end; ++k) {  // positions in increasing order (stable sort)
        const TD* src = dout + order[k] * d + c;
        float v[N];
        Vec8<TD>::load(src, v);
        if constexpr (Vec8<TD>::N == 4) Vec8<TD>::load(src + 4, v + 4);
#pragma unroll
        for (int e = 0; e < N; ++e) acc[e] += v[e];
      }
      float g[N];
      Vec8<TG>::load(row + c, g);
      if constexpr (Vec8<TG>::N == 4) Vec8<TG>::load(row + c + 4, g + 4);
#pragma unroll
      for (int e = 0; e < N; ++e) g[e] += scale * acc[e];
      Vec8<TG>::store(row + c, g);
      if constexpr (Vec8<TG>::N == 4) Vec8<TG>::store(row + c + 4, g + 4);
    }
  }
}

int* bad_flag(const at::Device& dev) {
  static at::Tensor flags[64];
  const int i = dev.index();
  if (!flags[i].defined()) flags[i] = at::zeros({1}, at::TensorOptions().device(dev).dtype(at::kInt));
  return flags[i].data_ptr<int>();
}

int grid_warps(int64_t rows) {
  const int64_t blocks = (rows * 32 + 255) / 256;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, 148 * 16)));
}

}  // namespace

// out = scale * weight[ids]; ids int32/int64 of any shape, weight [V, d] bf16 or fp32 (d % 8 == 0).
at::Tensor embed_fwd(at::Tensor ids, at::Tensor weight, double scale) {
  TORCH_CHECK(ids.is_cuda() && weight.is_cuda() && weight.dim() == 2 && weight.is_contiguous(),
              "ids and a contiguous [V, d] weight on the GPU");
  TORCH_CHECK(ids.scalar_type() == at::kInt || ids.scalar_type() == at::kLong, "ids: int32 or int64");
  TORCH_CHECK(weight.scalar_type() == at::kBFloat16 || weight.scalar_type() == at::kFloat, "weight: bf16 or fp32");
  const int64_t d = weight.size(1), V = weight.size(0);
  TORCH_CHECK(d % 8 == 0, "embedding width must be a multiple of 8");
  const c10::cuda::CUDAGuard guard(weight.device());
  auto flat = ids.contiguous().view(-1);
  auto sizes = ids.sizes().vec();
  sizes.push_back(d);
  at::Tensor out = at::empty(sizes, weight.options());
  const int64_t T = flat.numel();
  if (T == 0) return out;
  auto st = at::cuda::getCurrentCUDAStream();
  int* bad = bad_flag(weight.device());
  const float s = static_cast<float>(scale);
#define MIMIR_EMBED_FWD(TW, TI)                                                                                   \
  embed_fwd_kernel<TW, TI><<<grid_warps(T), 256, 0, st>>>(flat.data_ptr<TI>(),                                   \
                                                          reinterpret_cast<const TW*>(weight.data_ptr()),        \
                                                          reinterpret_cast<TW*>(out.data_ptr()), T, (int)d, V, s, bad)
  if (weight.scalar_type() == at::kBFloat16) {
    if (flat.scalar_type() == at::kInt) MIMIR_EMBED_FWD(__nv_bfloat16, int32_t);
    else MIMIR_EMBED_FWD(__nv_bfloat16, int64_t);
  } else {
    if (flat.scalar_type() == at::kInt) MIMIR_EMBED_FWD(float, int32_t);
    else MIMIR_EMBED_FWD(float, int64_t);
  }
#undef MIMIR_EMBED_FWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// grad[v] += scale * sum of dout rows whose id is v.  sorted_ids / order: the stable sort of the
// flattened ids (int64) and the original positions; dout [T, d]; grad [V, d] (bf16 or fp32).
void embed_bwd(at::Tensor dout, at::Tensor sorted_ids, at::Tensor order, at::Tensor grad, double scale) {
  TORCH_CHECK(dout.is_cuda() && grad.is_cuda() && dout.is_contiguous() && grad.is_contiguous() && grad.dim() == 2,
              "contiguous dout and [V, d] grad on the GPU");
  TORCH_CHECK(sorted_ids.scalar_type() == at::kLong && order.scalar_type() == at::kLong && sorted_ids.is_contiguous() &&
                  order.is_contiguous() && sorted_ids.numel() == order.numel(),
              "sorted ids and positions: int64, one per token");
  const int64_t d = grad.size(1), V = grad.size(0), T = sorted_ids.numel();
  TORCH_CHECK(d % 8 == 0 && dout.numel() == T * d, "dout must be [tokens, d] with d % 8 == 0");
  const c10::cuda::CUDAGuard guard(grad.device());
  if (T == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  const float s = static_cast<float>(scale);
#define MIMIR_EMBED_BWD(TD, TG)                                                                          \
  embed_bwd_kernel<TD, TG><<<grid_warps(T), 256, 0, st>>>(                                              \
      reinterpret_cast<const TD*>(dout.data_ptr()), sorted_ids.data_ptr<int64_t>(), order.data_ptr<int64_t>(), \
      reinterpret_cast<TG*>(grad.data_ptr()), T, (int)d, V, s)
  const bool db = dout.scalar_type() == at::kBFloat16, gb = grad.scalar_type() == at::kBFloat16;
  TORCH_CHECK((db || dout.scalar_type() == at::kFloat) && (gb || grad.scalar_type() == at::kFloat),
              "dout and grad: bf16 or fp32");
  if (db && gb) MIMIR_EMBED_BWD(__nv_bfloat16, __nv_bfloat16);
  else if (db) MIMIR_EMBED_BWD(__nv_bfloat16, float);
  else if (gb) MIMIR_EMBED_BWD(float, __nv_bfloat16);
  else MIMIR_EMBED_BWD(float, float);
#undef MIMIR_EMBED_BWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// 1 if a forward saw an id outside [0, V) since the last read (its row was written as zeros).
int64_t embed_status(int64_t device) {
  int* flag = bad_flag(at::Device(at::kCUDA, static_cast<c10::DeviceIndex>(device)));
  int host = 0;
  C10_CUDA_CHECK(cudaMemcpy(&host, flag, sizeof(int), cudaMemcpyDeviceToHost));
  if (host) C10_CUDA_CHECK(cudaMemset(flag, 0, sizeof(int)));
  return host;
}
