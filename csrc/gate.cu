// Invocation-gate epilogue: out = inj * (1 + alpha * tanh(pre + bias)), fused, with its backward.
//
// `pre` is the gate projection W [hidden; injection] computed by the dense GEMM; this kernel adds
// the bias, applies tanh and the gate in fp32 and rounds once.  One thread per (token tile,
// channel); the backward writes d pre and d inj and a per-tile partial of d bias ([tiles, C],
// summed by the caller in tile order).  alpha (a model buffer) is read on the device.
//
//   t = tanh(pre + bias);  d inj = dout (1 + alpha t);  d pre = dout inj alpha (1 - t^2)
//
// Reference: `src/mimir/model/mimir2.py:135-141` (invocation gate).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

namespace {

constexpr int kThreads = 256;
constexpr int kTileT = 32;

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  if constexpr (std::is_same_v<T, float>) return *p;
  else return __bfloat162float(*p);
}
template <typename T>
__device__ __forceinline__ void stf(T* p, float v) {
  if constexpr (std::is_same_v<T, float>) *p = v;
  else *p = __float2bfloat16(v);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) gate_fwd_kernel(const T* __restrict__ pre, const T* __restrict__ inj,
                                                            const float* __restrict__ bias,
                                                            const float* __restrict__ alpha, T* __restrict__ out,
                                                            int64_t rows, int C) {
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= C) return;
  const float a = *alpha, b = bias[c];
  const int64_t end = min((int64_t)(blockIdx.y + 1) * kTileT, rows);
  for (int64_t t = (int64_t)blockIdx.y * kTileT; t < end; ++t) {
    const int64_t i = t * C + c;
    stf(out + i, ldf(inj + i) * (1.f + a * tanhf(ldf(pre + i) + b)));
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) gate_bwd_kernel(const T* __restrict__ dout, const T* __restrict__ pre,
                                                            const T* __restrict__ inj, const float* __restrict__ bias,
                                                            const float* __restrict__ alpha, T* __restrict__ dpre,
                                                            T* __restrict__ dinj, float* __restrict__ dbias,
                                                            int64_t rows, int C) {
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= C) return;
  const float a = *alpha, b = bias[c];
  float db = 0.f;
  const int64_t end = min((int64_t)(blockIdx.y + 1) * kTileT, rows);
  for (int64_t t = (int64_t)blockIdx.y * kTileT; t < end; ++t) {
    const int64_t i = t * C + c;
    const float th = tanhf(ldf(pre + i) + b), g = ldf(dout + i);
    const float dp = g * ldf(inj + i) * a * (1.f - th * th);
    stf(dinj + i, g * (1.f + a * th));
    stf(dpre + i, dp);
    db += dp;
  }
  dbias[(int64_t)blockIdx.y * C + c] = db;
}

void check(const at::Tensor& pre, const at::Tensor& inj, const at::Tensor& bias, const at::Tensor& alpha) {
  TORCH_CHECK(pre.is_cuda() && pre.is_contiguous() && pre.dim() == 2, "pre: contiguous [rows, C] CUDA tensor");
  TORCH_CHECK(pre.scalar_type() == at::kBFloat16 || pre.scalar_type() == at::kFloat, "pre: bf16 or fp32");
  TORCH_CHECK(inj.sizes() == pre.sizes() && inj.scalar_type() == pre.scalar_type() && inj.is_contiguous(),
              "injection: same shape and dtype as pre");
  TORCH_CHECK(bias.scalar_type() == at::kFloat && bias.is_contiguous() && bias.numel() == pre.size(1), "bias: fp32 [C]");
  TORCH_CHECK(alpha.scalar_type() == at::kFloat && alpha.numel() == 1 && alpha.is_cuda(), "alpha: fp32 device scalar");
}

dim3 grid(int64_t rows, int64_t C) {
  return dim3((unsigned)((C + kThreads - 1) / kThreads), (unsigned)((rows + kTileT - 1) / kTileT));
}

}  // namespace

at::Tensor invocation_gate_fwd(at::Tensor pre, at::Tensor inj, at::Tensor bias, at::Tensor alpha) {
  check(pre, inj, bias, alpha);
  const c10::cuda::CUDAGuard guard(pre.device());
  auto out = at::empty_like(pre);
  const int64_t rows = pre.size(0), C = pre.size(1);
  if (rows == 0) return out;
  auto st = at::cuda::getCurrentCUDAStream();
  if (pre.scalar_type() == at::kFloat)
    gate_fwd_kernel<float><<<grid(rows, C), kThreads, 0, st>>>(pre.data_ptr<float>(), inj.data_ptr<float>(),
                                                              bias.data_ptr<float>(), alpha.data_ptr<float>(),
                                                              out.data_ptr<float>(), rows, (int)C);
  else
    gate_fwd_kernel<__nv_bfloat16><<<grid(rows, C), kThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(pre.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(inj.data_ptr()),
        bias.data_ptr<float>(), alpha.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows,
        (int)C);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Returns (d pre, d injection, d bias fp32 [C]).
std::vector<at::Tensor> invocation_gate_bwd(at::Tensor dout, at::Tensor pre, at::Tensor inj, at::Tensor bias,
                                            at::Tensor alpha) {
  check(pre, inj, bias, alpha);
  TORCH_CHECK(dout.sizes() == pre.sizes() && dout.scalar_type() == pre.scalar_type() && dout.is_contiguous(),
              "dout: same shape and dtype as pre");
  const c10::cuda::CUDAGuard guard(pre.device());
  const int64_t rows = pre.size(0), C = pre.size(1);
  auto dpre = at::empty_like(pre), dinj = at::empty_like(pre);
  const dim3 g = grid(rows, C);
  auto partial = at::zeros({(int64_t)g.y, C}, pre.options().dtype(at::kFloat));
  if (rows > 0) {
    auto st = at::cuda::getCurrentCUDAStream();
    if (pre.scalar_type() == at::kFloat)
      gate_bwd_kernel<float><<<g, kThreads, 0, st>>>(dout.data_ptr<float>(), pre.data_ptr<float>(),
                                                     inj.data_ptr<float>(), bias.data_ptr<float>(),
                                                     alpha.data_ptr<float>(), dpre.data_ptr<float>(),
                                                     dinj.data_ptr<float>(), partial.data_ptr<float>(), rows, (int)C);
    else
      gate_bwd_kernel<__nv_bfloat16><<<g, kThreads, 0, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(pre.data_ptr()),
          reinterpret_cast<const __nv_bfloat16*>(inj.data_ptr()), bias.data_ptr<float>(), alpha.data_ptr<float>(),
          reinterpret_cast<__nv_bfloat16*>(dpre.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dinj.data_ptr()),
          partial.data_ptr<float>(), rows, (int)C);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {dpre, dinj, partial.sum(0)};
}
