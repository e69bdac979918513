// Cross-entropy over bf16 logits rows with fp32 math (forward: loss, lse, argmax-correct;
// backward: in-place g * (softmax - onehot)).  One CTA per row; each thread streams 16-byte
// vectors and keeps an online (max, sum-exp) pair plus a first-index argmax.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

using namespace mimir;

namespace {

constexpr int kThreads = 512;
constexpr float kLog2e = 1.4426950408889634f;

struct Stats {
  float m;    // running max (natural units)
  float s;    // sum exp(x - m)
  float bv;   // best value
  int bi;     // best index (first occurrence)
};

__device__ __forceinline__ Stats combine(Stats a, Stats b) {
  Stats r;
  r.m = fmaxf(a.m, b.m);
  r.s = (a.m == -INFINITY ? 0.f : a.s * exp2f((a.m - r.m) * kLog2e)) +
        (b.m == -INFINITY ? 0.f : b.s * exp2f((b.m - r.m) * kLog2e));
  if (b.bv > a.bv || (b.bv == a.bv && b.bi < a.bi)) {
    r.bv = b.bv;
    r.bi = b.bi;
  } else {
    r.bv = a.bv;
    r.bi = a.bi;
  }
  return r;
}

__global__ void __launch_bounds__(kThreads) ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits,
                                                          const int64_t* __restrict__ labels, int64_t V,
                                                          float* __restrict__ loss, float* __restrict__ lse_out,
                                                          bool* __restrict__ correct) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * V;
  Stats st{-INFINITY, 0.f, -INFINITY, INT_MAX};
  const int64_t nvec = V / 8;
  for (int64_t v = threadIdx.x; v < nvec; v += kThreads) {
    uint4 u = *reinterpret_cast<const uint4*>(x + v * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
    float lm = f[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) lm = fmaxf(lm, f[i]);
    const float nm = fmaxf(st.m, lm);
    float add = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) add += exp2f((f[i] - nm) * kLog2e);
    st.s = (st.m == -INFINITY ? 0.f : st.s * exp2f((st.m - nm) * kLog2e)) + add;
    st.m = nm;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (f[i] > st.bv) {  // strictly greater keeps the first index within this thread's sweep
        st.bv = f[i];
        st.bi = (int)(v * 8 + i);
      }
    }
  }
  // tail (V not a multiple of 8)
  for (int64_t i = nvec * 8 + threadIdx.x; i < V; i += kThreads) {
    const float f = __bfloat162float(x[i]);
    Stats one{f, 1.f, f, (int)i};
    st = combine(st, one);
  }
  // warp then block combine
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Stats other;
    other.m = __shfl_xor_sync(0xffffffff, st.m, o);
    other.s = __shfl_xor_sync(0xffffffff, st.s, o);
    other.bv = __shfl_xor_sync(0xffffffff, st.bv, o);
    other.bi = __shfl_xor_sync(0xffffffff, st.bi, o);
    st = combine(st, other);
  }
  __shared__ Stats part[kThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = st;
  __syncthreads();
  if (warp == 0) {
    st = lane < kThreads / 32 ? part[lane] : Stats{-INFINITY, 0.f, -INFINITY, INT_MAX};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Stats other;
      other.m = __shfl_xor_sync(0xffffffff, st.m, o);
      other.s = __shfl_xor_sync(0xffffffff, st.s, o);
      other.bv = __shfl_xor_sync(0xffffffff, st.bv, o);
      other.bi = __shfl_xor_sync(0xffffffff, st.bi, o);
      st = combine(st, other);
    }
    if (lane == 0) {
      const float lse = st.m + logf(st.s);
      const int64_t lab = labels[row];
      lse_out[row] = lse;
      if (lab >= 0 && lab < V) {
        loss[row] = lse - __bfloat162float(x[lab]);
      } else {
        loss[row] = 0.f;
      }
      correct[row] = (lab == (int64_t)st.bi);
    }
  }
}

__global__ void __launch_bounds__(kThreads) ce_bwd_kernel(__nv_bfloat16* __restrict__ logits,
                                                          const float* __restrict__ lse_in,
                                                          const int64_t* __restrict__ labels, int64_t V,
                                                          const float* __restrict__ gscale) {
  const int64_t row = blockIdx.x;
  __nv_bfloat16* x = logits + row * V;
  const int64_t lab = labels[row];
  const bool active = lab >= 0 && lab < V;
  const float lse = lse_in[row];
  const float g = gscale[0];
  const int64_t nvec = V / 8;
  for (int64_t v = threadIdx.x; v < nvec; v += kThreads) {
    uint4 u = *reinterpret_cast<const uint4*>(x + v * 8);
    uint4 out;
    uint32_t* w = reinterpret_cast<uint32_t*>(&out);
    if (active) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 t = __bfloat1622float2(h[i]);
        const int64_t c0 = v * 8 + 2 * i;
        float a = exp2f((t.x - lse) * kLog2e) - (c0 == lab ? 1.f : 0.f);
        float b = exp2f((t.y - lse) * kLog2e) - (c0 + 1 == lab ? 1.f : 0.f);
        w[i] = pack_bf16x2(a * g, b * g);
      }
    } else {
      out = make_uint4(0, 0, 0, 0);
    }
    *reinterpret_cast<uint4*>(x + v * 8) = out;
  }
  for (int64_t i = nvec * 8 + threadIdx.x; i < V; i += kThreads) {
    const float t = __bfloat162float(x[i]);
    const float d = active ? (exp2f((t - lse) * kLog2e) - (i == lab ? 1.f : 0.f)) * g : 0.f;
    x[i] = __float2bfloat16(d);
  }
}

}  // namespace

std::vector<at::Tensor> ce_fwd(at::Tensor logits, at::Tensor labels) {
  TORCH_CHECK(logits.is_cuda() && logits.is_contiguous() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2);
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() == logits.size(0));
  c10::cuda::CUDAGuard guard(logits.device());
  const int64_t N = logits.size(0), V = logits.size(1);
  auto loss = at::empty({N}, logits.options().dtype(at::kFloat));
  auto lse = at::empty({N}, logits.options().dtype(at::kFloat));
  auto correct = at::empty({N}, logits.options().dtype(at::kBool));
  if (N == 0) return {loss, lse, correct};
  TORCH_CHECK(V % 8 == 0 || true);
  ce_fwd_kernel<<<N, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), labels.data_ptr<int64_t>(), V, loss.data_ptr<float>(),
      lse.data_ptr<float>(), correct.data_ptr<bool>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {loss, lse, correct};
}

void ce_bwd_inplace(at::Tensor logits, at::Tensor lse, at::Tensor labels, at::Tensor gscale) {
  TORCH_CHECK(logits.is_cuda() && logits.is_contiguous() && logits.scalar_type() == at::kBFloat16);
  TORCH_CHECK(gscale.scalar_type() == at::kFloat && gscale.numel() == 1 && gscale.is_cuda());
  c10::cuda::CUDAGuard guard(logits.device());
  const int64_t N = logits.size(0), V = logits.size(1);
  if (N == 0) return;
  ce_bwd_kernel<<<N, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), lse.data_ptr<float>(), labels.data_ptr<int64_t>(), V,
      gscale.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
