// Fused multi-tensor AdamATan2 step (decoupled weight decay, atan2 update, optional first
// moment, optional EMA).  One launch per (param dtype, ema dtype) bucket: a small device
// table describes every tensor and the CTA range that owns it; each CTA finds its tensor
// by binary search and streams CHUNK elements with fp32 math.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kChunk = kThreads * 4 * 8;  // elements per CTA (8 iterations of 4-wide vectors)

struct TensorEntry {
  uint64_t p, g, m, v, e;
  int64_t n;
  int64_t block_start;
  float lr, bc1, bc2_sqrt;
  int vec;  // all slot pointers 16-byte aligned: use 4-wide vector accesses
};

template <typename T>
struct V4;
template <>
struct V4<float> {
  __device__ static void load(const float* p, float (&f)[4]) {
    const float4 u = *reinterpret_cast<const float4*>(p);
    f[0] = u.x, f[1] = u.y, f[2] = u.z, f[3] = u.w;
  }
  __device__ static void store(float* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};
template <>
struct V4<__nv_bfloat16> {
  __device__ static void load(const __nv_bfloat16* p, float (&f)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    f[0] = a.x, f[1] = a.y, f[2] = b.x, f[3] = b.y;
  }
  __device__ static void store(__nv_bfloat16* p, const float (&f)[4]) {
    *reinterpret_cast<uint2*>(p) = make_uint2(mimir::pack_bf16x2(f[0], f[1]), mimir::pack_bf16x2(f[2], f[3]));
  }
};

template <typename T>
__device__ __forceinline__ float ld(const T* p) {
  return static_cast<float>(*p);
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename T>
__device__ __forceinline__ void st(T* p, float v) {
  *p = static_cast<T>(v);
}
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16(v);
}

template <typename P, typename E>
__global__ void __launch_bounds__(kThreads) adam_atan2_kernel(const TensorEntry* __restrict__ table, int ntensors,
                                                              float b1, float b2, float wd, float ema_decay) {
  // binary search: last entry with block_start <= blockIdx.x
  int lo = 0, hi = ntensors - 1;
  const int64_t b = blockIdx.x;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (table[mid].block_start <= b) lo = mid;
    else hi = mid - 1;
  }
  const TensorEntry t = table[lo];
  P* p = reinterpret_cast<P*>(t.p);
  const P* g = reinterpret_cast<const P*>(t.g);
  P* m = reinterpret_cast<P*>(t.m);
  P* v = reinterpret_cast<P*>(t.v);
  E* e = reinterpret_cast<E*>(t.e);
  const int64_t start = (b - t.block_start) * kChunk;
  const int64_t end = min(start + (int64_t)kChunk, t.n);
  const float decay = 1.f - t.lr * wd;
  const float step_size = t.lr / t.bc1;
  if (t.vec) {
    // 4-wide path: same arithmetic as the scalar loop below, one 16-byte (fp32) access per slot.
    for (int64_t i = start + 4 * threadIdx.x; i + 3 < end; i += 4 * kThreads) {
      float gi[4], pi[4], vi[4], mi[4], ei[4];
      V4<P>::load(g + i, gi);
      V4<P>::load(p + i, pi);
      V4<P>::load(v + i, vi);
      if (m != nullptr) V4<P>::load(m + i, mi);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (wd != 0.f) pi[k] = pi[k] * decay;
        vi[k] = b2 * vi[k] + (1.f - b2) * gi[k] * gi[k];
        const float denom = sqrtf(vi[k]) / t.bc2_sqrt;
        if (m != nullptr) {
          mi[k] = mi[k] + (1.f - b1) * (gi[k] - mi[k]);
          pi[k] = pi[k] - step_size * atan2f(mi[k], denom);
        } else {
          pi[k] = pi[k] - t.lr * atan2f(gi[k], denom);
        }
      }
      V4<P>::store(v + i, vi);
      V4<P>::store(p + i, pi);
      if (m != nullptr) V4<P>::store(m + i, mi);
      if (e != nullptr) {
        float stored[4];
        V4<P>::load(p + i, stored);  // EMA follows the stored (rounded) parameter
        V4<E>::load(e + i, ei);
#pragma unroll
        for (int k = 0; k < 4; ++k) ei[k] = ei[k] + (1.f - ema_decay) * (stored[k] - ei[k]);
        V4<E>::store(e + i, ei);
      }
    }
    return;  // vec tensors have n % 4 == 0, so the chunk is fully covered
  }
  for (int64_t i = start + threadIdx.x; i < end; i += kThreads) {
    const float gi = ld(g + i);
    float pi = ld(p + i);
    if (wd != 0.f) pi = pi * decay;
    float vi = ld(v + i);
    vi = b2 * vi + (1.f - b2) * gi * gi;
    const float denom = sqrtf(vi) / t.bc2_sqrt;
    if (m != nullptr) {
      float mi = ld(m + i);
      mi = mi + (1.f - b1) * (gi - mi);
      st(m + i, mi);
      pi = pi - step_size * atan2f(mi, denom);
    } else {
      pi = pi - t.lr * atan2f(gi, denom);
    }
    st(v + i, vi);
    st(p + i, pi);
    if (e != nullptr) {
      const float ei = ld(e + i);
      // EMA reads the stored (rounded) parameter, as the reference lerps toward p.
      st(e + i, ei + (1.f - ema_decay) * (ld(p + i) - ei));
    }
  }
}

}  // namespace

void adam_atan2_multi(std::vector<at::Tensor> params, std::vector<at::Tensor> grads,
                      c10::optional<std::vector<at::Tensor>> exp_avgs, std::vector<at::Tensor> exp_avg_sqs,
                      c10::optional<std::vector<at::Tensor>> emas, std::vector<double> lrs, std::vector<double> bc1,
                      std::vector<double> bc2_sqrt, double beta1, double beta2, double weight_decay, double ema_decay) {
  const int n = (int)params.size();
  if (n == 0) return;
  TORCH_CHECK(grads.size() == (size_t)n && exp_avg_sqs.size() == (size_t)n && lrs.size() == (size_t)n);
  const bool has_m = exp_avgs.has_value();
  const bool has_e = emas.has_value();
  c10::cuda::CUDAGuard guard(params[0].device());
  auto host = at::empty({(int64_t)(n * sizeof(TensorEntry))}, at::TensorOptions().dtype(at::kByte).pinned_memory(true));
  auto* tab = reinterpret_cast<TensorEntry*>(host.data_ptr());
  int64_t blocks = 0;
  const auto pdt = params[0].scalar_type();
  const auto edt = has_e ? (*emas)[0].scalar_type() : pdt;
  for (int i = 0; i < n; ++i) {
    const auto& p = params[i];
    TORCH_CHECK(p.is_cuda() && p.is_contiguous() && p.scalar_type() == pdt, "adam: params must share dtype");
    TORCH_CHECK(grads[i].is_contiguous() && grads[i].scalar_type() == pdt && grads[i].numel() == p.numel(),
                "adam: grad must match param dtype/shape");
    TORCH_CHECK(exp_avg_sqs[i].is_contiguous() && exp_avg_sqs[i].scalar_type() == pdt);
    tab[i].p = reinterpret_cast<uint64_t>(p.data_ptr());
    tab[i].g = reinterpret_cast<uint64_t>(grads[i].data_ptr());
    tab[i].v = reinterpret_cast<uint64_t>(exp_avg_sqs[i].data_ptr());
    if (has_m) {
      TORCH_CHECK((*exp_avgs)[i].is_contiguous() && (*exp_avgs)[i].scalar_type() == pdt);
      tab[i].m = reinterpret_cast<uint64_t>((*exp_avgs)[i].data_ptr());
    } else {
      tab[i].m = 0;
    }
    if (has_e) {
      TORCH_CHECK((*emas)[i].is_contiguous() && (*emas)[i].scalar_type() == edt);
      tab[i].e = reinterpret_cast<uint64_t>((*emas)[i].data_ptr());
    } else {
      tab[i].e = 0;
    }
    tab[i].n = p.numel();
    tab[i].block_start = blocks;
    tab[i].lr = (float)lrs[i];
    tab[i].bc1 = (float)bc1[i];
    tab[i].bc2_sqrt = (float)bc2_sqrt[i];
    auto al = [](uint64_t ptr) { return ptr % 16 == 0; };
    tab[i].vec = (p.numel() % 4 == 0) && al(tab[i].p) && al(tab[i].g) && al(tab[i].v) && (tab[i].m == 0 || al(tab[i].m)) &&
                 (tab[i].e == 0 || al(tab[i].e));
    blocks += (p.numel() + kChunk - 1) / kChunk;
  }
  if (blocks == 0) return;
  auto dev = host.to(params[0].device(), /*non_blocking=*/true);
  auto stream = at::cuda::getCurrentCUDAStream();
  const auto* dtab = reinterpret_cast<const TensorEntry*>(dev.data_ptr());
  const float b1 = (float)beta1, b2 = (float)beta2, wd = (float)weight_decay, ed = (float)ema_decay;
  TORCH_CHECK(blocks < (1ll << 31));
  if (pdt == at::kFloat && edt == at::kFloat) {
    adam_atan2_kernel<float, float><<<blocks, kThreads, 0, stream>>>(dtab, n, b1, b2, wd, ed);
  } else if (pdt == at::kBFloat16 && edt == at::kFloat) {
    adam_atan2_kernel<__nv_bfloat16, float><<<blocks, kThreads, 0, stream>>>(dtab, n, b1, b2, wd, ed);
  } else if (pdt == at::kBFloat16 && edt == at::kBFloat16) {
    adam_atan2_kernel<__nv_bfloat16, __nv_bfloat16><<<blocks, kThreads, 0, stream>>>(dtab, n, b1, b2, wd, ed);
  } else {
    TORCH_CHECK(false, "adam_atan2_multi: unsupported dtype combination");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  // The pinned staging block is not reused before the async copy completes: the caching
  // host allocator records an event for it inside `to(..., non_blocking=true)`.
}
