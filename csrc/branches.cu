// Residual-branch mixes of a branched stack, fused (forward and backward).
//
// Streams s[t, b, c] (B <= 8 branches, channel c contiguous; any token/branch strides, so a
// broadcast view of one stream is read in place).  Per channel the weights over the branch axis
// are w_b = softmax_b(alpha * (L[b, c] + tanh(s[t, b, c]) * G[b, c]))  (G optional), computed in
// fp32 in registers, one thread per (token, channel):
//
//   read:   x[t, c]      = sum_b w_b s[t, b, c]
//   write:  o[t, b, c]   = s[t, b, c] + B * w_b * u[t, c]
//
// Backward (with z_b the logits and dz_b = w_b (g_b - sum_k w_k g_k), g_b = dLoss/dw_b):
//   read:  g_b = dx s_b,      ds_b = w_b dx + alpha dz_b G_b (1 - tanh^2 s_b)
//   write: g_b = B u do_b,    ds_b = do_b + alpha dz_b G_b (1 - tanh^2 s_b),  du = B sum_b w_b do_b
//   dL_b = alpha sum_t dz_b,  dG_b = alpha sum_t dz_b tanh(s_b)
// The parameter gradients are per-CTA partial sums over a tile of tokens ([tiles, B, C] fp32),
// summed by the caller in tile order (deterministic).  alpha is read from device memory (a model
// buffer), so no host synchronisation is needed.
//
// Reference: `src/mimir/model/residual_branches.py:27-40` (ResidualConnection.read / write).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

namespace {

constexpr int kMaxB = 8;
constexpr int kThreads = 256;  // channels per CTA
constexpr int kTileT = 32;     // tokens per CTA

template <typename T>
__device__ __forceinline__ float ld(const T* p) {
  if constexpr (std::is_same_v<T, float>) return *p;
  else return __bfloat162float(*p);
}
template <typename T>
__device__ __forceinline__ void st(T* p, float v) {
  if constexpr (std::is_same_v<T, float>) *p = v;
  else *p = __float2bfloat16(v);
}

struct Mix {
  const float* logits;  // [B, C]
  const float* gain;    // [B, C] or nullptr
  const float* alpha;   // device scalar
  int B, C;
  int64_t T, ts, bs;    // tokens, token stride and branch stride of the streams (elements)
};

__device__ __forceinline__ int64_t tile_end(const Mix& m) {
  const int64_t e = (blockIdx.y + 1) * (int64_t)kTileT;
  return e < m.T ? e : m.T;
}

// w[b] and tanh(s[b]) for one (token, channel).
template <typename TS>
__device__ __forceinline__ void weights(const Mix& m, const TS* s, int c, float a, float (&sv)[kMaxB],
                                        float (&th)[kMaxB], float (&w)[kMaxB]) {
  float mx = -INFINITY;
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) {
    if (b >= m.B) break;
    sv[b] = ld(s + b * m.bs);
    th[b] = m.gain != nullptr ? tanhf(sv[b]) : 0.f;
    float z = m.logits[b * m.C + c];
    if (m.gain != nullptr) z += th[b] * m.gain[b * m.C + c];
    w[b] = a * z;
    mx = fmaxf(mx, w[b]);
  }
  float sum = 0.f;
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) {
    if (b >= m.B) break;
    w[b] = __expf(w[b] - mx);
    sum += w[b];
  }
  const float inv = 1.f / sum;
#pragma unroll
  for (int b = 0; b < kMaxB; ++b)
    if (b < m.B) w[b] *= inv;
}

template <typename TS>
__global__ void __launch_bounds__(kThreads) read_fwd(Mix m, const TS* __restrict__ s, TS* __restrict__ x) {
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= m.C) return;
  const float a = *m.alpha;
  for (int64_t t = blockIdx.y * (int64_t)kTileT, e = tile_end(m); t < e; ++t) {
    float sv[kMaxB], th[kMaxB], w[kMaxB];
    weights(m, s + t * m.ts + c, c, a, sv, th, w);
    float acc = 0.f;
#pragma unroll
    for (int b = 0; b < kMaxB; ++b)
      if (b < m.B) acc += w[b] * sv[b];
    st(x + t * m.C + c, acc);
  }
}

template <typename TS>
__global__ void __launch_bounds__(kThreads) write_fwd(Mix m, const TS* __restrict__ s, const TS* __restrict__ u,
                                                      TS* __restrict__ o) {
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= m.C) return;
  const float a = *m.alpha;
  for (int64_t t = blockIdx.y * (int64_t)kTileT, e = tile_end(m); t < e; ++t) {
    float sv[kMaxB], th[kMaxB], w[kMaxB];
    weights(m, s + t * m.ts + c, c, a, sv, th, w);
    const float uv = ld(u + t * m.C + c);
#pragma unroll
    for (int b = 0; b < kMaxB; ++b)
      if (b < m.B) st(o + (t * m.B + b) * (int64_t)m.C + c, sv[b] + m.B * w[b] * uv);
  }
}

// kWrite = false: read backward (grad = dx [T, C]); true: write backward (grad = do [T, B, C]).
template <typename TS, bool kWrite>
__global__ void __launch_bounds__(kThreads) mix_bwd(Mix m, const TS* __restrict__ s, const TS* __restrict__ u,
                                                    const TS* __restrict__ grad, TS* __restrict__ ds,
                                                    TS* __restrict__ du, float* __restrict__ dlog,
                                                    float* __restrict__ dgain) {
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= m.C) return;
  const float a = *m.alpha;
  float pl[kMaxB], pg[kMaxB];
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) pl[b] = pg[b] = 0.f;
  for (int64_t t = blockIdx.y * (int64_t)kTileT, e = tile_end(m); t < e; ++t) {
    float sv[kMaxB], th[kMaxB], w[kMaxB], g[kMaxB], go[kMaxB];
    weights(m, s + t * m.ts + c, c, a, sv, th, w);
    float dot = 0.f, uv = 0.f, dx = 0.f;
    if constexpr (kWrite) uv = ld(u + t * m.C + c);
    else dx = ld(grad + t * m.C + c);
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      if (b >= m.B) break;
      if constexpr (kWrite) {
        go[b] = ld(grad + (t * m.B + b) * (int64_t)m.C + c);
        g[b] = m.B * uv * go[b];
      } else {
        g[b] = dx * sv[b];
      }
      dot += w[b] * g[b];
    }
    float dsum_u = 0.f;
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      if (b >= m.B) break;
      const float dz = w[b] * (g[b] - dot);
      pl[b] += dz;
      float dsb = kWrite ? go[b] : w[b] * dx;
      if (m.gain != nullptr) {
        pg[b] += dz * th[b];
        dsb += a * dz * m.gain[b * m.C + c] * (1.f - th[b] * th[b]);
      }
      st(ds + (t * m.B + b) * (int64_t)m.C + c, dsb);
      if constexpr (kWrite) dsum_u += w[b] * go[b];
    }
    if constexpr (kWrite) st(du + t * m.C + c, m.B * dsum_u);
  }
  float* dl = dlog + (int64_t)blockIdx.y * m.B * m.C;
  float* dg = dgain != nullptr ? dgain + (int64_t)blockIdx.y * m.B * m.C : nullptr;
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) {
    if (b >= m.B) break;
    dl[b * m.C + c] = a * pl[b];
    if (dg != nullptr) dg[b * m.C + c] = a * pg[b];
  }
}

Mix make_mix(const at::Tensor& s, const at::Tensor& logits, const c10::optional<at::Tensor>& gain,
             const at::Tensor& alpha) {
  TORCH_CHECK(s.is_cuda() && s.dim() == 3 && s.stride(2) == 1, "streams: [T, B, C] CUDA tensor, channels contiguous");
  TORCH_CHECK(s.scalar_type() == at::kBFloat16 || s.scalar_type() == at::kFloat, "streams: bf16 or fp32");
  const int B = (int)s.size(1), C = (int)s.size(2);
  TORCH_CHECK(B >= 1 && B <= kMaxB, "1..", kMaxB, " branches");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous() && logits.size(0) == B &&
                  logits.size(1) == C, "logits: fp32 [B, C]");
  if (gain) TORCH_CHECK(gain->scalar_type() == at::kFloat && gain->is_contiguous() && gain->sizes() == logits.sizes(),
                        "gain: fp32 [B, C]");
  TORCH_CHECK(alpha.scalar_type() == at::kFloat && alpha.numel() == 1 && alpha.is_cuda(), "alpha: fp32 device scalar");
  Mix m{};
  m.logits = logits.data_ptr<float>();
  m.gain = gain ? gain->data_ptr<float>() : nullptr;
  m.alpha = alpha.data_ptr<float>();
  m.B = B;
  m.C = C;
  m.T = s.size(0);
  m.ts = s.stride(0);
  m.bs = s.stride(1);
  return m;
}

dim3 grid_for(const Mix& m) {
  return dim3((unsigned)((m.C + kThreads - 1) / kThreads), (unsigned)((m.T + kTileT - 1) / kTileT));
}

}  // namespace

#define MIMIR_BRANCH_DISPATCH(S, ...)                                   \
  if ((S).scalar_type() == at::kBFloat16) {                              \
    using TS = __nv_bfloat16;                                            \
    __VA_ARGS__;                                                         \
  } else {                                                               \
    using TS = float;                                                    \
    __VA_ARGS__;                                                         \
  }

at::Tensor branch_read(at::Tensor s, at::Tensor logits, c10::optional<at::Tensor> gain, at::Tensor alpha) {
  const c10::cuda::CUDAGuard guard(s.device());
  Mix m = make_mix(s, logits, gain, alpha);
  auto x = at::empty({m.T, (int64_t)m.C}, s.options());
  if (m.T == 0) return x;
  auto st = at::cuda::getCurrentCUDAStream();
  MIMIR_BRANCH_DISPATCH(s, read_fwd<TS><<<grid_for(m), kThreads, 0, st>>>(
      m, reinterpret_cast<const TS*>(s.data_ptr()), reinterpret_cast<TS*>(x.data_ptr())));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return x;
}

at::Tensor branch_write(at::Tensor s, at::Tensor u, at::Tensor logits, c10::optional<at::Tensor> gain,
                        at::Tensor alpha) {
  const c10::cuda::CUDAGuard guard(s.device());
  Mix m = make_mix(s, logits, gain, alpha);
  TORCH_CHECK(u.scalar_type() == s.scalar_type() && u.is_contiguous() && u.numel() == m.T * m.C, "update: [T, C]");
  auto o = at::empty({m.T, (int64_t)m.B, (int64_t)m.C}, s.options());
  if (m.T == 0) return o;
  auto st = at::cuda::getCurrentCUDAStream();
  MIMIR_BRANCH_DISPATCH(s, write_fwd<TS><<<grid_for(m), kThreads, 0, st>>>(
      m, reinterpret_cast<const TS*>(s.data_ptr()), reinterpret_cast<const TS*>(u.data_ptr()),
      reinterpret_cast<TS*>(o.data_ptr())));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return o;
}

// Returns (d streams [T, B, C], d update [T, C] or empty, d logits [B, C], d gain [B, C] or empty).
std::vector<at::Tensor> branch_mix_bwd(at::Tensor grad, at::Tensor s, c10::optional<at::Tensor> u, at::Tensor logits,
                                       c10::optional<at::Tensor> gain, at::Tensor alpha) {
  const c10::cuda::CUDAGuard guard(s.device());
  Mix m = make_mix(s, logits, gain, alpha);
  const bool write = u.has_value();
  TORCH_CHECK(grad.scalar_type() == s.scalar_type() && grad.is_contiguous() &&
                  grad.numel() == m.T * m.C * (write ? m.B : 1), "grad: contiguous, streams dtype");
  if (write) TORCH_CHECK(u->scalar_type() == s.scalar_type() && u->is_contiguous() && u->numel() == m.T * m.C,
                         "update: [T, C]");
  auto ds = at::empty({m.T, (int64_t)m.B, (int64_t)m.C}, s.options());
  auto du = write ? at::empty({m.T, (int64_t)m.C}, s.options()) : at::Tensor();
  const dim3 grid = grid_for(m);
  auto f32 = s.options().dtype(at::kFloat);
  auto dlog = at::zeros({(int64_t)grid.y, (int64_t)m.B, (int64_t)m.C}, f32);
  auto dgain = gain ? at::zeros({(int64_t)grid.y, (int64_t)m.B, (int64_t)m.C}, f32) : at::Tensor();
  if (m.T > 0) {
    auto st = at::cuda::getCurrentCUDAStream();
    float* dg = gain ? dgain.data_ptr<float>() : nullptr;
    if (write) {
      MIMIR_BRANCH_DISPATCH(s, mix_bwd<TS, true><<<grid, kThreads, 0, st>>>(
          m, reinterpret_cast<const TS*>(s.data_ptr()), reinterpret_cast<const TS*>(u->data_ptr()),
          reinterpret_cast<const TS*>(grad.data_ptr()), reinterpret_cast<TS*>(ds.data_ptr()),
          reinterpret_cast<TS*>(du.data_ptr()), dlog.data_ptr<float>(), dg));
    } else {
      MIMIR_BRANCH_DISPATCH(s, mix_bwd<TS, false><<<grid, kThreads, 0, st>>>(
          m, reinterpret_cast<const TS*>(s.data_ptr()), nullptr, reinterpret_cast<const TS*>(grad.data_ptr()),
          reinterpret_cast<TS*>(ds.data_ptr()), nullptr, dlog.data_ptr<float>(), dg));
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {ds, du, dlog.sum(0), gain ? dgain.sum(0) : at::Tensor()};
}
