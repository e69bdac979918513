// Memory-bound fused kernels: weightless RMSNorm (fwd/bwd), SwiGLU (fwd/bwd), RoPE on the
// packed [gate|Q|K|V] projection (fwd/bwd), the attention output-gate backward, and the
// attention "delta" row reduction.  All use 16-byte vector accesses and fp32 math.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "swiglu_math.cuh"

using namespace mimir;

namespace {

template <typename T>
struct Vec;  // 16 bytes of T
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&f)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  __device__ static void store(__nv_bfloat16* p, const float (&f)[8]) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = pack_bf16x2(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&f)[4]) {
    float4 u = *reinterpret_cast<const float4*>(p);
    f[0] = u.x, f[1] = u.y, f[2] = u.z, f[3] = u.w;
  }
  __device__ static void store(float* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  return static_cast<float>(v);
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// Block-wide sum for blockDim.x <= 1024 (multiple of 32).
__device__ float block_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = lane < nw ? scratch[lane] : 0.f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

// ------------------------------------------------------------------ RMSNorm
// One CTA per row; each thread caches VPT vectors of the row in registers.
template <typename T, int VPT>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                          float* __restrict__ rstd_out, int d, float eps) {
  constexpr int N = Vec<T>::N;
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * d;
  T* yr = y + row * d;
  float v[VPT][N];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * blockDim.x + threadIdx.x) * N;
    if (c < d) {
      Vec<T>::load(xr + c, v[i]);
#pragma unroll
      for (int j = 0; j < N; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = block_sum(ss, scratch);
  const float r = rsqrtf(ss / d + eps);
  if (threadIdx.x == 0) rstd_out[row] = r;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * blockDim.x + threadIdx.x) * N;
    if (c < d) {
      float o[N];
#pragma unroll
      for (int j = 0; j < N; ++j) o[j] = v[i][j] * r;
      Vec<T>::store(yr + c, o);
    }
  }
}

template <typename T, int VPT>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                          const float* __restrict__ rstd, T* __restrict__ dx, int d) {
  constexpr int N = Vec<T>::N;
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const float r = rstd[row];
  float xv[VPT][N], gv[VPT][N];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * blockDim.x + threadIdx.x) * N;
    if (c < d) {
      Vec<T>::load(x + row * d + c, xv[i]);
      Vec<T>::load(dy + row * d + c, gv[i]);
#pragma unroll
      for (int j = 0; j < N; ++j) dot += gv[i][j] * xv[i][j] * r;
    }
  }
  dot = block_sum(dot, scratch) / d;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * blockDim.x + threadIdx.x) * N;
    if (c < d) {
      float o[N];
#pragma unroll
      for (int j = 0; j < N; ++j) o[j] = r * (gv[i][j] - xv[i][j] * r * dot);
      Vec<T>::store(dx + row * d + c, o);
    }
  }
}

// h = x + delta (rounded to T, as the unfused residual add stores it); y = rmsnorm(h).
template <typename T, int VPT>
__global__ void __launch_bounds__(256) add_rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ delta,
                                                              T* __restrict__ h, T* __restrict__ y,
                                                              float* __restrict__ rstd_out, int d, float eps) {
  constexpr int N = Vec<T>::N;
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  float v[VPT][N];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * blockDim.x + threadIdx.x) * N;
    if (c < d) {
      float a[N];
      Vec<T>::load(x + row * d + c, v[i]);
      Vec<T>::load(delta + row * d + c, a);
#pragma unroll
      for (int j = 0; j < N; ++j) v[i][j] += a[j];
      Vec<T>::store(h + row * d + c, v[i]);
      Vec<T>::load(h + row * d + c, v[i]);  // the rounded sum, exactly what a separate add would store
#pragma unroll
      for (int j = 0; j < N; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = block_sum(ss, scratch);
  const float r = rsqrtf(ss / d + eps);
  if (threadIdx.x == 0) rstd_out[row] = r;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * blockDim.x + threadIdx.x) * N;
    if (c < d) {
      float o[N];
#pragma unroll
      for (int j = 0; j < N; ++j) o[j] = v[i][j] * r;
      Vec<T>::store(y + row * d + c, o);
    }
  }
}

// dx = rmsnorm_bwd(dy; x, rstd) + dres: the residual stream's own gradient joins in the same pass.
template <typename T, int VPT>
__global__ void __launch_bounds__(256) rmsnorm_bwd_res_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                              const float* __restrict__ rstd,
                                                              const T* __restrict__ dres, T* __restrict__ dx, int d) {
  constexpr int N = Vec<T>::N;
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const float r = rstd[row];
  float xv[VPT][N], gv[VPT][N];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * blockDim.x + threadIdx.x) * N;
    if (c < d) {
      Vec<T>::load(x + row * d + c, xv[i]);
      Vec<T>::load(dy + row * d + c, gv[i]);
#pragma unroll
      for (int j = 0; j < N; ++j) dot += gv[i][j] * xv[i][j] * r;
    }
  }
  dot = block_sum(dot, scratch) / d;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * blockDim.x + threadIdx.x) * N;
    if (c < d) {
      float o[N], rv[N];
      Vec<T>::load(dres + row * d + c, rv);
#pragma unroll
      for (int j = 0; j < N; ++j) o[j] = r * (gv[i][j] - xv[i][j] * r * dot) + rv[j];
      Vec<T>::store(dx + row * d + c, o);
    }
  }
}

// ------------------------------------------------------------------ SwiGLU
__device__ __forceinline__ float silu_f(float g) { return swiglu_silu(g); }

template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t rows, int f) {
  constexpr int N = Vec<T>::N;
  const int vecs = f / N;
  const int64_t total = rows * vecs;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vecs;
    const int c = (int)(i - r * vecs) * N;
    float g[N], u[N], o[N];
    Vec<T>::load(gu + r * 2 * f + c, g);
    Vec<T>::load(gu + r * 2 * f + f + c, u);
#pragma unroll
    for (int j = 0; j < N; ++j) o[j] = silu_f(g[j]) * u[j];
    Vec<T>::store(out + r * f + c, o);
  }
}

template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ dp, const T* __restrict__ gu, T* __restrict__ dgu,
                                  int64_t rows, int f) {
  constexpr int N = Vec<T>::N;
  const int vecs = f / N;
  const int64_t total = rows * vecs;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vecs;
    const int c = (int)(i - r * vecs) * N;
    float g[N], u[N], d[N], dg[N], du[N];
    Vec<T>::load(gu + r * 2 * f + c, g);
    Vec<T>::load(gu + r * 2 * f + f + c, u);
    Vec<T>::load(dp + r * f + c, d);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      swiglu_backward(d[j], g[j], u[j], dg[j], du[j]);
    }
    Vec<T>::store(dgu + r * 2 * f + c, dg);
    Vec<T>::store(dgu + r * 2 * f + f + c, du);
  }
}

// ------------------------------------------------------------------ RoPE on packed Q|K
// gqkv row layout: [gate H | q H | k KV | v KV] x 128.  Output qk row: [q H | k KV] x 128.
// One thread per (token, head, 8-wide chunk of the lower half).
template <typename TT>
__global__ void rope_qk_fwd_kernel(const __nv_bfloat16* __restrict__ gqkv, int64_t ld_in,
                                   __nv_bfloat16* __restrict__ qk, int64_t ld_out, const TT* __restrict__ cos_t,
                                   const TT* __restrict__ sin_t, const int* __restrict__ pos, int64_t T,
                                   int H, int heads /* H + KV */) {
  const int64_t total = T * heads * 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int chunk = (int)(i & 7);
    const int64_t th = i >> 3;
    const int h = (int)(th % heads);
    const int64_t t = th / heads;
    const int d0 = chunk * 8;
    const __nv_bfloat16* src = gqkv + t * ld_in + (int64_t)(H + h) * 128;
    __nv_bfloat16* dst = qk + t * ld_out + (int64_t)h * 128;
    const int64_t p = pos[t];
    const TT* c = cos_t + p * 128;
    const TT* s = sin_t + p * 128;
    float lo[8], hi[8], olo[8], ohi[8];
    Vec<__nv_bfloat16>::load(src + d0, lo);
    Vec<__nv_bfloat16>::load(src + 64 + d0, hi);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      olo[j] = lo[j] * to_f(c[d0 + j]) - hi[j] * to_f(s[d0 + j]);
      ohi[j] = hi[j] * to_f(c[64 + d0 + j]) + lo[j] * to_f(s[64 + d0 + j]);
    }
    Vec<__nv_bfloat16>::store(dst + d0, olo);
    Vec<__nv_bfloat16>::store(dst + 64 + d0, ohi);
  }
}

// Adjoint of the rotation: writes un-rotated dq/dk and copies dv into the packed gradient.
template <typename TQ, typename TK, typename TV, typename TT>
__global__ void rope_qk_bwd_kernel(const TQ* __restrict__ dq, const TK* __restrict__ dk, const TV* __restrict__ dv,
                                   const TT* __restrict__ cos_t, const TT* __restrict__ sin_t,
                                   const int* __restrict__ pos, __nv_bfloat16* __restrict__ dgqkv, int64_t ld, int64_t T,
                                   int H, int KV) {
  const int heads = H + 2 * KV;  // q heads, k heads, v heads
  const int64_t total = T * heads * 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int chunk = (int)(i & 7);
    const int64_t th = i >> 3;
    const int h = (int)(th % heads);
    const int64_t t = th / heads;
    const int d0 = chunk * 8;
    __nv_bfloat16* dst = dgqkv + t * ld + (int64_t)(H + h) * 128;
    float lo[8], hi[8];
    if (h < H + KV) {
      if (h < H) {
        const TQ* src = dq + (t * H + h) * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) lo[j] = to_f(src[d0 + j]), hi[j] = to_f(src[64 + d0 + j]);
      } else {
        const TK* src = dk + (t * KV + (h - H)) * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) lo[j] = to_f(src[d0 + j]), hi[j] = to_f(src[64 + d0 + j]);
      }
      const int64_t p = pos[t];
      const TT* c = cos_t + p * 128;
      const TT* s = sin_t + p * 128;
      float olo[8], ohi[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        olo[j] = lo[j] * to_f(c[d0 + j]) + hi[j] * to_f(s[64 + d0 + j]);
        ohi[j] = hi[j] * to_f(c[64 + d0 + j]) - lo[j] * to_f(s[d0 + j]);
      }
      Vec<__nv_bfloat16>::store(dst + d0, olo);
      Vec<__nv_bfloat16>::store(dst + 64 + d0, ohi);
    } else {
      const TV* src = dv + (t * KV + (h - H - KV)) * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) lo[j] = to_f(src[d0 + j]), hi[j] = to_f(src[64 + d0 + j]);
      Vec<__nv_bfloat16>::store(dst + d0, lo);
      Vec<__nv_bfloat16>::store(dst + 64 + d0, hi);
    }
  }
}

// ------------------------------------------------------------------ attention gate backward
// y = sigmoid(g) * o.  do = dy * s ; dg = dy * o * s * (1 - s) ; delta[h, t] = sum_d do * o.
// One warp per (token, head): 32 lanes x 4 elements = 128.
__global__ void attn_gate_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ o,
                                     const __nv_bfloat16* __restrict__ gqkv, int64_t ld_g,
                                     __nv_bfloat16* __restrict__ d_o, __nv_bfloat16* __restrict__ dgqkv,
                                     float* __restrict__ delta, int64_t T, int H, int64_t delta_ld) {
  const int64_t warp_id = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= T * H) return;
  const int64_t t = warp_id / H;
  const int h = (int)(warp_id % H);
  const int64_t off = (t * H + h) * 128 + lane * 4;
  const int64_t goff = t * ld_g + (int64_t)h * 128 + lane * 4;
  float acc = 0.f;
  float dov[4], dgv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float g = __bfloat162float(gqkv[goff + j]);
    const float s = 1.f / (1.f + __expf(-g));
    const float d = __bfloat162float(dy[off + j]);
    const float ov = __bfloat162float(o[off + j]);
    dov[j] = d * s;
    dgv[j] = d * ov * s * (1.f - s);
    acc += __bfloat162float(__float2bfloat16(dov[j])) * ov;
  }
  *reinterpret_cast<uint2*>(d_o + off) = make_uint2(pack_bf16x2(dov[0], dov[1]), pack_bf16x2(dov[2], dov[3]));
  *reinterpret_cast<uint2*>(dgqkv + goff) = make_uint2(pack_bf16x2(dgv[0], dgv[1]), pack_bf16x2(dgv[2], dgv[3]));
  acc = warp_sum(acc);
  if (lane == 0) delta[(int64_t)h * delta_ld + t] = acc;
}

// delta[h, t] = sum_d do[t,h,d] * o[t,h,d] (ungated attention).
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ d_o, const __nv_bfloat16* __restrict__ o,
                                  float* __restrict__ delta, int64_t T, int H, int64_t delta_ld) {
  const int64_t warp_id = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= T * H) return;
  const int64_t t = warp_id / H;
  const int h = (int)(warp_id % H);
  const int64_t off = (t * H + h) * 128 + lane * 4;
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) acc += __bfloat162float(d_o[off + j]) * __bfloat162float(o[off + j]);
  acc = warp_sum(acc);
  if (lane == 0) delta[(int64_t)h * delta_ld + t] = acc;
}

int grid_for(int64_t work, int threads) {
  int64_t blocks = (work + threads - 1) / threads;
  const int cap = 148 * 16;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, cap));
}

template <typename T>
void launch_rmsnorm_fwd(const at::Tensor& x, at::Tensor& y, at::Tensor& rstd, float eps, cudaStream_t st) {
  const int d = x.size(-1);
  const int64_t rows = x.numel() / d;
  const int vecs = d / Vec<T>::N;
  const int threads = std::min(256, ((vecs + 31) / 32) * 32);
  const int vpt = (vecs + threads - 1) / threads;
  auto xp = reinterpret_cast<const T*>(x.data_ptr());
  auto yp = reinterpret_cast<T*>(y.data_ptr());
  float* rp = rstd.data_ptr<float>();
  if (rows == 0) return;
  if (vpt <= 1) rmsnorm_fwd_kernel<T, 1><<<rows, threads, 0, st>>>(xp, yp, rp, d, eps);
  else if (vpt <= 2) rmsnorm_fwd_kernel<T, 2><<<rows, threads, 0, st>>>(xp, yp, rp, d, eps);
  else if (vpt <= 4) rmsnorm_fwd_kernel<T, 4><<<rows, threads, 0, st>>>(xp, yp, rp, d, eps);
  else if (vpt <= 8) rmsnorm_fwd_kernel<T, 8><<<rows, threads, 0, st>>>(xp, yp, rp, d, eps);
  else TORCH_CHECK(false, "rmsnorm: hidden size too large");
}

template <typename T>
void launch_rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& rstd, at::Tensor& dx,
                        cudaStream_t st) {
  const int d = x.size(-1);
  const int64_t rows = x.numel() / d;
  const int vecs = d / Vec<T>::N;
  const int threads = std::min(256, ((vecs + 31) / 32) * 32);
  const int vpt = (vecs + threads - 1) / threads;
  auto a = reinterpret_cast<const T*>(dy.data_ptr());
  auto b = reinterpret_cast<const T*>(x.data_ptr());
  auto o = reinterpret_cast<T*>(dx.data_ptr());
  const float* r = rstd.data_ptr<float>();
  if (rows == 0) return;
  if (vpt <= 1) rmsnorm_bwd_kernel<T, 1><<<rows, threads, 0, st>>>(a, b, r, o, d);
  else if (vpt <= 2) rmsnorm_bwd_kernel<T, 2><<<rows, threads, 0, st>>>(a, b, r, o, d);
  else if (vpt <= 4) rmsnorm_bwd_kernel<T, 4><<<rows, threads, 0, st>>>(a, b, r, o, d);
  else if (vpt <= 8) rmsnorm_bwd_kernel<T, 8><<<rows, threads, 0, st>>>(a, b, r, o, d);
  else TORCH_CHECK(false, "rmsnorm: hidden size too large");
}

template <typename T>
void launch_add_rmsnorm_fwd(const at::Tensor& x, const at::Tensor& delta, at::Tensor& h, at::Tensor& y,
                            at::Tensor& rstd, float eps, cudaStream_t st) {
  const int d = x.size(-1);
  const int64_t rows = x.numel() / d;
  const int vecs = d / Vec<T>::N;
  const int threads = std::min(256, ((vecs + 31) / 32) * 32);
  const int vpt = (vecs + threads - 1) / threads;
  auto xp = reinterpret_cast<const T*>(x.data_ptr());
  auto dp = reinterpret_cast<const T*>(delta.data_ptr());
  auto hp = reinterpret_cast<T*>(h.data_ptr());
  auto yp = reinterpret_cast<T*>(y.data_ptr());
  float* rp = rstd.data_ptr<float>();
  if (rows == 0) return;
  if (vpt <= 1) add_rmsnorm_fwd_kernel<T, 1><<<rows, threads, 0, st>>>(xp, dp, hp, yp, rp, d, eps);
  else if (vpt <= 2) add_rmsnorm_fwd_kernel<T, 2><<<rows, threads, 0, st>>>(xp, dp, hp, yp, rp, d, eps);
  else if (vpt <= 4) add_rmsnorm_fwd_kernel<T, 4><<<rows, threads, 0, st>>>(xp, dp, hp, yp, rp, d, eps);
  else if (vpt <= 8) add_rmsnorm_fwd_kernel<T, 8><<<rows, threads, 0, st>>>(xp, dp, hp, yp, rp, d, eps);
  else TORCH_CHECK(false, "add_rmsnorm: hidden size too large");
}

template <typename T>
void launch_rmsnorm_bwd_res(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& rstd,
                            const at::Tensor& dres, at::Tensor& dx, cudaStream_t st) {
  const int d = x.size(-1);
  const int64_t rows = x.numel() / d;
  const int vecs = d / Vec<T>::N;
  const int threads = std::min(256, ((vecs + 31) / 32) * 32);
  const int vpt = (vecs + threads - 1) / threads;
  auto a = reinterpret_cast<const T*>(dy.data_ptr());
  auto b = reinterpret_cast<const T*>(x.data_ptr());
  auto res = reinterpret_cast<const T*>(dres.data_ptr());
  auto o = reinterpret_cast<T*>(dx.data_ptr());
  const float* r = rstd.data_ptr<float>();
  if (rows == 0) return;
  if (vpt <= 1) rmsnorm_bwd_res_kernel<T, 1><<<rows, threads, 0, st>>>(a, b, r, res, o, d);
  else if (vpt <= 2) rmsnorm_bwd_res_kernel<T, 2><<<rows, threads, 0, st>>>(a, b, r, res, o, d);
  else if (vpt <= 4) rmsnorm_bwd_res_kernel<T, 4><<<rows, threads, 0, st>>>(a, b, r, res, o, d);
  else if (vpt <= 8) rmsnorm_bwd_res_kernel<T, 8><<<rows, threads, 0, st>>>(a, b, r, res, o, d);
  else TORCH_CHECK(false, "rmsnorm: hidden size too large");
}

void check_cuda_contig(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

}  // namespace

std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, double eps) {
  check_cuda_contig(x, "x");
  c10::cuda::CUDAGuard guard(x.device());
  auto y = at::empty_like(x);
  const int64_t rows = x.numel() / x.size(-1);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kBFloat16) launch_rmsnorm_fwd<__nv_bfloat16>(x, y, rstd, (float)eps, st);
  else if (x.scalar_type() == at::kFloat) launch_rmsnorm_fwd<float>(x, y, rstd, (float)eps, st);
  else TORCH_CHECK(false, "rmsnorm: unsupported dtype");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, rstd};
}

at::Tensor rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor rstd) {
  check_cuda_contig(dy, "dy");
  check_cuda_contig(x, "x");
  c10::cuda::CUDAGuard guard(x.device());
  auto dx = at::empty_like(x);
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kBFloat16) launch_rmsnorm_bwd<__nv_bfloat16>(dy, x, rstd, dx, st);
  else if (x.scalar_type() == at::kFloat) launch_rmsnorm_bwd<float>(dy, x, rstd, dx, st);
  else TORCH_CHECK(false, "rmsnorm: unsupported dtype");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dx;
}

std::vector<at::Tensor> add_rmsnorm_fwd(at::Tensor x, at::Tensor delta, double eps) {
  check_cuda_contig(x, "x");
  check_cuda_contig(delta, "delta");
  TORCH_CHECK(x.sizes() == delta.sizes() && x.scalar_type() == delta.scalar_type(), "add_rmsnorm: x/delta mismatch");
  c10::cuda::CUDAGuard guard(x.device());
  auto h = at::empty_like(x);
  auto y = at::empty_like(x);
  const int64_t rows = x.numel() / x.size(-1);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kBFloat16) launch_add_rmsnorm_fwd<__nv_bfloat16>(x, delta, h, y, rstd, (float)eps, st);
  else if (x.scalar_type() == at::kFloat) launch_add_rmsnorm_fwd<float>(x, delta, h, y, rstd, (float)eps, st);
  else TORCH_CHECK(false, "add_rmsnorm: unsupported dtype");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {h, y, rstd};
}

at::Tensor rmsnorm_bwd_res(at::Tensor dy, at::Tensor x, at::Tensor rstd, at::Tensor dres) {
  check_cuda_contig(dy, "dy");
  check_cuda_contig(x, "x");
  check_cuda_contig(dres, "dres");
  c10::cuda::CUDAGuard guard(x.device());
  auto dx = at::empty_like(x);
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kBFloat16) launch_rmsnorm_bwd_res<__nv_bfloat16>(dy, x, rstd, dres, dx, st);
  else if (x.scalar_type() == at::kFloat) launch_rmsnorm_bwd_res<float>(dy, x, rstd, dres, dx, st);
  else TORCH_CHECK(false, "rmsnorm: unsupported dtype");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dx;
}

at::Tensor swiglu_fwd(at::Tensor gu) {
  check_cuda_contig(gu, "gu");
  c10::cuda::CUDAGuard guard(gu.device());
  const int f = gu.size(-1) / 2;
  const int64_t rows = gu.numel() / gu.size(-1);
  auto sizes = gu.sizes().vec();
  sizes.back() = f;
  auto out = at::empty(sizes, gu.options());
  auto st = at::cuda::getCurrentCUDAStream();
  if (rows == 0) return out;
  if (gu.scalar_type() == at::kBFloat16) {
    TORCH_CHECK(f % 8 == 0);
    swiglu_fwd_kernel<__nv_bfloat16><<<grid_for(rows * f / 8, 256), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, f);
  } else {
    TORCH_CHECK(gu.scalar_type() == at::kFloat && f % 4 == 0);
    swiglu_fwd_kernel<float><<<grid_for(rows * f / 4, 256), 256, 0, st>>>(gu.data_ptr<float>(), out.data_ptr<float>(),
                                                                           rows, f);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

at::Tensor swiglu_bwd(at::Tensor dp, at::Tensor gu) {
  check_cuda_contig(dp, "dp");
  check_cuda_contig(gu, "gu");
  c10::cuda::CUDAGuard guard(gu.device());
  const int f = gu.size(-1) / 2;
  const int64_t rows = gu.numel() / gu.size(-1);
  auto dgu = at::empty_like(gu);
  auto st = at::cuda::getCurrentCUDAStream();
  if (rows == 0) return dgu;
  if (gu.scalar_type() == at::kBFloat16) {
    swiglu_bwd_kernel<__nv_bfloat16><<<grid_for(rows * f / 8, 256), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(dp.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), rows, f);
  } else {
    swiglu_bwd_kernel<float><<<grid_for(rows * f / 4, 256), 256, 0, st>>>(dp.data_ptr<float>(), gu.data_ptr<float>(),
                                                                           dgu.data_ptr<float>(), rows, f);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dgu;
}

at::Tensor rope_qk(at::Tensor gqkv, at::Tensor cos_t, at::Tensor sin_t, at::Tensor pos, int64_t H, int64_t KV) {
  check_cuda_contig(gqkv, "gqkv");
  TORCH_CHECK(gqkv.scalar_type() == at::kBFloat16 && gqkv.dim() == 2);
  TORCH_CHECK((cos_t.scalar_type() == at::kFloat || cos_t.scalar_type() == at::kBFloat16) && cos_t.size(-1) == 128 &&
              cos_t.is_contiguous() && sin_t.is_contiguous() && sin_t.scalar_type() == cos_t.scalar_type(),
              "rope tables must be contiguous fp32/bf16 [max_seq, 128]");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.is_contiguous());
  c10::cuda::CUDAGuard guard(gqkv.device());
  const int64_t T = gqkv.size(0);
  TORCH_CHECK(gqkv.size(1) == (2 * H + 2 * KV) * 128, "gqkv width mismatch");
  auto qk = at::empty({T, (H + KV) * 128}, gqkv.options());
  auto st = at::cuda::getCurrentCUDAStream();
  if (T == 0) return qk;
  const int heads = (int)(H + KV);
  auto launch = [&](auto* c, auto* s) {
    rope_qk_fwd_kernel<<<grid_for(T * heads * 8, 256), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(gqkv.data_ptr()), gqkv.size(1),
        reinterpret_cast<__nv_bfloat16*>(qk.data_ptr()), qk.size(1), c, s, pos.data_ptr<int>(), T, (int)H, heads);
  };
  if (cos_t.scalar_type() == at::kFloat) launch(cos_t.data_ptr<float>(), sin_t.data_ptr<float>());
  else launch(reinterpret_cast<const __nv_bfloat16*>(cos_t.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(sin_t.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return qk;
}

void rope_qk_bwd(at::Tensor dq, at::Tensor dk, at::Tensor dv, at::Tensor cos_t, at::Tensor sin_t, at::Tensor pos,
                 at::Tensor dgqkv, int64_t H, int64_t KV) {
  check_cuda_contig(dq, "dq");
  check_cuda_contig(dk, "dk");
  check_cuda_contig(dv, "dv");
  check_cuda_contig(dgqkv, "dgqkv");
  c10::cuda::CUDAGuard guard(dgqkv.device());
  const int64_t T = dgqkv.size(0);
  auto st = at::cuda::getCurrentCUDAStream();
  if (T == 0) return;
  const int64_t work = T * (H + 2 * KV) * 8;
  const bool tf = cos_t.scalar_type() == at::kFloat;
  auto args = [&](auto* q, auto* k, auto* v) {
    auto* out = reinterpret_cast<__nv_bfloat16*>(dgqkv.data_ptr());
    if (tf)
      rope_qk_bwd_kernel<<<grid_for(work, 256), 256, 0, st>>>(q, k, v, cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                                                              pos.data_ptr<int>(), out, dgqkv.size(1), T, (int)H, (int)KV);
    else
      rope_qk_bwd_kernel<<<grid_for(work, 256), 256, 0, st>>>(
          q, k, v, reinterpret_cast<const __nv_bfloat16*>(cos_t.data_ptr()),
          reinterpret_cast<const __nv_bfloat16*>(sin_t.data_ptr()), pos.data_ptr<int>(), out, dgqkv.size(1), T, (int)H,
          (int)KV);
  };
  using bf = __nv_bfloat16;
  const bool qf = dq.scalar_type() == at::kFloat, kf = dk.scalar_type() == at::kFloat, vf = dv.scalar_type() == at::kFloat;
  auto qb = reinterpret_cast<const bf*>(dq.data_ptr());
  auto kb = reinterpret_cast<const bf*>(dk.data_ptr());
  auto vb = reinterpret_cast<const bf*>(dv.data_ptr());
  if (qf && kf && vf) args(dq.data_ptr<float>(), dk.data_ptr<float>(), dv.data_ptr<float>());
  else if (qf && !kf && !vf) args(dq.data_ptr<float>(), kb, vb);
  else if (!qf && !kf && !vf) args(qb, kb, vb);
  else if (qf && kf && !vf) args(dq.data_ptr<float>(), dk.data_ptr<float>(), vb);
  else TORCH_CHECK(false, "rope_qk_bwd: unsupported dtype combination");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

std::vector<at::Tensor> attn_gate_bwd(at::Tensor dy, at::Tensor o, at::Tensor gqkv, at::Tensor dgqkv, int64_t H) {
  check_cuda_contig(dy, "dy");
  check_cuda_contig(o, "o");
  c10::cuda::CUDAGuard guard(o.device());
  const int64_t T = o.size(0);
  auto d_o = at::empty_like(o);
  const int64_t tpad = ((T + 127) / 128) * 128;
  auto delta = at::empty({H, tpad}, o.options().dtype(at::kFloat));
  auto st = at::cuda::getCurrentCUDAStream();
  if (T == 0) return {d_o, delta};
  const int64_t warps = T * H;
  attn_gate_bwd_kernel<<<(warps * 32 + 255) / 256, 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(gqkv.data_ptr()), gqkv.size(1),
      reinterpret_cast<__nv_bfloat16*>(d_o.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dgqkv.data_ptr()),
      delta.data_ptr<float>(), T, (int)H, tpad);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {d_o, delta};
}

at::Tensor attn_delta(at::Tensor d_o, at::Tensor o, int64_t H) {
  check_cuda_contig(d_o, "do");
  check_cuda_contig(o, "o");
  c10::cuda::CUDAGuard guard(o.device());
  const int64_t T = o.size(0);
  const int64_t tpad = ((T + 127) / 128) * 128;
  auto delta = at::empty({H, tpad}, o.options().dtype(at::kFloat));
  auto st = at::cuda::getCurrentCUDAStream();
  if (T == 0) return delta;
  attn_delta_kernel<<<(T * H * 32 + 255) / 256, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(d_o.data_ptr()),
                                                             reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()),
                                                             delta.data_ptr<float>(), T, (int)H, tpad);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return delta;
}
