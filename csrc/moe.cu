// Mixture-of-experts token exchange over NVLink peer memory (expert parallelism), fused with the
// top-k permutation and the routing-weight combine.
//
// Every rank owns E/W experts.  A token-slot (t, j) — token t's j-th routed expert e — has a
// destination rank dst = e / (E/W) and a row in that rank's receive buffer; rows are grouped by
// expert, then by source rank, then by token (the host computes them from the all-gathered
// per-expert counts, so the layout is "capacity free": a buffer holds exactly the routed rows).
// The receive buffers are CUDA-IPC mappings, so the exchange is plain loads and stores:
//
//   dispatch      recv[dst][row(t,j)]  = x[t]                       (one load of x[t], k peer stores)
//   combine       out[t] = sum_j w[t,j] * y[dst][row(t,j)]          (peer loads, fp32 accumulate;
//                 optionally the loaded rows are kept:  ys[t*k+j] = y[dst][row(t,j)])
//   combine_bwd   dy[dst][row(t,j)] = w[t,j] * dout[t]              (peer stores)
//                 dw[t,j] = <dout[t], ys[t*k+j]>                    (local rows kept by the forward)
//   gather_sum    dx[t] = sum_j dxp[dst][row(t,j)]                  (combine with unit weights)
//
// One warp per token walks the hidden dimension in 16-byte vectors, kUnroll vectors per lane at a
// time (loads first, then the arithmetic and stores).  With W = 1 the same
// kernels are the local permutation and un-permutation.  Nothing here waits on a peer: the
// caller orders each exchange with the other ranks by a collective before and after it.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <type_traits>

#include "common.cuh"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kWarps = 8;
constexpr int kMaxTopK = 8;

struct PeerRows {
  uint64_t ptr[kMaxRanks];  // every rank's buffer (bf16 [rows, d])
  int nranks;               // valid destination ranks
  int64_t capacity;         // valid rows per rank's buffer
  int* bad;                 // set to 1 when a route names a rank or row outside these bounds
};

// A route (rank q, row r) outside the buffers is skipped (no peer access; zero contribution)
// and reported through the status word, which the host reads with the other kernel statuses.
__device__ __forceinline__ bool route_ok(const PeerRows& p, int q, int r) {
  const bool ok = q >= 0 && q < p.nranks && r >= 0 && r < p.capacity;
  if (!ok) atomicExch(p.bad, 1);
  return ok;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 t = __bfloat1622float2(h[k]);
    f[2 * k] = t.x;
    f[2 * k + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(mimir::pack_bf16x2(f[0], f[1]), mimir::pack_bf16x2(f[2], f[3]), mimir::pack_bf16x2(f[4], f[5]),
                    mimir::pack_bf16x2(f[6], f[7]));
}

__device__ __forceinline__ const uint4* row_ptr(const PeerRows& p, int rank, int64_t row, int64_t d) {
  return reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.ptr[rank]) + row * d);
}

__device__ __forceinline__ uint4* row_ptr_mut(const PeerRows& p, int rank, int64_t row, int64_t d) {
  return reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.ptr[rank]) + row * d);
}

// Every lane first loads kUnroll 16-byte vectors (of each of the K rows) and only then uses them,
// so a warp keeps several loads in flight per lane: the copies are latency-bound otherwise.
constexpr int kUnroll = 4;

template <int K>
__global__ void __launch_bounds__(kWarps * 32) moe_dispatch_kernel(const __nv_bfloat16* __restrict__ x,
                                                                    const int32_t* __restrict__ rows,
                                                                    const int32_t* __restrict__ dst,
                                                                    const __grid_constant__ PeerRows recv, int64_t T,
                                                                    int64_t d) {
  const int64_t t = int64_t(blockIdx.x) * kWarps + threadIdx.x / 32;
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  int r[K], q[K];
  bool ok[K];
#pragma unroll
  for (int j = 0; j < K; ++j) r[j] = rows[t * K + j], q[j] = dst[t * K + j], ok[j] = route_ok(recv, q[j], r[j]);
  const uint4* src = reinterpret_cast<const uint4*>(x + t * d);
  const int64_t nv = d / 8;
  for (int64_t v0 = lane; v0 < nv; v0 += 32 * kUnroll) {
    uint4 val[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (v0 + 32 * u < nv) val[u] = src[v0 + 32 * u];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (v0 + 32 * u < nv) {
#pragma unroll
        for (int j = 0; j < K; ++j)
          if (ok[j]) row_ptr_mut(recv, q[j], r[j], d)[v0 + 32 * u] = val[u];
      }
    }
  }
  __threadfence_system();  // this thread's peer stores are visible before the closing collective
}

// out[t] = sum_j w[t,j] * y[dst][row]   (w == nullptr: unit weights); ys[t*K+j] = the loaded rows
template <int K>
__global__ void __launch_bounds__(kWarps * 32) moe_combine_kernel(const __grid_constant__ PeerRows y,
                                                                   const int32_t* __restrict__ rows,
                                                                   const int32_t* __restrict__ dst,
                                                                   const float* __restrict__ w,
                                                                   __nv_bfloat16* __restrict__ out,
                                                                   __nv_bfloat16* __restrict__ ys, int64_t T,
                                                                   int64_t d) {
  const int64_t t = int64_t(blockIdx.x) * kWarps + threadIdx.x / 32;
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  int r[K], q[K];
  float wt[K];
  bool ok[K];
#pragma unroll
  for (int j = 0; j < K; ++j)
    r[j] = rows[t * K + j], q[j] = dst[t * K + j], wt[j] = w != nullptr ? w[t * K + j] : 1.f,
    ok[j] = route_ok(y, q[j], r[j]);
  uint4* o = reinterpret_cast<uint4*>(out + t * d);
  const int64_t nv = d / 8;
  for (int64_t v0 = lane; v0 < nv; v0 += 32 * kUnroll) {
    uint4 raw[kUnroll][K];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (v0 + 32 * u < nv) {
#pragma unroll
        for (int j = 0; j < K; ++j) raw[u][j] = ok[j] ? row_ptr(y, q[j], r[j], d)[v0 + 32 * u] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = v0 + 32 * u;
      if (v >= nv) continue;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < K; ++j) {
        if (ys != nullptr) reinterpret_cast<uint4*>(ys + (t * K + j) * d)[v] = raw[u][j];
        float f[8];
        unpack8(raw[u][j], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += wt[j] * f[e];
      }
      o[v] = pack8(acc);
    }
  }
}

// dy[dst][row] = bf16(w[t,j] * dout[t]);  dw[t,j] = <dout[t], ys[t*K+j]>
template <int K>
__global__ void __launch_bounds__(kWarps * 32) moe_combine_bwd_kernel(const __nv_bfloat16* __restrict__ dout,
                                                                       const float* __restrict__ w,
                                                                       const int32_t* __restrict__ rows,
                                                                       const int32_t* __restrict__ dst,
                                                                       const __nv_bfloat16* __restrict__ ys,
                                                                       const __grid_constant__ PeerRows dy,
                                                                       float* __restrict__ dw, int64_t T, int64_t d) {
  const int64_t t = int64_t(blockIdx.x) * kWarps + threadIdx.x / 32;
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  int r[K], q[K];
  float wt[K], dot[K];
  bool ok[K];
#pragma unroll
  for (int j = 0; j < K; ++j)
    r[j] = rows[t * K + j], q[j] = dst[t * K + j], wt[j] = w[t * K + j], dot[j] = 0.f, ok[j] = route_ok(dy, q[j], r[j]);
  const uint4* g = reinterpret_cast<const uint4*>(dout + t * d);
  const int64_t nv = d / 8;
  for (int64_t v0 = lane; v0 < nv; v0 += 32 * kUnroll) {
    uint4 gr[kUnroll], yr[kUnroll][K];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (v0 + 32 * u < nv) {
        gr[u] = g[v0 + 32 * u];
#pragma unroll
        for (int j = 0; j < K; ++j) yr[u][j] = reinterpret_cast<const uint4*>(ys + (t * K + j) * d)[v0 + 32 * u];
      }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = v0 + 32 * u;
      if (v >= nv) continue;
      float gf[8];
      unpack8(gr[u], gf);
#pragma unroll
      for (int j = 0; j < K; ++j) {
        float yf[8], sc[8];
        unpack8(yr[u][j], yf);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          dot[j] += gf[e] * yf[e];
          sc[e] = wt[j] * gf[e];
        }
        if (ok[j]) row_ptr_mut(dy, q[j], r[j], d)[v] = pack8(sc);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < K; ++j) {
    float sm = dot[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
    if (lane == 0) dw[t * K + j] = sm;
  }
  __threadfence_system();
}

// Calls `launch(std::integral_constant<int, K>{})` for the top-k in use (1..kMaxTopK).
template <typename F>
void with_topk(int64_t k, F&& launch) {
  switch (k) {
    case 1: launch(std::integral_constant<int, 1>{}); break;
    case 2: launch(std::integral_constant<int, 2>{}); break;
    case 3: launch(std::integral_constant<int, 3>{}); break;
    case 4: launch(std::integral_constant<int, 4>{}); break;
    case 5: launch(std::integral_constant<int, 5>{}); break;
    case 6: launch(std::integral_constant<int, 6>{}); break;
    case 7: launch(std::integral_constant<int, 7>{}); break;
    case 8: launch(std::integral_constant<int, 8>{}); break;
    default: TORCH_CHECK(false, "top-k must be in [1, ", kMaxTopK, "]");
  }
}

int* route_flag(const at::Device& dev) {
  static at::Tensor flags[64];
  const int i = dev.index();
  if (!flags[i].defined()) flags[i] = at::zeros({1}, at::TensorOptions().device(dev).dtype(at::kInt));
  return flags[i].data_ptr<int>();
}

PeerRows make_rows(const std::vector<int64_t>& ptrs, int64_t capacity, const at::Device& dev) {
  TORCH_CHECK(ptrs.size() >= 1 && ptrs.size() <= kMaxRanks, "expert parallelism supports 1..", kMaxRanks, " ranks");
  TORCH_CHECK(capacity >= 0, "row capacity must be non-negative");
  PeerRows p{};
  for (size_t k = 0; k < ptrs.size(); ++k) {
    TORCH_CHECK(ptrs[k] % 16 == 0 && ptrs[k] != 0, "peer row buffers must be non-null and 16-byte aligned");
    p.ptr[k] = static_cast<uint64_t>(ptrs[k]);
  }
  p.nranks = static_cast<int>(ptrs.size());
  p.capacity = capacity;
  p.bad = route_flag(dev);
  return p;
}

void check_routes(const at::Tensor& rows, const at::Tensor& dst, int64_t T, int64_t k) {
  TORCH_CHECK(k >= 1 && k <= kMaxTopK, "top-k must be in [1, ", kMaxTopK, "]");
  for (const at::Tensor* t : {&rows, &dst})
    TORCH_CHECK(t->is_cuda() && t->dtype() == at::kInt && t->is_contiguous() && t->numel() == T * k,
                "routes must be contiguous int32 [T, k]");
}

unsigned blocks_for(int64_t T) { return static_cast<unsigned>((T + kWarps - 1) / kWarps); }

}  // namespace

void moe_dispatch(at::Tensor x, at::Tensor rows, at::Tensor dst, std::vector<int64_t> recv, int64_t k,
                  int64_t capacity) {
  TORCH_CHECK(x.is_cuda() && x.dtype() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x: bf16 [T, d]");
  const int64_t T = x.size(0), d = x.size(1);
  TORCH_CHECK(d % 8 == 0, "hidden size must be a multiple of 8");
  check_routes(rows, dst, T, k);
  const c10::cuda::CUDAGuard guard(x.device());
  if (T == 0) return;
  with_topk(k, [&](auto kk) {
    moe_dispatch_kernel<decltype(kk)::value><<<blocks_for(T), kWarps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), rows.data_ptr<int32_t>(), dst.data_ptr<int32_t>(),
        make_rows(recv, capacity, x.device()), T, d);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

at::Tensor moe_combine(std::vector<int64_t> y, at::Tensor rows, at::Tensor dst, c10::optional<at::Tensor> w,
                       int64_t T, int64_t k, int64_t d, c10::optional<at::Tensor> ys, int64_t capacity) {
  TORCH_CHECK(d % 8 == 0, "hidden size must be a multiple of 8");
  check_routes(rows, dst, T, k);
  if (w) TORCH_CHECK(w->is_cuda() && w->dtype() == at::kFloat && w->is_contiguous() && w->numel() == T * k,
                     "weights: fp32 [T, k]");
  if (ys) TORCH_CHECK(ys->is_cuda() && ys->dtype() == at::kBFloat16 && ys->is_contiguous() && ys->numel() == T * k * d,
                      "ys: contiguous bf16 [T * k, d]");
  const c10::cuda::CUDAGuard guard(rows.device());
  at::Tensor out = at::empty({T, d}, rows.options().dtype(at::kBFloat16));
  if (T == 0) return out;
  with_topk(k, [&](auto kk) {
    moe_combine_kernel<decltype(kk)::value><<<blocks_for(T), kWarps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
        make_rows(y, capacity, rows.device()), rows.data_ptr<int32_t>(), dst.data_ptr<int32_t>(),
        w ? w->data_ptr<float>() : nullptr,
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
        ys ? reinterpret_cast<__nv_bfloat16*>(ys->data_ptr()) : nullptr, T, d);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

at::Tensor moe_combine_bwd(at::Tensor dout, at::Tensor w, at::Tensor rows, at::Tensor dst, at::Tensor ys,
                           std::vector<int64_t> dy, int64_t k, int64_t capacity) {
  TORCH_CHECK(dout.is_cuda() && dout.dtype() == at::kBFloat16 && dout.is_contiguous() && dout.dim() == 2,
              "dout: bf16 [T, d]");
  const int64_t T = dout.size(0), d = dout.size(1);
  TORCH_CHECK(d % 8 == 0, "hidden size must be a multiple of 8");
  check_routes(rows, dst, T, k);
  TORCH_CHECK(w.is_cuda() && w.dtype() == at::kFloat && w.is_contiguous() && w.numel() == T * k,
              "weights: fp32 [T, k]");
  TORCH_CHECK(ys.is_cuda() && ys.dtype() == at::kBFloat16 && ys.is_contiguous() && ys.numel() == T * k * d,
              "ys: contiguous bf16 [T * k, d] (the rows the forward combine loaded)");
  const c10::cuda::CUDAGuard guard(dout.device());
  at::Tensor dw = at::empty({T, k}, w.options());
  if (T == 0) return dw;
  with_topk(k, [&](auto kk) {
    moe_combine_bwd_kernel<decltype(kk)::value><<<blocks_for(T), kWarps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), w.data_ptr<float>(), rows.data_ptr<int32_t>(),
        dst.data_ptr<int32_t>(), reinterpret_cast<const __nv_bfloat16*>(ys.data_ptr()),
        make_rows(dy, capacity, dout.device()),
        dw.data_ptr<float>(), T, d);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dw;
}

// 1 if an exchange kernel met a route outside its buffers since the last read (that slot was skipped).
int64_t moe_route_status(int64_t device) {
  int* flag = route_flag(at::Device(at::kCUDA, static_cast<c10::DeviceIndex>(device)));
  int host = 0;
  C10_CUDA_CHECK(cudaMemcpy(&host, flag, sizeof(int), cudaMemcpyDeviceToHost));
  if (host) C10_CUDA_CHECK(cudaMemset(flag, 0, sizeof(int)));
  return host;
}
