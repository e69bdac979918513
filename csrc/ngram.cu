// Hashed n-gram memory: for each token, order and head, recompute the polynomial hash of
// the previous `order` tokens, check that they are consecutive positions of one packed
// sequence, and sum the gathered table rows (forward); scatter-add gradients into fp32
// table gradients (backward).  One warp per token.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace {

constexpr int kMaxOrders = 8;
constexpr int kMaxHeads = 16;

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ float from_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

struct NGramArgs {
  const int64_t* ids;
  const int64_t* pos;
  int64_t S;
  int64_t buckets;
  int norders, heads, width;  // width = hidden / heads
  int orders[kMaxOrders];
  uint64_t tables[kMaxOrders * kMaxHeads];  // table pointer per (order index, head)
};

// Hash of the `order` tokens ending at t for head h; valid = consecutive same-sequence positions.
__device__ __forceinline__ bool ngram_hash(const NGramArgs& a, int64_t t, int order, int h, int64_t& out) {
  const int64_t base = 65599 + 2 * h;
  int64_t v = 0;
  for (int o = 0; o < order; ++o) {
    if (t - o < 0) return false;
    if (a.pos[t] - a.pos[t - o] != o) return false;
    v = (v * base + a.ids[t - o] + 1) % a.buckets;
  }
  out = v;
  return true;
}

template <typename TT, typename TO>
__global__ void ngram_fwd_kernel(NGramArgs a, TO* __restrict__ out) {
  const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= a.S) return;
  const int hidden = a.width * a.heads;
  float acc_cache[32];  // up to 1024 hidden / 32 lanes
  const int per_lane = (hidden + 31) / 32;
  for (int i = 0; i < per_lane && i < 32; ++i) acc_cache[i] = 0.f;
  for (int oi = 0; oi < a.norders; ++oi) {
    for (int h = 0; h < a.heads; ++h) {
      int64_t hv;
      if (!ngram_hash(a, t, a.orders[oi], h, hv)) continue;
      const TT* row = reinterpret_cast<const TT*>(a.tables[oi * a.heads + h]) + hv * a.width;
      for (int i = 0; i < per_lane && i < 32; ++i) {
        const int c = lane + i * 32;
        if (c < hidden && c / a.width == h) acc_cache[i] += to_float(row[c - h * a.width]);
      }
    }
  }
  for (int i = 0; i < per_lane && i < 32; ++i) {
    const int c = lane + i * 32;
    if (c < hidden) out[t * hidden + c] = from_float<TO>(acc_cache[i]);
  }
}

template <typename TO>
__global__ void ngram_bwd_kernel(NGramArgs a, const TO* __restrict__ dout) {
  const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= a.S) return;
  const int hidden = a.width * a.heads;
  for (int oi = 0; oi < a.norders; ++oi) {
    for (int h = 0; h < a.heads; ++h) {
      int64_t hv;
      if (!ngram_hash(a, t, a.orders[oi], h, hv)) continue;
      float* row = reinterpret_cast<float*>(a.tables[oi * a.heads + h]) + hv * a.width;
      for (int c = lane; c < a.width; c += 32) atomicAdd(row + c, to_float(dout[t * hidden + h * a.width + c]));
    }
  }
}

NGramArgs make_args(const at::Tensor& ids, const at::Tensor& pos, const std::vector<at::Tensor>& tables,
                    const std::vector<int64_t>& orders, int64_t heads, int64_t buckets) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.dim() == 1);
  TORCH_CHECK(pos.scalar_type() == at::kLong && pos.is_contiguous() && pos.numel() == ids.numel());
  TORCH_CHECK((int64_t)orders.size() <= kMaxOrders && heads <= kMaxHeads);
  TORCH_CHECK((int64_t)tables.size() == (int64_t)orders.size() * heads);
  NGramArgs a{};
  a.ids = ids.data_ptr<int64_t>();
  a.pos = pos.data_ptr<int64_t>();
  a.S = ids.numel();
  a.buckets = buckets;
  a.norders = (int)orders.size();
  a.heads = (int)heads;
  a.width = (int)tables[0].size(1);
  TORCH_CHECK(a.width * a.heads <= 1024, "n-gram hidden size above 1024 is not supported by the kernel");
  for (size_t i = 0; i < orders.size(); ++i) a.orders[i] = (int)orders[i];
  for (size_t i = 0; i < tables.size(); ++i) {
    TORCH_CHECK(tables[i].is_contiguous() && tables[i].size(0) == buckets && tables[i].size(1) == a.width);
    a.tables[i] = reinterpret_cast<uint64_t>(tables[i].data_ptr());
  }
  return a;
}

}  // namespace

at::Tensor ngram_fwd(at::Tensor ids, at::Tensor pos, std::vector<at::Tensor> tables, std::vector<int64_t> orders,
                     int64_t heads, int64_t buckets, at::ScalarType dtype) {
  c10::cuda::CUDAGuard guard(ids.device());
  NGramArgs a = make_args(ids, pos, tables, orders, heads, buckets);
  auto out = at::empty({a.S, (int64_t)a.width * heads}, ids.options().dtype(dtype));
  if (a.S == 0) return out;
  const int threads = 256;
  const int64_t blocks = (a.S * 32 + threads - 1) / threads;
  auto st = at::cuda::getCurrentCUDAStream();
  const auto tdt = tables[0].scalar_type();
  if (tdt == at::kFloat && dtype == at::kFloat) ngram_fwd_kernel<float, float><<<blocks, threads, 0, st>>>(a, out.data_ptr<float>());
  else if (tdt == at::kFloat && dtype == at::kBFloat16)
    ngram_fwd_kernel<float, __nv_bfloat16><<<blocks, threads, 0, st>>>(a, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  else if (tdt == at::kBFloat16 && dtype == at::kBFloat16)
    ngram_fwd_kernel<__nv_bfloat16, __nv_bfloat16><<<blocks, threads, 0, st>>>(a, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  else if (tdt == at::kBFloat16 && dtype == at::kFloat)
    ngram_fwd_kernel<__nv_bfloat16, float><<<blocks, threads, 0, st>>>(a, out.data_ptr<float>());
  else TORCH_CHECK(false, "ngram_fwd: unsupported dtypes");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void ngram_bwd(at::Tensor dout, at::Tensor ids, at::Tensor pos, std::vector<at::Tensor> grads,
               std::vector<int64_t> orders, int64_t heads, int64_t buckets) {
  c10::cuda::CUDAGuard guard(ids.device());
  for (auto& g : grads) TORCH_CHECK(g.scalar_type() == at::kFloat, "ngram_bwd: table grads must be fp32");
  NGramArgs a = make_args(ids, pos, grads, orders, heads, buckets);
  if (a.S == 0) return;
  const int threads = 256;
  const int64_t blocks = (a.S * 32 + threads - 1) / threads;
  auto st = at::cuda::getCurrentCUDAStream();
  if (dout.scalar_type() == at::kFloat) ngram_bwd_kernel<float><<<blocks, threads, 0, st>>>(a, dout.data_ptr<float>());
  else ngram_bwd_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(a, reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
