// Hashed n-gram memory: for each token, order and head, recompute the polynomial hash of
// the previous `order` tokens, check that they are consecutive positions of one packed
// sequence, and sum the gathered table rows (forward, one warp per token); the backward sums
// each hashed row's gradient over a sorted key list (below).
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

// Backward, deterministic and without atomics.  Pass 1 gives every (token, order, head) a key:
// (order index * heads + head) * buckets + hash, or kNoKey when the n-gram is not valid.  The
// caller sorts the keys stably; pass 2 runs one warp per sorted position: the warp at the head
// of a run of equal keys sums that run's dout slices in fp32, in token order, and adds the sum
// to the gradient row once (read-modify-write in the gradient's dtype).  Only hashed rows are
// touched, so the gradient can be the optimizer's accumulation buffer itself.
constexpr int64_t kNoKey = INT64_MAX;

__global__ void ngram_keys_kernel(NGramArgs a, int64_t* __restrict__ keys) {
  const int per = a.norders * a.heads;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= a.S * per) return;
  const int64_t t = i / per;
  const int j = static_cast<int>(i % per);
  int64_t hv;
  keys[i] = ngram_hash(a, t, a.orders[j / a.heads], j % a.heads, hv) ? int64_t(j) * a.buckets + hv : kNoKey;
}

__device__ __forceinline__ float load_f(const float* p) { return *p; }
__device__ __forceinline__ float load_f(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void store_f(float* p, float v) { *p = v; }
__device__ __forceinline__ void store_f(__nv_bfloat16* p, float v) { *p = __float2bfloat16(v); }

template <typename TD, typename TG>
__global__ void ngram_bwd_kernel(NGramArgs a, const TD* __restrict__ dout, const int64_t* __restrict__ keys,
                                 const int64_t* __restrict__ order, int64_t n) {
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int per = a.norders * a.heads;
  const int hidden = a.width * a.heads;
  for (int64_t i = warp; i < n; i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t key = keys[i];
    if (key == kNoKey || (i > 0 && keys[i - 1] == key)) continue;  // invalid, or not a run head
    int64_t end = i + 1;
    while (end < n && keys[end] == key) ++end;
    const int j = static_cast<int>(key / a.buckets);
    const int h = j % a.heads;
    TG* row = reinterpret_cast<TG*>(a.tables[j]) + (key % a.buckets) * a.width;
    for (int c = lane; c < a.width; c += 32) {
      float acc = 0.f;
      for (int64_t k = i; k < end; ++k) acc += to_float(dout[(order[k] / per) * hidden + h * a.width + c]);
      store_f(row + c, load_f(row + c) + acc);
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

// Keys of every (token, order, head), for the caller's stable sort.
at::Tensor ngram_keys(at::Tensor ids, at::Tensor pos, std::vector<int64_t> orders, int64_t heads, int64_t buckets,
                      int64_t width) {
  c10::cuda::CUDAGuard guard(ids.device());
  TORCH_CHECK((int64_t)orders.size() <= kMaxOrders && heads <= kMaxHeads, "too many n-gram orders or heads");
  NGramArgs a{};
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.dim() == 1);
  TORCH_CHECK(pos.scalar_type() == at::kLong && pos.is_contiguous() && pos.numel() == ids.numel());
  a.ids = ids.data_ptr<int64_t>();
  a.pos = pos.data_ptr<int64_t>();
  a.S = ids.numel();
  a.buckets = buckets;
  a.norders = (int)orders.size();
  a.heads = (int)heads;
  a.width = (int)width;
  for (size_t i = 0; i < orders.size(); ++i) a.orders[i] = (int)orders[i];
  auto keys = at::empty({a.S * a.norders * a.heads}, ids.options());
  if (keys.numel() == 0) return keys;
  const int threads = 256;
  ngram_keys_kernel<<<(keys.numel() + threads - 1) / threads, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      a, keys.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return keys;
}

// grads[j] += sum of dout slices whose sorted key names table j; sorted_keys / order: the stable
// sort of ngram_keys() and the original indices.  grads: [buckets, width], bf16 or fp32.
void ngram_bwd(at::Tensor dout, at::Tensor ids, at::Tensor pos, at::Tensor sorted_keys, at::Tensor order,
               std::vector<at::Tensor> grads, std::vector<int64_t> orders, int64_t heads, int64_t buckets) {
  c10::cuda::CUDAGuard guard(ids.device());
  NGramArgs a = make_args(ids, pos, grads, orders, heads, buckets);
  const auto gdt = grads[0].scalar_type();
  for (auto& g : grads)
    TORCH_CHECK(g.scalar_type() == gdt && (gdt == at::kFloat || gdt == at::kBFloat16),
                "ngram_bwd: table grads must all be fp32 or all bf16");
  const int64_t n = sorted_keys.numel();
  TORCH_CHECK(sorted_keys.scalar_type() == at::kLong && order.scalar_type() == at::kLong && order.numel() == n &&
                  n == a.S * a.norders * a.heads && sorted_keys.is_contiguous() && order.is_contiguous(),
              "ngram_bwd: one sorted key and index per (token, order, head)");
  TORCH_CHECK(dout.is_contiguous() && dout.numel() == a.S * a.width * a.heads, "ngram_bwd: dout [tokens, hidden]");
  if (n == 0) return;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((n * 32 + threads - 1) / threads, 148 * 16);
  auto st = at::cuda::getCurrentCUDAStream();
  const int64_t* k = sorted_keys.data_ptr<int64_t>();
  const int64_t* o = order.data_ptr<int64_t>();
  const bool fd = dout.scalar_type() == at::kFloat;
  TORCH_CHECK(fd || dout.scalar_type() == at::kBFloat16, "ngram_bwd: dout must be fp32 or bf16");
  const auto* db = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  if (fd && gdt == at::kFloat) ngram_bwd_kernel<float, float><<<blocks, threads, 0, st>>>(a, dout.data_ptr<float>(), k, o, n);
  else if (fd) ngram_bwd_kernel<float, __nv_bfloat16><<<blocks, threads, 0, st>>>(a, dout.data_ptr<float>(), k, o, n);
  else if (gdt == at::kFloat) ngram_bwd_kernel<__nv_bfloat16, float><<<blocks, threads, 0, st>>>(a, db, k, o, n);
  else ngram_bwd_kernel<__nv_bfloat16, __nv_bfloat16><<<blocks, threads, 0, st>>>(a, db, k, o, n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
