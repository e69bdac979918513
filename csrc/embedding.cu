// Scaled token embedding: out[t, :] = scale * E[ids[t], :] and its gradient
//   dE[v, :] += scale * sum_{t : ids[t] = v} dout[t, :].
//
// Forward: one warp per token row, 16-byte vector loads and stores, the scale applied in fp32 and
// rounded once (what `scale * F.embedding(ids, E)` computes for bf16 and fp32).
//
// Backward without atomics on the gradient, deterministic: the caller passes the token ids sorted
// stably (so the positions of one id are in increasing order).  One warp per sorted position; the
// warp that starts a run of equal ids sums a short run's dout rows in fp32, in position order, and
// adds scale * sum to the gradient row once (read-modify-write in the gradient's dtype); a long
// run goes to a second kernel in which one CTA sums it with eight warps in a fixed order.  Every
// other warp exits.  Reference: `src/mimir/model/layers.py:103-104` (ScaledEmbeddingInit.forward).
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

// 8 consecutive elements of one row as fp32 (one 16-byte load for bf16, two for fp32).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  Vec8<T>::load(p, v);
  if constexpr (Vec8<T>::N == 4) Vec8<T>::load(p + 4, v + 4);
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]) {
  Vec8<T>::store(p, v);
  if constexpr (Vec8<T>::N == 4) Vec8<T>::store(p + 4, v + 4);
}

constexpr int kShortRun = 32;      // runs up to this many rows are summed by one warp
constexpr int kPasses = 8;         // 256-column passes a warp keeps in flight per row (2048 columns)
constexpr int kLongWarps = 8;      // warps that share one long run

// One warp per sorted position.  The warp that starts a run finds its end 32 positions at a
// time; a short run is summed here (row by row, every column pass of the row in flight), a long
// run is appended to `long_runs` for embed_bwd_long_kernel.  Each run sums in position order.
template <typename TD, typename TG>
__global__ void embed_bwd_kernel(const TD* __restrict__ dout, const int64_t* __restrict__ sorted_ids,
                                 const int64_t* __restrict__ order, TG* __restrict__ grad, int64_t tokens, int d,
                                 int64_t vocab, float scale, int64_t* __restrict__ long_runs, int* __restrict__ n_long) {
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t i = warp; i < tokens; i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t id = sorted_ids[i];
    if ((i > 0 && sorted_ids[i - 1] == id) || id < 0 || id >= vocab) continue;  // not a run head
    int64_t end = i + 1;
    while (true) {
      const int64_t q = end + lane;
      const unsigned same = __ballot_sync(0xffffffffu, q < tokens && sorted_ids[q] == id);
      if (same != 0xffffffffu) {
        end += __ffs(~same) - 1;
        break;
      }
      end += 32;
    }
    const int len = end - i > kShortRun ? kShortRun + 1 : static_cast<int>(end - i);
    if (len > kShortRun) {
      if (lane == 0) {
        const int slot = atomicAdd(n_long, 1);
        long_runs[2 * slot] = i;
        long_runs[2 * slot + 1] = end;
      }
      continue;
    }
    const int64_t mine = lane < len ? order[i + lane] : 0;  // the run's positions, one per lane
    TG* row = grad + id * d;
    for (int c0 = 0; c0 < d; c0 += kPasses * 256) {
      float acc[kPasses][8];
#pragma unroll
      for (int p = 0; p < kPasses; ++p)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[p][e] = 0.f;
      for (int k = 0; k < len; ++k) {
        const TD* src = dout + __shfl_sync(0xffffffffu, mine, k) * d;
#pragma unroll
        for (int p = 0; p < kPasses; ++p) {
          const int c = c0 + p * 256 + lane * 8;
          if (c < d) {
            float v[8];
            load8(src + c, v);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[p][e] += v[e];
          }
        }
      }
#pragma unroll
      for (int p = 0; p < kPasses; ++p) {
        const int c = c0 + p * 256 + lane * 8;
        if (c < d) {
          float g[8];
          load8(row + c, g);
#pragma unroll
          for (int e = 0; e < 8; ++e) g[e] += scale * acc[p][e];
          store8(row + c, g);
        }
      }
    }
  }
}

// One CTA per long run (runs listed by embed_bwd_kernel): warp w sums rows i + w, i + w + 8, ...
// in order, the eight partial sums meet in shared memory and are added in warp order, so the
// result does not depend on scheduling.  Zipf-distributed token ids give runs of thousands of
// rows, which one warp would sum serially.
template <typename TD, typename TG>
__global__ void __launch_bounds__(32 * kLongWarps) embed_bwd_long_kernel(
    const TD* __restrict__ dout, const int64_t* __restrict__ sorted_ids, const int64_t* __restrict__ order,
    TG* __restrict__ grad, int d, float scale, const int64_t* __restrict__ long_runs, const int* __restrict__ n_long) {
  extern __shared__ float part[];  // [kLongWarps][kPasses * 256]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int count = *n_long;
  for (int r = blockIdx.x; r < count; r += gridDim.x) {
    const int64_t i = long_runs[2 * r], end = long_runs[2 * r + 1];
    TG* row = grad + sorted_ids[i] * d;
    for (int c0 = 0; c0 < d; c0 += kPasses * 256) {
      float acc[kPasses][8];
#pragma unroll
      for (int p = 0; p < kPasses; ++p)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[p][e] = 0.f;
      for (int64_t k0 = i + warp; k0 < end; k0 += 32 * kLongWarps) {
        // this warp's next 32 rows: k0, k0 + 8, ..., one position per lane
        const int64_t kl = k0 + static_cast<int64_t>(lane) * kLongWarps;
        const int64_t mine = kl < end ? order[kl] : 0;
        const int64_t left = (end - k0 + kLongWarps - 1) / kLongWarps;
        const int rows = left < 32 ? static_cast<int>(left) : 32;
        for (int j = 0; j < rows; ++j) {
          const TD* src = dout + __shfl_sync(0xffffffffu, mine, j) * d;
#pragma unroll
          for (int p = 0; p < kPasses; ++p) {
            const int c = c0 + p * 256 + lane * 8;
            if (c < d) {
              float v[8];
              load8(src + c, v);
#pragma unroll
              for (int e = 0; e < 8; ++e) acc[p][e] += v[e];
            }
          }
        }
      }
#pragma unroll
      for (int p = 0; p < kPasses; ++p)
#pragma unroll
        for (int e = 0; e < 8; ++e) part[warp * kPasses * 256 + p * 256 + lane * 8 + e] = acc[p][e];
      __syncthreads();
      for (int c = threadIdx.x * 8; c < kPasses * 256 && c0 + c < d; c += 32 * kLongWarps * 8) {
        float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int w = 0; w < kLongWarps; ++w)
#pragma unroll
          for (int e = 0; e < 8; ++e) sum[e] += part[w * kPasses * 256 + c + e];
        float g[8];
        load8(row + c0 + c, g);
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] += scale * sum[e];
        store8(row + c0 + c, g);
      }
      __syncthreads();
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

// Short runs and the list of long runs, then one CTA per long run.
template <typename TD, typename TG>
void launch_embed_bwd(const at::Tensor& dout, const at::Tensor& sorted_ids, const at::Tensor& order, at::Tensor& grad,
                      int64_t T, int64_t d, int64_t V, float s, cudaStream_t st) {
  // at most one long run per kShortRun + 1 positions
  at::Tensor long_runs = at::empty({2 * (T / (kShortRun + 1) + 1)}, sorted_ids.options());
  at::Tensor n_long = at::zeros({1}, sorted_ids.options().dtype(at::kInt));
  embed_bwd_kernel<TD, TG><<<grid_warps(T), 256, 0, st>>>(
      reinterpret_cast<const TD*>(dout.data_ptr()), sorted_ids.data_ptr<int64_t>(), order.data_ptr<int64_t>(),
      reinterpret_cast<TG*>(grad.data_ptr()), T, static_cast<int>(d), V, s, long_runs.data_ptr<int64_t>(),
      n_long.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  constexpr int smem = kLongWarps * kPasses * 256 * static_cast<int>(sizeof(float));
  static bool attr[64] = {false};
  const int dev = grad.device().index();
  if (!attr[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(embed_bwd_long_kernel<TD, TG>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  embed_bwd_long_kernel<TD, TG><<<296, 32 * kLongWarps, smem, st>>>(
      reinterpret_cast<const TD*>(dout.data_ptr()), sorted_ids.data_ptr<int64_t>(), order.data_ptr<int64_t>(),
      reinterpret_cast<TG*>(grad.data_ptr()), static_cast<int>(d), s, long_runs.data_ptr<int64_t>(),
      n_long.data_ptr<int>());
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
  const bool db = dout.scalar_type() == at::kBFloat16, gb = grad.scalar_type() == at::kBFloat16;
  TORCH_CHECK((db || dout.scalar_type() == at::kFloat) && (gb || grad.scalar_type() == at::kFloat),
              "dout and grad: bf16 or fp32");
  if (db && gb) launch_embed_bwd<__nv_bfloat16, __nv_bfloat16>(dout, sorted_ids, order, grad, T, d, V, s, st);
  else if (db) launch_embed_bwd<__nv_bfloat16, float>(dout, sorted_ids, order, grad, T, d, V, s, st);
  else if (gb) launch_embed_bwd<float, __nv_bfloat16>(dout, sorted_ids, order, grad, T, d, V, s, st);
  else launch_embed_bwd<float, float>(dout, sorted_ids, order, grad, T, d, V, s, st);
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
