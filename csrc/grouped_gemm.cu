// Grouped GEMM on the 5th-generation tensor cores for the MoE experts:
//
//   C[r, n] = sum_k A[r, k] * B_g[n, k]        for the rows r of group g   ("nt", forward)
//   C[r, n] = sum_k A[r, k] * B_g[k, n]        for the rows r of group g   ("nn", input gradient)
//
// A is one row-major bf16 buffer [R, K] whose rows are grouped (group g owns `counts[g]` rows
// starting at the sum of the previous counts — the receive layout of the expert exchange);
// every group has its own weight B_g (row-major [N, K] for "nt", [K, N] for "nn"; arbitrary
// address, one TMA tensor map per group in global memory); C is row-major [R, ldc].  For "nn"
// the B tile is K-rows x BN columns, loaded as BN/64 column chunks and fed to the MMA as an
// MN-major operand (no transpose pass).  The counts stay on the device, so no
// host synchronisation is needed to schedule the tiles.
//
// Persistent kernel, one CTA per SM, 6 warps:
//   warp 0      TMA producer: A tile [128 x 64] and B tile [BN x 64] per k-block, 128-byte
//               swizzle, a ring of kStages shared-memory stages (full/empty mbarriers).
//   warp 1      MMA issuer: tcgen05.mma kind::f16 (M = 128, N = BN, K = 16) into one of two
//               TMEM accumulators (2 x BN fp32 columns), so the epilogue of tile i overlaps the
//               MMAs of tile i + 1.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp owns its 32 TMEM lanes =
//               32 rows), bf16 conversion, masked 16-byte stores of the rows that belong to
//               the group.
// Tiles are (group, 128-row block, BN-column block) in that order; CTA b takes tiles
// b, b + grid, ...  Every mbarrier wait is bounded (common.cuh); on a timeout the kernel records
// a status code, stops issuing work, waits for its own copies and MMAs and frees TMEM.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "tma.cuh"

using namespace mimir;

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kMaxGroups = 256;

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kSmem = kStages * kStageBytes + 1024;  // + alignment slack
  static constexpr uint32_t kTmemCols = 2 * BN;
};

struct Bars {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t done;
  uint32_t tmem_base;
  int group_row[kMaxGroups + 1];   // first row of each group
  int group_tile[kMaxGroups + 1];  // first m-tile of each group
};

__device__ __forceinline__ int find_group(const Bars* b, int G, int mtile) {
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b->group_tile[mid] <= mtile) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <int BN, bool kBnMajor>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                       const CUtensorMap* __restrict__ maps_b,
                                                                       const int32_t* __restrict__ counts, int G,
                                                                       __nv_bfloat16* __restrict__ C, int64_t ldc,
                                                                       int N, int K, int* status) {
  using CF = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Bars bars;
  Bars* bar = &bars;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    int row = 0, tile = 0;
    for (int g = 0; g < G; ++g) {
      bar->group_row[g] = row;
      bar->group_tile[g] = tile;
      const int n = counts[g];
      row += n;
      tile += (n + kBM - 1) / kBM;
    }
    bar->group_row[G] = row;
    bar->group_tile[G] = tile;
    for (int s = 0; s < CF::kStages; ++s) {
      mbar_init(&bar->full[s], 1);
      mbar_init(&bar->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->acc_full[i], 1);
      mbar_init(&bar->acc_empty[i], 4);
    }
    mbar_init(&bar->done, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_base, CF::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&map_a);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  const int ntn = N / BN, nkb = K / kBK;
  const int total = bar->group_tile[G] * ntn;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        const int mt = t / ntn, n0 = (t % ntn) * BN;
        const int g = find_group(bar, G, mt);
        const int row0 = bar->group_row[g] + (mt - bar->group_tile[g]) * kBM;
        const CUtensorMap* mb = maps_b + g;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CF::kStages;
          if (it >= CF::kStages &&
              !mbar_wait(&bar->empty[s], ((it / CF::kStages) - 1) & 1, status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * CF::kStageBytes;
          mbar_arrive_expect_tx(&bar->full[s], CF::kStageBytes);
          tma_load_2d(sa, &map_a, &bar->full[s], kb * kBK, row0);
          if (kBnMajor) {  // B_g is [K, N]: BN/64 chunks of [64 k-rows x 64 n-columns]
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(sa + CF::kABytes + c * (kBK * 128), mb, &bar->full[s], n0 + c * 64, kb * kBK);
          } else {
            tma_load_2d(sa + CF::kABytes, mb, &bar->full[s], kb * kBK, n0);
          }
        }
      }
      // Teardown: every issued copy has landed before the CTA can exit.
      for (int j = max(0, it - CF::kStages); j < it; ++j)
        mbar_wait(&bar->full[j % CF::kStages], (j / CF::kStages) & 1, status, kStatusTimeoutKV);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kBM, BN, 0, kBnMajor ? 1 : 0);
      int it = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (i >= 2 && !mbar_wait(&bar->acc_empty[buf], ((i >> 1) - 1) & 1, status, kStatusTimeoutO)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CF::kStages;
          if (!mbar_wait(&bar->full[s], (it / CF::kStages) & 1, status, kStatusTimeoutKV)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * CF::kStageBytes);
          const uint32_t sb = sa + CF::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // K-major B: 16 k = 32 bytes along the swizzled row.  MN-major B: 16 k-rows = 2048
            // bytes; the 64-column chunks sit kBK*128 bytes apart (leading byte offset).
            const uint64_t bdesc = kBnMajor ? smem_desc(sb + kk * 2048, kBK * 128, 1024, kLayoutSW128)
                                            : smem_desc(sb + kk * 32, 16, 1024, kLayoutSW128);
            mma_bf16_ss(acc, smem_desc(sa + kk * 32, 16, 1024, kLayoutSW128), bdesc, idesc,
                        (kb | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&bar->empty[s]);  // the stage is free once these MMAs have read it
        }
        if (ok) mma_commit(&bar->acc_full[buf]);
      }
      // Teardown: every MMA issued by this thread completes before TMEM is released.
      mma_commit(&bar->done);
      mbar_wait(&bar->done, 0, status, kStatusTimeoutOther);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    int i = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
      const int buf = i & 1;
      if (!warp_wait(&bar->acc_full[buf], (i >> 1) & 1, status, kStatusTimeoutS)) break;
      tc_fence_after();
      const int mt = t / ntn, n0 = (t % ntn) * BN;
      const int g = find_group(bar, G, mt);
      const int m_in = (mt - bar->group_tile[g]) * kBM + r;
      const bool valid = m_in < counts[g];
      __nv_bfloat16* crow = C + int64_t(bar->group_row[g] + m_in) * ldc + n0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(tmem + lane_off + buf * BN + c * 32, v);
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(crow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                                pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, CF::kTmemCols);
  }
}

// Per-group B tensor maps, cached by (pointers, N, K, BN): expert weights keep their addresses
// across steps, so the maps are encoded and uploaded once.
struct MapCache {
  std::mutex mu;
  std::unordered_map<std::string, at::Tensor> maps;
};

MapCache& map_cache() {
  static MapCache c;
  return c;
}

at::Tensor group_maps(const std::vector<at::Tensor>& bs, int64_t N, int64_t K, int BN, bool bn_major,
                      const at::Device& dev) {
  std::string key = std::to_string(N) + "," + std::to_string(K) + "," + std::to_string(BN) + "," +
                    std::to_string(bn_major) + "," + std::to_string(dev.index());
  for (const auto& b : bs) key += "," + std::to_string(reinterpret_cast<uintptr_t>(b.data_ptr()));
  auto& cache = map_cache();
  std::lock_guard<std::mutex> lock(cache.mu);
  auto it = cache.maps.find(key);
  if (it != cache.maps.end()) return it->second;
  at::Tensor host = at::empty({static_cast<int64_t>(bs.size() * sizeof(CUtensorMap))},
                              at::TensorOptions().dtype(at::kByte).pinned_memory(true));
  auto* m = reinterpret_cast<CUtensorMap*>(host.data_ptr());
  for (size_t g = 0; g < bs.size(); ++g)
    m[g] = bn_major ? make_tmap_bf16_2d(bs[g].data_ptr(), K, N, N, 64, kBK)
                    : make_tmap_bf16_2d(bs[g].data_ptr(), N, K, K, kBK, BN);
  at::Tensor dev_maps = host.to(at::TensorOptions().device(dev), /*non_blocking=*/false);
  if (cache.maps.size() > 4096) cache.maps.clear();
  cache.maps.emplace(key, dev_maps);
  return dev_maps;
}

int* status_word(const at::Device& dev) {
  static int* words[64] = {nullptr};
  const int i = dev.index();
  if (words[i] == nullptr) {
    C10_CUDA_CHECK(cudaMalloc(&words[i], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(words[i], 0, sizeof(int)));
  }
  return words[i];
}

template <int BN, bool kBnMajor>
void launch(const CUtensorMap& ma, const at::Tensor& maps, const at::Tensor& counts, int G, at::Tensor& c, int N, int K,
            int* status, cudaStream_t st, int sms) {
  using CF = Cfg<BN>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(grouped_gemm_kernel<BN, kBnMajor>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kSmem));
    attr = true;
  }
  grouped_gemm_kernel<BN, kBnMajor><<<sms, kThreads, CF::kSmem, st>>>(
      ma, reinterpret_cast<const CUtensorMap*>(maps.data_ptr()), counts.data_ptr<int32_t>(), G,
      reinterpret_cast<__nv_bfloat16*>(c.data_ptr()), c.stride(0), N, K, status);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------------------------
// Weight gradients: for every group g,  W_g[m, n] += sum_{r in g} A[r, m] * B[r, n]
// (A = the output gradient rows of the group, B = the input rows).  The reduction runs over the
// group's rows, so each group has its own pair of TMA maps whose row extent is the group's row
// count: the tail k-block reads zeros past the group's end (TMA out-of-bounds fill) instead of
// the next group's rows.  Both operands are MN-major tiles ([64 rows x 64 columns] chunks); the
// epilogue adds the fp32 accumulator to the bf16 weight gradient in place.
struct WgradGroup {
  CUtensorMap a;     // [rows_g, M] window of A
  CUtensorMap b;     // [rows_g, N] window of B
  uint64_t out;      // W_g gradient, contiguous bf16 [M, N]
  int32_t kblocks;   // ceil(rows_g / 64)
  int32_t pad[13];
};
static_assert(sizeof(WgradGroup) % 64 == 0, "tensor maps must stay 64-byte aligned");

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) grouped_wgrad_kernel(const WgradGroup* __restrict__ groups, int G,
                                                                      int M, int N, int* status) {
  using CF = Cfg<BN>;
  constexpr int kABytes = kBK * kBM * 2;  // [64 rows x 128 m] as two 64-column chunks
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Bars bars;
  Bars* bar = &bars;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < CF::kStages; ++s) {
      mbar_init(&bar->full[s], 1);
      mbar_init(&bar->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->acc_full[i], 1);
      mbar_init(&bar->acc_empty[i], 4);
    }
    mbar_init(&bar->done, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_base, CF::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  const int ntm = M / kBM, ntn = N / BN;
  const int per_group = ntm * ntn;
  const int total = G * per_group;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        const WgradGroup* gr = groups + t / per_group;
        const int m0 = ((t % per_group) / ntn) * kBM, n0 = (t % ntn) * BN;
        for (int kb = 0; kb < gr->kblocks; ++kb, ++it) {
          const int s = it % CF::kStages;
          if (it >= CF::kStages &&
              !mbar_wait(&bar->empty[s], ((it / CF::kStages) - 1) & 1, status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * CF::kStageBytes;
          mbar_arrive_expect_tx(&bar->full[s], CF::kStageBytes);
#pragma unroll
          for (int c = 0; c < kBM / 64; ++c) tma_load_2d(sa + c * (kBK * 128), &gr->a, &bar->full[s], m0 + c * 64, kb * kBK);
#pragma unroll
          for (int c = 0; c < BN / 64; ++c)
            tma_load_2d(sa + kABytes + c * (kBK * 128), &gr->b, &bar->full[s], n0 + c * 64, kb * kBK);
        }
      }
      for (int j = max(0, it - CF::kStages); j < it; ++j)
        mbar_wait(&bar->full[j % CF::kStages], (j / CF::kStages) & 1, status, kStatusTimeoutKV);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kBM, BN, 1, 1);
      int it = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++i) {
        const int buf = i & 1;
        const int nkb = groups[t / per_group].kblocks;
        if (i >= 2 && !mbar_wait(&bar->acc_empty[buf], ((i >> 1) - 1) & 1, status, kStatusTimeoutO)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CF::kStages;
          if (!mbar_wait(&bar->full[s], (it / CF::kStages) & 1, status, kStatusTimeoutKV)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * CF::kStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16_ss(acc, smem_desc(sa + kk * 2048, kBK * 128, 1024, kLayoutSW128),
                        smem_desc(sb + kk * 2048, kBK * 128, 1024, kLayoutSW128), idesc, (kb | kk) != 0 ? 1u : 0u);
          mma_commit(&bar->empty[s]);
        }
        if (ok) mma_commit(&bar->acc_full[buf]);
      }
      mma_commit(&bar->done);
      mbar_wait(&bar->done, 0, status, kStatusTimeoutOther);
    }
  } else {
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    int i = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
      const int buf = i & 1;
      if (!warp_wait(&bar->acc_full[buf], (i >> 1) & 1, status, kStatusTimeoutS)) break;
      tc_fence_after();
      const WgradGroup* gr = groups + t / per_group;
      const int m0 = ((t % per_group) / ntn) * kBM, n0 = (t % ntn) * BN;
      __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(gr->out) + int64_t(m0 + r) * N + n0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(tmem + lane_off + buf * BN + c * 32, v);
        uint4* dst = reinterpret_cast<uint4*>(row + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 old = dst[q];
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&old);
          float o[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h[e]);
            o[2 * e] = f.x + v[8 * q + 2 * e];
            o[2 * e + 1] = f.y + v[8 * q + 2 * e + 1];
          }
          dst[q] = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                              pack_bf16x2(o[6], o[7]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, CF::kTmemCols);
  }
}

// One launch of the weight-gradient kernel; the shared-memory attribute is set once per
// instantiation (each BN has its own flag).
template <int BN>
void launch_wgrad(const WgradGroup* groups, int G, int64_t M, int64_t N, int* status, cudaStream_t st, int sms) {
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(grouped_wgrad_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        Cfg<BN>::kSmem));
    attr = true;
  }
  grouped_wgrad_kernel<BN><<<sms, kThreads, Cfg<BN>::kSmem, st>>>(groups, G, static_cast<int>(M), static_cast<int>(N),
                                                                  status);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

// out[rows, :N] = a[rows, :K] @ b_g^T ("nt": b_g is [N, K]) or a[rows, :K] @ b_g ("nn": b_g is
// [K, N]) for the row blocks given by `counts` (int32 on the device).  `out` may be a view with a
// row stride (e.g. one half of a peer-visible buffer).
void grouped_gemm(at::Tensor a, std::vector<at::Tensor> bs, at::Tensor counts, at::Tensor out, bool b_kn) {
  TORCH_CHECK(a.is_cuda() && a.dtype() == at::kBFloat16 && a.dim() == 2 && a.stride(1) == 1, "a: bf16 [R, K]");
  TORCH_CHECK(out.is_cuda() && out.dtype() == at::kBFloat16 && out.dim() == 2 && out.stride(1) == 1,
              "out: bf16 [R, N] with unit column stride");
  const int G = static_cast<int>(bs.size());
  TORCH_CHECK(G >= 1 && G <= kMaxGroups, "1..", kMaxGroups, " groups");
  TORCH_CHECK(counts.is_cuda() && counts.dtype() == at::kInt && counts.numel() == G, "counts: int32 [G] on device");
  const int64_t K = a.size(1), N = b_kn ? bs[0].size(1) : bs[0].size(0);
  for (const auto& b : bs)
    TORCH_CHECK(b.is_cuda() && b.dtype() == at::kBFloat16 && b.is_contiguous() && b.dim() == 2 &&
                    (b_kn ? (b.size(0) == K && b.size(1) == N) : (b.size(0) == N && b.size(1) == K)),
                "every group weight: contiguous bf16 ", b_kn ? "[K, N]" : "[N, K]");
  TORCH_CHECK(K % kBK == 0 && N % 128 == 0, "K must be a multiple of 64 and N of 128");
  TORCH_CHECK(out.size(1) >= N && out.size(0) >= a.size(0), "out too small");
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (out.stride(0) * 2) % 16 == 0, "row strides must be 16-byte multiples");
  const c10::cuda::CUDAGuard guard(a.device());
  if (a.size(0) == 0) return;
  const int BN = N % 256 == 0 ? 256 : 128;
  const CUtensorMap ma = make_tmap_bf16_2d(a.data_ptr(), a.size(0), K, a.stride(0), kBK, kBM);
  at::Tensor maps = group_maps(bs, N, K, BN, b_kn, a.device());
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, a.device().index()));
  auto st = at::cuda::getCurrentCUDAStream();
  int* status = status_word(a.device());
  if (BN == 256) {
    if (b_kn) launch<256, true>(ma, maps, counts, G, out, N, K, status, st, sms);
    else launch<256, false>(ma, maps, counts, G, out, N, K, status, st, sms);
  } else {
    if (b_kn) launch<128, true>(ma, maps, counts, G, out, N, K, status, st, sms);
    else launch<128, false>(ma, maps, counts, G, out, N, K, status, st, sms);
  }
}


// grads[g] += a_g^T @ b_g for the row blocks given by the host list `rows` (a: [R, M], b: [R, N],
// bf16, rows grouped in order; grads: contiguous bf16 [M, N]).  Groups without rows are skipped.
void grouped_wgrad(at::Tensor a, at::Tensor b, std::vector<int64_t> rows, std::vector<at::Tensor> grads) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.dtype() == at::kBFloat16 && b.dtype() == at::kBFloat16 && a.dim() == 2 &&
                  b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 && a.size(0) == b.size(0),
              "a, b: bf16 [R, M], [R, N] with unit column stride");
  TORCH_CHECK(rows.size() == grads.size(), "one row count per gradient");
  const int64_t M = a.size(1), N = b.size(1);
  TORCH_CHECK(M % kBM == 0 && N % 128 == 0, "M must be a multiple of 128 and N of 128");
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0, "row strides must be 16-byte multiples");
  const c10::cuda::CUDAGuard guard(a.device());
  const int BN = N % 256 == 0 ? 256 : 128;
  std::vector<WgradGroup> host;
  int64_t row = 0;
  for (size_t g = 0; g < rows.size(); ++g) {
    const auto& w = grads[g];
    TORCH_CHECK(w.is_cuda() && w.dtype() == at::kBFloat16 && w.is_contiguous() && w.size(0) == M && w.size(1) == N,
                "gradient ", g, ": contiguous bf16 [M, N]");
    const int64_t n = rows[g];
    if (n > 0) {
      WgradGroup gr{};
      const auto* ab = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()) + row * a.stride(0);
      const auto* bb = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()) + row * b.stride(0);
      gr.a = make_tmap_bf16_2d(ab, n, M, a.stride(0), 64, kBK);
      gr.b = make_tmap_bf16_2d(bb, n, N, b.stride(0), 64, kBK);
      gr.out = reinterpret_cast<uint64_t>(w.data_ptr());
      gr.kblocks = static_cast<int32_t>((n + kBK - 1) / kBK);
      host.push_back(gr);
    }
    row += n;
  }
  TORCH_CHECK(row <= a.size(0), "row counts exceed the buffers");
  if (host.empty()) return;
  const int64_t nbytes = static_cast<int64_t>(host.size() * sizeof(WgradGroup));
  at::Tensor pinned = at::empty({nbytes}, at::TensorOptions().dtype(at::kByte).pinned_memory(true));
  std::memcpy(pinned.data_ptr(), host.data(), nbytes);
  at::Tensor dev = pinned.to(at::TensorOptions().device(a.device()), /*non_blocking=*/true);
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, a.device().index()));
  auto st = at::cuda::getCurrentCUDAStream();
  int* status = status_word(a.device());
  const int G = static_cast<int>(host.size());
  const auto* groups = reinterpret_cast<const WgradGroup*>(dev.data_ptr());
  if (BN == 256) launch_wgrad<256>(groups, G, M, N, status, st, sms);
  else launch_wgrad<128>(groups, G, M, N, status, st, sms);
}

int64_t grouped_gemm_status(int64_t device) {
  int v = 0;
  int* w = status_word(at::Device(at::kCUDA, static_cast<c10::DeviceIndex>(device)));
  C10_CUDA_CHECK(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}
