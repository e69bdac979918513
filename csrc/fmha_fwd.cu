// Single-pass prefix-LM flash attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// One CTA computes a 128-row query tile of one head (head_dim 128) of one packed
// sequence.  Mask: a query row at sequence position r sees keys [0, P) if r < P (the
// bidirectional prompt) and keys [0, r] otherwise (P = 0 for plain causal attention).
// Key blocks past the tile's largest row limit are never loaded; blocks below its smallest
// limit run unmasked.
//
// Warp roles (192 threads, 1 CTA/SM):
//   warp 0      TMA producer: Q once, then K_j / V_j into a 2-stage ring.
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer:
//                 S_j = Q K_j^T  -> TMEM (two ping-pong S buffers of 128 fp32 columns)
//                 O  += P_j V_j  -> TMEM (128 fp32 columns); P_j is read from shared memory
//   warps 2..5  softmax: thread = query row.  Online softmax in the log2 domain with lazy
//               O rescaling (only when the running max grows by more than 2^8), bf16 P
//               written into a 128B-swizzled K-major smem tile, and the epilogue
//               (O / l, optional sigmoid(gate) multiply, LSE).
// The MMA stream is S_0, S_1, PV_0, S_2, PV_1, ...: the tensor core computes S_{j+1}
// while the softmax warps turn S_j into P_j.
//
// All mbarrier waits are bounded (see common.cuh); a timeout records a status code and
// every role falls through to the teardown, which waits for in-flight async work and
// frees TMEM.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>

#include "common.cuh"
#include "fmha_noalloc.h"
#include "tma.cuh"

using namespace mimir;

namespace {

constexpr int kTile = 128;       // query rows per CTA, keys per block
constexpr int kHeadDim = 128;
constexpr int kThreads = 192;
constexpr uint32_t kTileBytes = kTile * kHeadDim * 2;  // 32 KB
constexpr uint32_t kChunkBytes = kTileBytes / 2;       // 64-column half: 16 KB
constexpr float kRescaleThreshold = 8.0f;              // log2 units
#ifndef MIMIR_FMHA_POLY_EVERY
#define MIMIR_FMHA_POLY_EVERY 4
#endif
constexpr int kPolyEvery = MIMIR_FMHA_POLY_EVERY;      // 0: every exponential on the MUFU pipe

struct FwdParams {
  __nv_bfloat16* y;            // [T, H*128] output (gated when gate != nullptr)
  __nv_bfloat16* o;            // optional ungated output [T, H*128]
  const __nv_bfloat16* gate;   // optional gate base (row stride gate_ld), head h at column gate_col + h*128
  int64_t gate_ld;
  int gate_col;
  float* lse;                  // [H, lse_ld], log2-domain log-sum-exp of scaled scores
  int64_t lse_ld;
  const int* cu_seqlens;
  const int* prefix_lens;
  const int2* tiles;
  const int* ntiles;
  int H, KV;
  int q_col, k_col, v_col;     // column offsets (elements) of head 0 inside each TMA tensor
  int is_causal;
  float scale_log2;
  int* status;
};

struct __align__(8) Barriers {
  uint64_t q_full;
  uint64_t k_full[2];
  uint64_t v_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full;
  uint64_t o_done;
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

constexpr uint32_t kSmemQ = 0;
constexpr uint32_t kSmemK0 = kTileBytes;                  // K stage s at kSmemK0 + s*2*kTileBytes
constexpr uint32_t kSmemP = kTileBytes * 5;               // after Q + 2 x (K, V)
constexpr uint32_t kSmemBar = kTileBytes * 6;
constexpr uint32_t kSmemBytes = kSmemBar + sizeof(Barriers) + 1024;  // + alignment slack

__device__ __forceinline__ uint8_t* k_stage(uint8_t* base, int s) { return base + kSmemK0 + s * 2 * kTileBytes; }
__device__ __forceinline__ uint8_t* v_stage(uint8_t* base, int s) { return k_stage(base, s) + kTileBytes; }

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bar = reinterpret_cast<Barriers*>(smem + kSmemBar);

  const int tile = blockIdx.y;
  if (tile >= *p.ntiles) return;  // CTA-uniform, before any allocation
  const int h = blockIdx.x;
  const int2 tq = p.tiles[tile];
  const int seq = tq.x;
  const int q0 = tq.y * kTile;
  const int start = p.cu_seqlens[seq];
  const int L = p.cu_seqlens[seq + 1] - start;
  const int P = p.is_causal ? 0 : p.prefix_lens[seq];
  const int last_row = min(q0 + kTile - 1, L - 1);
  const int max_lim = last_row >= P ? last_row : P - 1;
  const int min_lim = q0 < P ? P - 1 : q0;
  const int nkv = max_lim / kTile + 1;
  const int kvh = h / (p.H / p.KV);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->kv_empty[s], 1);
      mbar_init(&bar->s_full[s], 1);
      mbar_init(&bar->s_free[s], 4);
    }
    mbar_init(&bar->p_full, 4);
    mbar_init(&bar->o_done, 1);
    mbar_init(&bar->mma_done, 1);
    bar->abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_base, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  auto tS = [tmem](int s) -> uint32_t { return s ? tmem + 128 : tmem; };
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int qx = p.q_col + h * kHeadDim;
      const int kx = p.k_col + kvh * kHeadDim;
      const int vx = p.v_col + kvh * kHeadDim;
      mbar_arrive_expect_tx(&bar->q_full, kTileBytes);
      tma_load_2d(smem + kSmemQ, &map_q, &bar->q_full, qx, start + q0);
      tma_load_2d(smem + kSmemQ + kChunkBytes, &map_q, &bar->q_full, qx + 64, start + q0);
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&bar->kv_empty[s], ((j >> 1) - 1) & 1, p.status, kStatusTimeoutEmpty)) {
          bar->abort = 1;
          break;
        }
        const int row = start + j * kTile;
        mbar_arrive_expect_tx(&bar->k_full[s], kTileBytes);
        tma_load_2d(k_stage(smem, s), &map_k, &bar->k_full[s], kx, row);
        tma_load_2d(k_stage(smem, s) + kChunkBytes, &map_k, &bar->k_full[s], kx + 64, row);
        mbar_arrive_expect_tx(&bar->v_full[s], kTileBytes);
        tma_load_2d(v_stage(smem, s), &map_v, &bar->v_full[s], vx, row);
        tma_load_2d(v_stage(smem, s) + kChunkBytes, &map_v, &bar->v_full[s], vx + 64, row);
        issued = j + 1;
      }
      // Teardown: make sure no TMA write into this CTA's smem is still in flight.
      mbar_wait(&bar->q_full, 0, p.status, kStatusTimeoutQ);
      for (int j = max(0, issued - 2); j < issued; ++j) {
        mbar_wait(&bar->k_full[j & 1], (j >> 1) & 1, p.status, kStatusTimeoutKV);
        mbar_wait(&bar->v_full[j & 1], (j >> 1) & 1, p.status, kStatusTimeoutKV);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qk = idesc_bf16_f32(128, 128, 0, 0);
      const uint32_t idesc_pv = idesc_bf16_f32(128, 128, 0, 1);
      const uint32_t sq = smem_u32(smem + kSmemQ);
      const uint32_t sp = smem_u32(smem + kSmemP);
      bool ok = mbar_wait(&bar->q_full, 0, p.status, kStatusTimeoutQ);
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait(&bar->p_full, i & 1, p.status, kStatusTimeoutP)) return false;
        if (!mbar_wait(&bar->v_full[i & 1], (i >> 1) & 1, p.status, kStatusTimeoutKV)) return false;
        tc_fence_after();
        const uint32_t sv = smem_u32(v_stage(smem, i & 1));
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          // A = P (K-major, 128B swizzle): 16 kv columns = 32 bytes within a 64-column chunk.
          const uint64_t a = smem_desc(sp + (k >> 2) * kChunkBytes + (k & 3) * 32, 16, 1024, kLayoutSW128);
          // B = V (MN-major over head_dim): 16 kv rows = 2048 bytes; the second 64-wide
          // head_dim chunk sits 16 KB further (LBO).
          const uint64_t b = smem_desc(sv + k * 2048, kChunkBytes, 1024, kLayoutSW128);
          mma_ss(tO, a, b, idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&bar->o_done);
        mma_commit(&bar->kv_empty[i & 1]);
        return true;
      };
      for (int j = 0; ok && j < nkv; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&bar->k_full[s], (j >> 1) & 1, p.status, kStatusTimeoutKV)) { ok = false; break; }
        if (j >= 2 && !mbar_wait(&bar->s_free[s], ((j >> 1) - 1) & 1, p.status, kStatusTimeoutS)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sk = smem_u32(k_stage(smem, s));
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kChunkBytes + (k & 3) * 32;
          mma_ss(tS(s), smem_desc(sq + off, 16, 1024, kLayoutSW128), smem_desc(sk + off, 16, 1024, kLayoutSW128),
                 idesc_qk, k > 0 ? 1u : 0u);
        }
        mma_commit(&bar->s_full[s]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(nkv - 1);
      if (!ok) bar->abort = 1;
      // Teardown: wait for every MMA issued by this thread before TMEM is released.
      mma_commit(&bar->mma_done);
      mbar_wait(&bar->mma_done, 0, p.status, kStatusTimeoutOther);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int wq = warp & 3;                 // TMEM lane quarter accessible by this warp
    const int r = wq * 32 + lane;            // query row within the tile
    const int qpos = q0 + r;
    const int lim = qpos < P ? P - 1 : qpos;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    float m_i = -INFINITY, l_i = 0.f;
    const uint32_t sP_addr = smem_u32(smem + kSmemP);
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int s = j & 1;
      if (!warp_wait(&bar->s_full[s], (j >> 1) & 1, p.status, kStatusTimeoutS)) { ok = false; break; }
      tc_fence_after();
      float sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float part[32];
        tmem_ld32(tS(s) + lane_off + c * 32, part);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = part[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->s_free[s]);

      const int k0 = j * kTile;
      if (k0 + kTile - 1 > min_lim) {
        const int rel = lim - k0;  // keys with column index > rel are masked
#pragma unroll
        for (int c = 0; c < 128; ++c) sv[c] = c > rel ? -INFINITY : sv[c];
      }
      float mxp[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mxp[e] = sv[e];
#pragma unroll
      for (int c = 8; c < 128; c += 8) {
#pragma unroll
        for (int e = 0; e < 8; ++e) mxp[e] = fmaxf(mxp[e], sv[c + e]);
      }
      float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                       fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
      mx *= p.scale_log2;
      float m_use = m_i, alpha = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_use = mx;
      } else if (mx > m_i + kRescaleThreshold) {
        m_use = mx;
        alpha = fast_exp2(m_i - mx);
        rescale = true;
      }
      float sums[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        // Every kPolyEvery-th pair takes the FMA-pipe exponential so the MUFU pipe is not the
        // only exp2 unit in use.
        const bool poly = kPolyEvery > 0 && (c % kPolyEvery) == kPolyEvery - 1;
        const float xa = fmaf(sv[2 * c], p.scale_log2, -m_use), xb = fmaf(sv[2 * c + 1], p.scale_log2, -m_use);
        const float a = poly ? poly_exp2(xa) : fast_exp2(xa);
        const float b = poly ? poly_exp2(xb) : fast_exp2(xb);
        sums[c & 7] += a + b;
        pk[c] = pack_bf16x2(a, b);
      }
      const float rowsum = ((sums[0] + sums[1]) + (sums[2] + sums[3])) + ((sums[4] + sums[5]) + (sums[6] + sums[7]));
      l_i = l_i * alpha + rowsum;
      m_i = m_use;

      if (j > 0) {
        if (!warp_wait(&bar->o_done, (j - 1) & 1, p.status, kStatusTimeoutO)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffff, rescale)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float ov[32];
            tmem_ld32(tO + lane_off + c * 32, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= alpha;
            tmem_st32(tO + lane_off + c * 32, ov);
          }
          tmem_wait_st();
        }
      }
      // P row r -> 128B-swizzled K-major tile: chunk (64 keys) c, 16-byte unit u at (u ^ (r & 7)).
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int chunk = u >> 3, unit = u & 7;
        st_shared_v4(sP_addr + chunk * kChunkBytes + r * 128 + ((unit ^ (r & 7)) << 4), pk[4 * u], pk[4 * u + 1],
                     pk[4 * u + 2], pk[4 * u + 3]);
      }
      fence_async_shared();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->p_full);
    }
    if (ok && warp_wait(&bar->o_done, (nkv - 1) & 1, p.status, kStatusTimeoutO)) {
      tc_fence_after();
      const bool valid = qpos < L;
      const int64_t grow = (int64_t)start + qpos;
      const float inv_l = 1.f / l_i;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(tO + lane_off + c * 32, ov);
        if (valid) {
          const int64_t col = (int64_t)h * kHeadDim + c * 32;
          float gv[32];
          if (p.gate != nullptr) {
            const uint4* g = reinterpret_cast<const uint4*>(p.gate + grow * p.gate_ld + p.gate_col + col);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 u = g[v];
              const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                float2 f = __bfloat1622float2(hv[i]);
                gv[v * 8 + 2 * i] = 1.f / (1.f + __expf(-f.x));
                gv[v * 8 + 2 * i + 1] = 1.f / (1.f + __expf(-f.y));
              }
            }
          }
          uint4* yo = reinterpret_cast<uint4*>(p.y + grow * (int64_t)p.H * kHeadDim + col);
          uint4* oo = p.o != nullptr ? reinterpret_cast<uint4*>(p.o + grow * (int64_t)p.H * kHeadDim + col) : nullptr;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            float a[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = ov[v * 8 + i] * inv_l;
            if (oo != nullptr)
              oo[v] = make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]), pack_bf16x2(a[4], a[5]),
                                 pack_bf16x2(a[6], a[7]));
            if (p.gate != nullptr) {
#pragma unroll
              for (int i = 0; i < 8; ++i) a[i] *= gv[v * 8 + i];
            }
            yo[v] = make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]), pack_bf16x2(a[4], a[5]),
                               pack_bf16x2(a[6], a[7]));
          }
        }
      }
      if (valid) p.lse[(int64_t)h * p.lse_ld + grow] = m_i + __log2f(l_i);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Tile schedule: (sequence, query block) pairs ordered by decreasing key-block count, so
// the longest tiles start first.  One CTA; counting sort over key-block counts.
constexpr int kMaxBuckets = 1024;

__global__ void build_tiles_kernel(const int* __restrict__ cu, const int* __restrict__ prefix, int nseq, int is_causal,
                                   int2* __restrict__ tiles, int* __restrict__ ntiles, int max_tiles) {
  __shared__ int hist[kMaxBuckets];
  __shared__ int total;
  for (int i = threadIdx.x; i < kMaxBuckets; i += blockDim.x) hist[i] = 0;
  if (threadIdx.x == 0) total = 0;
  __syncthreads();
  auto work = [&](int s, int qb) {
    const int L = cu[s + 1] - cu[s];
    const int P = is_causal ? 0 : prefix[s];
    const int last = min(qb * kTile + kTile - 1, L - 1);
    const int mx = last >= P ? last : P - 1;
    return min(mx / kTile + 1, kMaxBuckets) - 1;
  };
  for (int s = threadIdx.x; s < nseq; s += blockDim.x) {
    const int L = cu[s + 1] - cu[s];
    const int nq = (L + kTile - 1) / kTile;
    for (int qb = 0; qb < nq; ++qb) atomicAdd(&hist[work(s, qb)], 1);
    atomicAdd(&total, nq);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;  // descending work order
    for (int b = kMaxBuckets - 1; b >= 0; --b) {
      const int c = hist[b];
      hist[b] = acc;
      acc += c;
    }
    *ntiles = min(total, max_tiles);
  }
  __syncthreads();
  for (int s = threadIdx.x; s < nseq; s += blockDim.x) {
    const int L = cu[s + 1] - cu[s];
    const int nq = (L + kTile - 1) / kTile;
    for (int qb = 0; qb < nq; ++qb) {
      const int pos = atomicAdd(&hist[work(s, qb)], 1);
      if (pos < max_tiles) tiles[pos] = make_int2(s, qb);
    }
  }
}

int* status_word(const at::Device& dev) {
  static at::Tensor words[16];
  const int idx = dev.index();
  if (!words[idx].defined()) words[idx] = at::zeros({1}, at::TensorOptions().device(dev).dtype(at::kInt));
  return words[idx].data_ptr<int>();
}

}  // namespace

int* fmha_status_ptr(const at::Device& dev) { return status_word(dev); }

// Returns (tiles, ntiles) for a packed batch; reused across layers of one forward.
std::vector<at::Tensor> fmha_plan(at::Tensor cu_seqlens, at::Tensor prefix_lens, int64_t numseqs, int64_t total_tokens,
                                  bool is_causal) {
  TORCH_CHECK(cu_seqlens.is_cuda() && cu_seqlens.scalar_type() == at::kInt);
  TORCH_CHECK(prefix_lens.scalar_type() == at::kInt);
  c10::cuda::CUDAGuard guard(cu_seqlens.device());
  const int64_t max_tiles = (total_tokens + kTile - 1) / kTile + numseqs;
  auto tiles = at::empty({std::max<int64_t>(max_tiles, 1), 2}, cu_seqlens.options());
  auto ntiles = at::zeros({1}, cu_seqlens.options());
  if (numseqs > 0) {
    build_tiles_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
        cu_seqlens.data_ptr<int>(), prefix_lens.data_ptr<int>(), (int)numseqs, is_causal ? 1 : 0,
        reinterpret_cast<int2*>(tiles.data_ptr<int>()), ntiles.data_ptr<int>(), (int)max_tiles);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {tiles, ntiles};
}

// y (and optionally o) = attention for every head; q/k/v are column windows of 2-D bf16
// tensors.  Returns {y, lse, o?}.
std::vector<at::Tensor> fmha_fwd(at::Tensor q_src, int64_t q_col, at::Tensor k_src, int64_t k_col, at::Tensor v_src,
                                 int64_t v_col, c10::optional<at::Tensor> gate_src, int64_t gate_col, int64_t H,
                                 int64_t KV, bool is_causal, at::Tensor cu_seqlens, at::Tensor prefix_lens,
                                 int64_t numseqs, at::Tensor tiles, at::Tensor ntiles) {
  for (const at::Tensor* t : {&q_src, &k_src, &v_src}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 2 && t->stride(1) == 1,
                "fmha_fwd: q/k/v sources must be 2-D bf16 row-major CUDA tensors");
  }
  TORCH_CHECK(H % KV == 0, "fmha_fwd: H must be a multiple of KV");
  TORCH_CHECK(q_col % 8 == 0 && k_col % 8 == 0 && v_col % 8 == 0, "fmha_fwd: column offsets must be 16-byte aligned");
  c10::cuda::CUDAGuard guard(q_src.device());
  const int64_t T = q_src.size(0);
  auto opts = q_src.options();
  auto y = at::empty({T, H * kHeadDim}, opts);
  const bool gated = gate_src.has_value();
  at::Tensor o = gated ? at::empty({T, H * kHeadDim}, opts) : at::Tensor();
  const int64_t lse_ld = ((T + 127) / 128) * 128;
  auto lse = at::empty({H, lse_ld}, opts.dtype(at::kFloat));
  if (T == 0 || numseqs == 0) return gated ? std::vector<at::Tensor>{y, lse, o} : std::vector<at::Tensor>{y, lse};

  CUtensorMap mq = make_tmap_bf16_2d(q_src.data_ptr(), T, q_src.size(1), q_src.stride(0), 64, kTile);
  CUtensorMap mk = make_tmap_bf16_2d(k_src.data_ptr(), T, k_src.size(1), k_src.stride(0), 64, kTile);
  CUtensorMap mv = make_tmap_bf16_2d(v_src.data_ptr(), T, v_src.size(1), v_src.stride(0), 64, kTile);

  FwdParams prm{};
  prm.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  prm.o = gated ? reinterpret_cast<__nv_bfloat16*>(o.data_ptr()) : nullptr;
  if (gated) {
    TORCH_CHECK(gate_src->stride(1) == 1 && gate_src->scalar_type() == at::kBFloat16);
    prm.gate = reinterpret_cast<const __nv_bfloat16*>(gate_src->data_ptr());
    prm.gate_ld = gate_src->stride(0);
    prm.gate_col = (int)gate_col;
  }
  prm.lse = lse.data_ptr<float>();
  prm.lse_ld = lse_ld;
  prm.cu_seqlens = cu_seqlens.data_ptr<int>();
  prm.prefix_lens = prefix_lens.data_ptr<int>();
  prm.tiles = reinterpret_cast<const int2*>(tiles.data_ptr<int>());
  prm.ntiles = ntiles.data_ptr<int>();
  prm.H = (int)H;
  prm.KV = (int)KV;
  prm.q_col = (int)q_col;
  prm.k_col = (int)k_col;
  prm.v_col = (int)v_col;
  prm.is_causal = is_causal ? 1 : 0;
  prm.scale_log2 = 1.4426950408889634f / sqrtf((float)kHeadDim);
  prm.status = status_word(q_src.device());

  static bool attr_set[16] = {false};
  if (!attr_set[q_src.device().index()]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(fmha_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    attr_set[q_src.device().index()] = true;
  }
  dim3 grid((unsigned)H, (unsigned)tiles.size(0));
  fmha_fwd_kernel<<<grid, kThreads, kSmemBytes, at::cuda::getCurrentCUDAStream()>>>(mq, mk, mv, prm);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return gated ? std::vector<at::Tensor>{y, lse, o} : std::vector<at::Tensor>{y, lse};
}

// Reads and clears the device status word of the attention kernels (0 = ok).
int64_t fmha_status(at::Device dev) {
  int* w = status_word(dev);
  int host = 0;
  C10_CUDA_CHECK(cudaMemcpy(&host, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (host != 0) C10_CUDA_CHECK(cudaMemset(w, 0, sizeof(int)));
  return host;
}

// ---------------------------------------------------------------------------------------------
// Allocation-free entry point (declared in fmha_noalloc.h; no counterpart in the reference).
// Scratch lives in file-scope device arrays; host code only ever passes the addresses that
// cudaGetSymbolAddress returns for the current device.
namespace {
static __device__ __align__(256) int2 g_noalloc_tiles[MIMIR_FMHA_NOALLOC_MAX_TILES];
// [0] tile count (rewritten by every call's schedule kernel), [1] kernel status: the first
// bounded-wait timeout of any call since the last mimir_fmha_noalloc_status() read.
static __device__ __align__(256) int g_noalloc_words[64];

struct NoAllocScratch {
  int2* tiles = nullptr;
  int* words = nullptr;
  bool ready = false;
};
NoAllocScratch g_scratch[64];
std::mutex g_noalloc_setup_mu;  // two host threads making their first call at once

// Once per device, with that device current: look up the scratch addresses and raise the
// kernel's dynamic shared-memory limit.
int noalloc_setup(int device) {
  if (device < 0 || device >= 64) return MIMIR_NOALLOC_ERR_ARGS;
  std::lock_guard<std::mutex> lock(g_noalloc_setup_mu);
  NoAllocScratch& s = g_scratch[device];
  if (s.ready) return MIMIR_NOALLOC_OK;
  int2* tiles = nullptr;
  int* words = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&tiles), g_noalloc_tiles) != cudaSuccess)
    return MIMIR_NOALLOC_ERR_CUDA;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&words), g_noalloc_words) != cudaSuccess)
    return MIMIR_NOALLOC_ERR_CUDA;
  if (cudaFuncSetAttribute(fmha_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
    return MIMIR_NOALLOC_ERR_CUDA;
  s.tiles = tiles;
  s.words = words;
  s.ready = true;
  return MIMIR_NOALLOC_OK;
}

bool make_tmap_noexcept(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || (ld * 2) % 16 != 0) return false;
  bind_device_context();  // the encoder needs a current context (first call on a new host thread)
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)kTile};
  cuuint32_t estr[2] = {1, 1};
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || fn == nullptr)
    return false;
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

extern "C" int mimir_fmha_fwd_noalloc(const void* q, int64_t q_ld, const void* k, int64_t k_ld, const void* v,
                                      int64_t v_ld, void* out, float* lse, int64_t lse_ld, const int* cu_seqlens,
                                      const int* prefix_lens, int numseqs, int64_t total_tokens, int num_heads,
                                      int num_kv_heads, int is_causal, cudaStream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || lse == nullptr || cu_seqlens == nullptr ||
      (prefix_lens == nullptr && !is_causal) || numseqs < 0 || total_tokens < 0 || num_heads <= 0 ||
      num_kv_heads <= 0 || num_heads % num_kv_heads != 0 || lse_ld < total_tokens ||
      q_ld < (int64_t)num_heads * kHeadDim || k_ld < (int64_t)num_kv_heads * kHeadDim ||
      v_ld < (int64_t)num_kv_heads * kHeadDim)
    return MIMIR_NOALLOC_ERR_ARGS;
  // The kernel stores `out` in 16-byte vectors and `lse` as fp32; the schedule reads int32.
  if (reinterpret_cast<uintptr_t>(out) % 16 != 0 || reinterpret_cast<uintptr_t>(lse) % 4 != 0 ||
      reinterpret_cast<uintptr_t>(cu_seqlens) % 4 != 0 ||
      (prefix_lens != nullptr && reinterpret_cast<uintptr_t>(prefix_lens) % 4 != 0))
    return MIMIR_NOALLOC_ERR_ARGS;
  if (total_tokens == 0 || numseqs == 0) return MIMIR_NOALLOC_OK;
  const int64_t max_tiles = (total_tokens + kTile - 1) / kTile + numseqs;
  if (max_tiles > MIMIR_FMHA_NOALLOC_MAX_TILES || max_tiles > 65535) return MIMIR_NOALLOC_ERR_TOO_LARGE;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return MIMIR_NOALLOC_ERR_CUDA;
  const int rc = noalloc_setup(device);
  if (rc != MIMIR_NOALLOC_OK) return rc;
  NoAllocScratch& s = g_scratch[device];
  CUtensorMap mq, mk, mv;
  if (!make_tmap_noexcept(&mq, q, total_tokens, q_ld, q_ld) || !make_tmap_noexcept(&mk, k, total_tokens, k_ld, k_ld) ||
      !make_tmap_noexcept(&mv, v, total_tokens, v_ld, v_ld))
    return MIMIR_NOALLOC_ERR_ARGS;
  // The tile count (words[0]) is rewritten by the schedule kernel; the status word keeps
  // collecting failures until mimir_fmha_noalloc_status() reads and clears it.
  // A causal call never reads prefix_lens; the schedule kernel gets the cu_seqlens pointer as a
  // harmless stand-in so it never dereferences a null pointer.
  const int* prefix = is_causal ? cu_seqlens : prefix_lens;
  build_tiles_kernel<<<1, 1024, 0, stream>>>(cu_seqlens, prefix, numseqs, is_causal ? 1 : 0, s.tiles, s.words,
                                             (int)max_tiles);
  FwdParams prm{};
  prm.y = reinterpret_cast<__nv_bfloat16*>(out);
  prm.lse = lse;
  prm.lse_ld = lse_ld;
  prm.cu_seqlens = cu_seqlens;
  prm.prefix_lens = prefix;
  prm.tiles = s.tiles;
  prm.ntiles = s.words;
  prm.H = num_heads;
  prm.KV = num_kv_heads;
  prm.is_causal = is_causal ? 1 : 0;
  prm.scale_log2 = 1.4426950408889634f / sqrtf((float)kHeadDim);
  prm.status = s.words + 1;
  dim3 grid((unsigned)num_heads, (unsigned)max_tiles);
  fmha_fwd_kernel<<<grid, kThreads, kSmemBytes, stream>>>(mq, mk, mv, prm);
  return cudaGetLastError() == cudaSuccess ? MIMIR_NOALLOC_OK : MIMIR_NOALLOC_ERR_CUDA;
}

extern "C" int mimir_fmha_noalloc_status(cudaStream_t stream, int* status_out) {
  if (status_out == nullptr) return MIMIR_NOALLOC_ERR_ARGS;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return MIMIR_NOALLOC_ERR_CUDA;
  const int rc = noalloc_setup(device);
  if (rc != MIMIR_NOALLOC_OK) return rc;
  int* word = g_scratch[device].words + 1;
  // Pageable destination: the copy is staged by the driver, so it is complete once the
  // stream has synchronised.
  if (cudaMemcpyAsync(status_out, word, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return MIMIR_NOALLOC_ERR_CUDA;
  if (*status_out != 0 && cudaMemsetAsync(word, 0, sizeof(int), stream) != cudaSuccess) return MIMIR_NOALLOC_ERR_CUDA;
  return MIMIR_NOALLOC_OK;
}
