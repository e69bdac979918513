// Dense GEMM on the 5th-generation tensor cores, one CTA pair per 256-row output tile.
//
//   C[M, N] = alpha * sum_k A[m, k] * B[n, k]  (+ beta * D[M, N])
//
// A is K-major ([M, K] row-major) or M-major ([K, M] row-major, i.e. the transpose is stored);
// B is K-major ([N, K]) or N-major ([K, N]).  The three GEMMs of a linear layer Y = X W^T are
//   forward         Y  = X  W^T   A = X  [T, in]  K-major, B = W [out, in] K-major   ("nt")
//   input gradient  dX = dY W     A = dY [T, out] K-major, B = W [out, in] N-major   ("nn")
//   weight gradient dW = dY^T X   A = dY [T, out] M-major, B = X [T, in]   N-major   ("tn")
// so no operand is ever transposed in memory.
//
// Tiling: a cluster of two CTAs (an SM pair) owns a 256 x BN output tile.  Each CTA stages its
// 128 rows of A and BN/2 rows of B per 64-deep k-block with TMA (128-byte swizzle, no
// multicast), and the even CTA issues tcgen05.mma.cta_group::2 (M = 256, N = BN, K = 16), which
// reads both CTAs' shared memory and writes each CTA's 128 accumulator rows into its own TMEM.
// Per SM that is half the shared-memory operand traffic of a one-CTA 128 x BN tile.
//
// Persistent kernel, one CTA per SM, 10 warps per CTA:
//   warp 0      TMA producer (both CTAs): ring of kStages stages; every stage's bytes from both
//               CTAs complete on the even CTA's `full` barrier.
//   warp 1      MMA issuer (even CTA only): 4 MMAs per k-block into one of two TMEM
//               accumulators; commits release the stage in both CTAs (`empty`) and hand the
//               finished accumulator to both CTAs' epilogues (`acc_full`).
//   warps 2-9   epilogue (both CTAs): tcgen05.ld of the CTA's 128 rows (one row per thread; two
//               warps per TMEM lane quarter, each converting half of the columns), the fused
//               epilogue, 16-byte global stores; the 16 epilogue warps of the pair release the
//               accumulator on the even CTA's `acc_empty` barrier.
// Tiles are visited in groups of `group_m` 256-row blocks (all column blocks of a group before
// the next group) so that the clusters running at the same time share A and B panels in L2.
//
// Fused epilogues: plain (alpha/beta with an optional bf16 or fp32 addend, which may alias the
// output: in-place gradient accumulation), SwiGLU forward (the CTA pair loads matching gate and
// up weight rows, writes gate|up for the backward and silu(gate) * up), and SwiGLU backward
// (the down projection's input gradient turned into d[gate|up] from the saved gate|up).
//
// Every mbarrier wait is bounded by a run-time limit (default 2 s); on a timeout the kernel
// records a status code, stops issuing work, waits (bounded) for its copies and MMAs, frees
// TMEM and returns.  `inject` = 1 is a test hook: one epilogue warp withholds its first
// accumulator release, so the MMA issuer's wait runs out (the timeout path without a GPU fault).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "swiglu_math.cuh"  // shared bit for bit with the standalone SwiGLU kernels
#include "tma.cuh"

using namespace mimir;

namespace {

constexpr int kBM = 128;  // A rows per CTA (256 per pair)
constexpr int kBK = 64;   // k per stage: one 128-byte swizzle row of bf16
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, each taking half of the tile's columns
constexpr int kThreads = 64 + 32 * kEpiWarps;

enum EpiKind : int { kEpiStore = 0, kEpiSwiGLU = 1, kEpiSwiGLUBwd = 2 };

struct GemmParams {
  void* out;  // [M, N] bf16, or fp32 when the kernel's kOutF32 is set
  int64_t ldo;
  const void* add;  // optional addend of the output's dtype and shape (may alias `out`)
  int64_t ldd;
  float alpha, beta;
  void* aux;  // SwiGLU: gate|up [M, 2F] bf16 (written by the forward, read by the backward)
  int64_t ldx;
  int ffn;  // SwiGLU: F
  int M, N, K;
  int batch;                          // independent problems; z coordinate of the 3-D TMA maps
  int64_t bs_out, bs_add, bs_aux;     // element strides between the problems' out / add / aux
  int tiles_m, tiles_n, group_m;
  int* status;
  unsigned long long wait_ns;
  int inject;
};

// Per-warp staging for the TMA-store epilogues: one [32 rows x 32 columns] bf16 chunk is 2 KB
// (64-byte rows, 64-byte swizzle).  Plain stores double-buffer one output; the SwiGLU forward
// stages three outputs (gate, up, product) and the SwiGLU backward two (d gate, d up).
template <int BN, int kEpi>
struct PairCfg {
  static constexpr int kBHalf = BN / 2;             // B rows staged per CTA
  static constexpr int kABytes = kBM * kBK * 2;     // 16 KB
  static constexpr int kBBytes = kBHalf * kBK * 2;  // 16 KB (BN 256) or 8 KB (BN 128)
  static constexpr int kStageBytes = kABytes + kBBytes;
  // A 160 KB ring (5 stages at BN 256, 6 at BN 128) keeps the tensor pipe fed and leaves room on
  // the SM for a CTA of another kernel (the optimizer update overlapping the backward).
  static constexpr int kStages = 163840 / kStageBytes;
  static constexpr int kChunkBytes = 32 * 32 * 2;
  static constexpr int kStagingPerWarp = (kEpi == 1 ? 3 : 2) * kChunkBytes;
  static constexpr int kStagingOffset = kStages * kStageBytes;  // 1024-aligned (stages are 8 KB multiples)
  static constexpr int kSmem = kStagingOffset + kEpiWarps * kStagingPerWarp + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
  static_assert(kStages <= 8, "barrier arrays hold 8 stages");
  static_assert(kSmem + 1024 <= 232448, "dynamic + static shared memory must fit one SM");
};

struct PairBars {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t done;
  uint32_t tmem_base;
};

__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& bt, int& mt, int& nt) {
  const int per_problem = p.tiles_m * p.tiles_n;
  bt = t / per_problem;
  t -= bt * per_problem;
  const int per_group = p.group_m * p.tiles_n;
  const int g = t / per_group;
  const int first = g * p.group_m;
  const int gsize = min(p.group_m, p.tiles_m - first);
  const int r = t - g * per_group;
  mt = first + r % gsize;
  nt = r / gsize;
}

// Element offsets of one output row of problem `bt` in out / add / aux.
struct RowOffsets {
  int64_t out, add, aux;
};
__device__ __forceinline__ RowOffsets row_offsets(const GemmParams& p, int bt, int row) {
  return {bt * p.bs_out + static_cast<int64_t>(row) * p.ldo, bt * p.bs_add + static_cast<int64_t>(row) * p.ldd,
          bt * p.bs_aux + static_cast<int64_t>(row) * p.ldx};
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    d[q] = make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                      pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&v)[32]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 w = s[q];
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&words[e]));
      v[8 * q + 2 * e] = f.x;
      v[8 * q + 2 * e + 1] = f.y;
    }
  }
}

// ------------------------------------------------------------------------------ staged stores
// Thread `lane` owns row `lane` of a [32 x 32] bf16 chunk: it writes its 64-byte row into the
// warp's staging tile with the 64-byte TMA swizzle (16-byte piece j of row r at piece
// j ^ ((r >> 1) & 3)), conflict-free; one lane then stores the tile with TMA.
__device__ __forceinline__ void stage_row_bf16(uint32_t tile, int lane, const float (&v)[32]) {
  const uint32_t row = tile + lane * 64;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    st_shared_v4(row + ((j ^ sw) << 4), pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                 pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t smem_src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_src), "r"(x), "r"(y), "r"(z)
               : "memory");
}

// Both loads in flight before the single wait.
__device__ __forceinline__ void tmem_ld32_pair(uint32_t a, uint32_t b, float (&va)[32], float (&vb)[32]) {
  uint32_t ra[32], rb[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(ra[0]), "=r"(ra[1]), "=r"(ra[2]), "=r"(ra[3]), "=r"(ra[4]), "=r"(ra[5]), "=r"(ra[6]), "=r"(ra[7]),
        "=r"(ra[8]), "=r"(ra[9]), "=r"(ra[10]), "=r"(ra[11]), "=r"(ra[12]), "=r"(ra[13]), "=r"(ra[14]), "=r"(ra[15]),
        "=r"(ra[16]), "=r"(ra[17]), "=r"(ra[18]), "=r"(ra[19]), "=r"(ra[20]), "=r"(ra[21]), "=r"(ra[22]), "=r"(ra[23]),
        "=r"(ra[24]), "=r"(ra[25]), "=r"(ra[26]), "=r"(ra[27]), "=r"(ra[28]), "=r"(ra[29]), "=r"(ra[30]), "=r"(ra[31]),
        "=r"(rb[0]), "=r"(rb[1]), "=r"(rb[2]), "=r"(rb[3]), "=r"(rb[4]), "=r"(rb[5]), "=r"(rb[6]), "=r"(rb[7]),
        "=r"(rb[8]), "=r"(rb[9]), "=r"(rb[10]), "=r"(rb[11]), "=r"(rb[12]), "=r"(rb[13]), "=r"(rb[14]), "=r"(rb[15]),
        "=r"(rb[16]), "=r"(rb[17]), "=r"(rb[18]), "=r"(rb[19]), "=r"(rb[20]), "=r"(rb[21]), "=r"(rb[22]), "=r"(rb[23]),
        "=r"(rb[24]), "=r"(rb[25]), "=r"(rb[26]), "=r"(rb[27]), "=r"(rb[28]), "=r"(rb[29]), "=r"(rb[30]), "=r"(rb[31])
      : "r"(a), "r"(b)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    va[i] = __uint_as_float(ra[i]);
    vb[i] = __uint_as_float(rb[i]);
  }
}

// Staging tiles of the calling warp and a running count of the chunks it has staged (across
// tiles), which decides when a tile may be reused.
struct Staging {
  uint32_t base;  // this warp's first tile
  uint32_t count;
};

// ------------------------------------------------------------------------------ epilogues
// One thread holds one accumulator row (its TMEM lane); `half` selects which half of the tile's
// 32-column chunks this warp converts.  tcgen05.ld is warp-collective, so it stays outside the
// per-thread `valid` branches.

template <int BN, bool kOutF32>
__device__ __forceinline__ void epilogue_store(const GemmParams& p, uint32_t tacc, const RowOffsets& ro, bool valid,
                                               int n0, int half) {
  constexpr int kChunks = BN / 64;
#pragma unroll 1
  for (int j = 0; j < kChunks; ++j) {
    const int c = half * kChunks + j;
    float v[32];
    tmem_ld32(tacc + c * 32, v);
    const int col = n0 + c * 32;
    if (!valid || col >= p.N) continue;
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] *= p.alpha;
    if (kOutF32) {
      if (p.add != nullptr) {
        const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.add) + ro.add + col);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 a = src[q];
          v[4 * q] += p.beta * a.x;
          v[4 * q + 1] += p.beta * a.y;
          v[4 * q + 2] += p.beta * a.z;
          v[4 * q + 3] += p.beta * a.w;
        }
      }
      float4* d4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + ro.out + col);
#pragma unroll
      for (int q = 0; q < 8; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
      if (p.add != nullptr) {
        float a[32];
        load_bf16x32(reinterpret_cast<const __nv_bfloat16*>(p.add) + ro.add + col, a);
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] += p.beta * a[e];
      }
      store_bf16x32(reinterpret_cast<__nv_bfloat16*>(p.out) + ro.out + col, v);
    }
  }
}

__device__ __forceinline__ void load_raw4(const __nv_bfloat16* src, uint4 (&r)[4]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) r[q] = __ldg(s + q);
}

__device__ __forceinline__ void unpack_bf16x32(const uint4 (&r)[4], float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t words[4] = {r[q].x, r[q].y, r[q].z, r[q].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&words[e]));
      v[8 * q + 2 * e] = f.x;
      v[8 * q + 2 * e + 1] = f.y;
    }
  }
}

// Plain bf16 output through TMA stores (no addend): double-buffered 2 KB tiles per warp.
template <int BN>
__device__ __forceinline__ void epilogue_store_tma(const GemmParams& p, const CUtensorMap* map_out, uint32_t tacc,
                                                   int lane, int row0, int bt, int n0, int half, Staging& st) {
  constexpr int kChunks = BN / 64;
#pragma unroll 1
  for (int j = 0; j < kChunks; ++j, ++st.count) {
    const int c = half * kChunks + j;
    float v[32];
    tmem_ld32(tacc + c * 32, v);
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] *= p.alpha;
    const uint32_t tile = st.base + (st.count & 1) * (32 * 32 * 2);
    if (st.count >= 2) {  // the store issued from this tile two chunks ago has read it
      if (lane == 0) bulk_wait_group_read1();
      __syncwarp();
    }
    stage_row_bf16(tile, lane, v);
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(map_out, tile, n0 + c * 32, row0, bt);
      bulk_commit_group();
    }
  }
}

// SwiGLU forward through TMA stores: gate and up to the gate|up buffer, the product to `out`.
template <int BN>
__device__ __forceinline__ void epilogue_swiglu_fwd_tma(const GemmParams& p, const CUtensorMap* map_out,
                                                        const CUtensorMap* map_aux, uint32_t tacc, int lane, int row0,
                                                        int bt, int h0, int half, Staging& st) {
  constexpr int kHalf = BN / 2;
  constexpr int kChunks = kHalf / 64;
  constexpr uint32_t kTile = 32 * 32 * 2;
#pragma unroll 1
  for (int j = 0; j < kChunks; ++j, ++st.count) {
    const int c = half * kChunks + j;
    float g[32], u[32];
    tmem_ld32_pair(tacc + c * 32, tacc + kHalf + c * 32, g, u);
    if (st.count >= 1) {  // the previous chunk's three stores have read their tiles
      if (lane == 0) bulk_wait_group_read0();
      __syncwarp();
    }
    stage_row_bf16(st.base, lane, g);
    stage_row_bf16(st.base + kTile, lane, u);
#pragma unroll
    for (int e = 0; e < 32; ++e) g[e] = swiglu_silu(bf16_round(g[e])) * bf16_round(u[e]);
    stage_row_bf16(st.base + 2 * kTile, lane, g);
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
      const int col = h0 + c * 32;
      tma_store_3d(map_aux, st.base, col, row0, bt);
      tma_store_3d(map_aux, st.base + kTile, p.ffn + col, row0, bt);
      tma_store_3d(map_out, st.base + 2 * kTile, col, row0, bt);
      bulk_commit_group();
    }
  }
}

// SwiGLU backward through TMA stores of d gate / d up; gate|up read with prefetched 16-byte loads.
template <int BN>
__device__ __forceinline__ bool epilogue_swiglu_bwd_tma(const GemmParams& p, const CUtensorMap* map_out,
                                                        uint64_t* acc_full, uint32_t parity, uint32_t tacc,
                                                        const RowOffsets& ro, bool valid, int lane, int row0, int bt,
                                                        int n0, int half, Staging& st) {
  constexpr int kChunks = BN / 64;
  constexpr uint32_t kTile = 32 * 32 * 2;
  const __nv_bfloat16* gu = reinterpret_cast<const __nv_bfloat16*>(p.aux) + ro.aux;
  uint4 gn[4], un[4];
  int c = half * kChunks;
  if (valid && n0 + c * 32 < p.N) {
    load_raw4(gu + n0 + c * 32, gn);
    load_raw4(gu + p.ffn + n0 + c * 32, un);
  }
  if (!warp_wait_ns(acc_full, parity, p.status, kStatusTimeoutS, p.wait_ns)) return false;
  tc_fence_after();
#pragma unroll 1
  for (int j = 0; j < kChunks; ++j, ++c, ++st.count) {
    const int col = n0 + c * 32;
    uint4 gc[4], uc[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      gc[q] = gn[q];
      uc[q] = un[q];
    }
    if (j + 1 < kChunks && valid && col + 32 < p.N) {
      load_raw4(gu + col + 32, gn);
      load_raw4(gu + p.ffn + col + 32, un);
    }
    float d[32];
    tmem_ld32(tacc + c * 32, d);
    float g[32], u[32];
    unpack_bf16x32(gc, g);
    unpack_bf16x32(uc, u);
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      float dg, du;
      swiglu_backward(bf16_round(d[e]), g[e], u[e], dg, du);
      g[e] = dg;
      u[e] = du;
    }
    if (st.count >= 1) {
      if (lane == 0) bulk_wait_group_read0();
      __syncwarp();
    }
    stage_row_bf16(st.base, lane, g);
    stage_row_bf16(st.base + kTile, lane, u);
    fence_async_shared();
    __syncwarp();
    if (lane == 0 && col < p.N) {
      tma_store_3d(map_out, st.base, col, row0, bt);
      tma_store_3d(map_out, st.base + kTile, p.ffn + col, row0, bt);
      bulk_commit_group();
    }
  }
  return true;
}

template <int BN, bool kAMn, bool kBMn, int kEpi, bool kOutF32>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_out, const __grid_constant__ CUtensorMap map_aux,
                     const GemmParams p) {
  using CF = PairCfg<BN, kEpi>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ PairBars bars;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  const int total = p.batch * p.tiles_m * p.tiles_n;
  const int nkb = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < CF::kStages; ++s) {
      mbar_init(&bars.full[s], 1);
      mbar_init(&bars.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.acc_full[i], 1);
      mbar_init(&bars.acc_empty[i], 2 * kEpiWarps);
    }
    mbar_init(&bars.done, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars.tmem_base, CF::kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem = bars.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = cid; ok && t < total; t += ncl) {
        int bt, mt, nt;
        tile_coords(t, p, bt, mt, nt);
        const int am = mt * 2 * kBM + static_cast<int>(rank) * kBM;
        const int bn = kEpi == kEpiSwiGLU ? nt * CF::kBHalf + (rank ? p.ffn : 0)  // gate rows | up rows
                                          : nt * BN + static_cast<int>(rank) * CF::kBHalf;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CF::kStages;
          if (it >= CF::kStages && !mbar_wait_ns(&bars.empty[s], ((it / CF::kStages) - 1) & 1, p.status,
                                                 kStatusTimeoutEmpty, p.wait_ns)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem_u32(smem + s * CF::kStageBytes);
          const uint32_t sb = sa + CF::kABytes;
          const uint32_t fb = mapa_shared(smem_u32(&bars.full[s]), 0);
          if (leader) mbar_arrive_expect_tx(&bars.full[s], 2 * CF::kStageBytes);
          const int k0 = kb * kBK;
          if (kAMn) {
#pragma unroll
            for (int c = 0; c < kBM / 64; ++c) tma_load_3d_pair(sa + c * (kBK * 128), &map_a, fb, am + c * 64, k0, bt);
          } else {
            tma_load_3d_pair(sa, &map_a, fb, k0, am, bt);
          }
          if (kBMn) {
#pragma unroll
            for (int c = 0; c < CF::kBHalf / 64; ++c)
              tma_load_3d_pair(sb + c * (kBK * 128), &map_b, fb, bn + c * 64, k0, bt);
          } else {
            tma_load_3d_pair(sb, &map_b, fb, k0, bn, bt);
          }
        }
      }
      // Tail: the last stages are released once the pair's MMAs have read them, which also
      // means their copies have landed.
      // After a timeout nothing releases the stages any more: give the copies in flight a fixed
      // millisecond to land instead.
      for (int j = max(0, it - CF::kStages); j < it; ++j) {
        if (!mbar_wait_ns(&bars.empty[j % CF::kStages], (j / CF::kStages) & 1, p.status, kStatusTimeoutKV,
                          p.wait_ns)) {
          spin_ns(1000000ull);
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(2 * kBM, BN, kAMn ? 1 : 0, kBMn ? 1 : 0);
      int it = 0, i = 0;
      bool ok = true;
      for (int t = cid; ok && t < total; t += ncl, ++i) {
        const int buf = i & 1;
        if (i >= 2 &&
            !mbar_wait_ns(&bars.acc_empty[buf], ((i >> 1) - 1) & 1, p.status, kStatusTimeoutO, p.wait_ns))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CF::kStages;
          if (!mbar_wait_ns(&bars.full[s], (it / CF::kStages) & 1, p.status, kStatusTimeoutKV, p.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * CF::kStageBytes);
          const uint32_t sb = sa + CF::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // K-major: 16 k = 32 bytes along the swizzled row.  MN-major: 16 k-rows = 2048 bytes;
            // the 64-wide column chunks sit kBK * 128 bytes apart (leading byte offset).
            const uint64_t ad = kAMn ? smem_desc(sa + kk * 2048, kBK * 128, 1024, kLayoutSW128)
                                     : smem_desc(sa + kk * 32, 16, 1024, kLayoutSW128);
            const uint64_t bd = kBMn ? smem_desc(sb + kk * 2048, kBK * 128, 1024, kLayoutSW128)
                                     : smem_desc(sb + kk * 32, 16, 1024, kLayoutSW128);
            mma_bf16_pair(acc, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          mma_commit_pair(&bars.empty[s], 0x3);  // the stage is free in both CTAs once read
        }
        if (ok) mma_commit_pair(&bars.acc_full[buf], 0x3);
      }
      mma_commit_pair(&bars.done, 0x3);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // Warp w reads TMEM lanes 32 * (w % 4) .. + 32 (its rows) and one half of the columns.
    const int wq = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    // bf16 outputs without an addend leave through TMA stores from per-warp staging tiles.
    const bool staged = !kOutF32 && (kEpi != kEpiStore || p.add == nullptr);
    Staging st{smem_u32(smem + CF::kStagingOffset) + static_cast<uint32_t>((warp - 2) * CF::kStagingPerWarp), 0u};
    int i = 0;
    for (int t = cid; t < total; t += ncl, ++i) {
      const int buf = i & 1;
      int bt, mt, nt;
      tile_coords(t, p, bt, mt, nt);
      const int row0 = mt * 2 * kBM + static_cast<int>(rank) * kBM + wq * 32;
      const int row = row0 + lane;
      const bool valid = row < p.M;
      const RowOffsets ro = row_offsets(p, bt, row);
      const uint32_t tacc = tmem + lane_off + buf * BN;
      if (kEpi == kEpiSwiGLUBwd) {
        // Issues its first operand loads before waiting for the accumulator.
        if (!epilogue_swiglu_bwd_tma<BN>(p, &map_out, &bars.acc_full[buf], (i >> 1) & 1, tacc, ro, valid, lane, row0,
                                         bt, nt * BN, half, st))
          break;
      } else {
        if (!warp_wait_ns(&bars.acc_full[buf], (i >> 1) & 1, p.status, kStatusTimeoutS, p.wait_ns)) break;
        tc_fence_after();
        if (kEpi == kEpiSwiGLU) {
          epilogue_swiglu_fwd_tma<BN>(p, &map_out, &map_aux, tacc, lane, row0, bt, nt * (BN / 2), half, st);
        } else if (staged) {
          epilogue_store_tma<BN>(p, &map_out, tacc, lane, row0, bt, nt * BN, half, st);
        } else {
          epilogue_store<BN, kOutF32>(p, tacc, ro, valid, nt * BN, half);
        }
      }
      tc_fence_before();
      __syncwarp();
      const bool withhold = p.inject == 1 && i == 0 && leader && warp == 4;
      if (lane == 0 && !withhold) mbar_arrive_remote(mapa_shared(smem_u32(&bars.acc_empty[buf]), 0));
    }
    if (staged && lane == 0) bulk_wait_group0();  // every staged store has landed before exit
    __syncwarp();
    // Every MMA that writes this CTA's TMEM has completed before TMEM is freed (the last
    // accumulator was just read, so in a normal run this wait is short).
    if (warp == 2 && lane == 0) mbar_wait_ns(&bars.done, 0, p.status, kStatusTimeoutOther, p.wait_ns);
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, CF::kTmemCols);
  }
}

// ------------------------------------------------------------------------------ all-gather + GEMM
// Forward of a linear layer whose weight W [N, K] is sharded by rows over the `world` GPUs of one
// node: rank k holds rows [k * S, (k + 1) * S) (S = N / world) in memory that every rank maps.
// One launch computes y = x W^T and leaves the whole of W in this GPU's buffer G, which the
// backward's input gradient then reads locally (no second all-gather).
//
// Nothing waits on another CTA or another GPU, so no launch order or co-residency matters:
//   * The odd CTA of every pair runs a gatherer (its warp 1, idle in the pair kernel): it copies
//     items of W (128 rows x a range of k-blocks, 16 KB per TMA load, two loads in flight) from
//     their owner's memory into G with TMA stores, and after an item's stores are complete adds
//     one to its 128-row block's counter (release, GPU scope).  Items run in ring order: the
//     next rank's rows first, this rank's own rows (a local copy) last.
//   * Tiles run column by column starting at this rank's own columns, so the first waves read
//     only local weight rows while the gatherers pull the next ranks' rows over NVLink.
//   * For each tile the producer reads its 128-row block's counter once (acquire): a complete
//     block is read from G; otherwise the rows come straight from the owner's memory (correct,
//     only more NVLink traffic), so a late gatherer costs bandwidth, never a wait.
// The counters grow by `parts` per call and never reset: a block is complete for call e when
// its counter reaches e * parts.  Loads from peer memory are plain tiled TMA (no multicast).
struct GatherArgs {
  CUtensorMap shard[8];  // rank k's rows [S, K], box 64 x 128
  CUtensorMap g;         // G [N, K] on this GPU, box 64 x 128
  unsigned* flags;       // [N / 128] completion counters
  unsigned target;       // counter value of a block that is complete in this call
  int rank, world, shard_rows, parts;
};

constexpr int kGatherSlotBytes = 128 * kBK * 2;  // one 128-row x 64-column bf16 box

__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* ptr) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add_u32(unsigned* ptr, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// 3-D tiled TMA load into this CTA's shared memory, completion on this CTA's barrier.
__device__ __forceinline__ void tma_load_3d_cta(uint32_t smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Column-major tile order starting at the column block that holds this rank's first row.
template <int BN>
__device__ __forceinline__ void gather_tile(int t, const GemmParams& p, const GatherArgs& ga, int& mt, int& nt) {
  const int col = t / p.tiles_m;
  mt = t - col * p.tiles_m;
  nt = (col + (ga.rank * ga.shard_rows) / BN) % p.tiles_n;
}

// Position of one gatherer in its item sequence (items cid, cid + ncl, ...).
struct GatherCursor {
  int item, kb, hi;
};
__device__ __forceinline__ void cursor_set(GatherCursor& c, int item, int parts, int nkb) {
  c.item = item;
  c.kb = ((item % parts) * nkb) / parts;
  c.hi = ((item % parts + 1) * nkb) / parts;
}
__device__ __forceinline__ void cursor_next(GatherCursor& c, int ncl, int parts, int nkb) {
  if (++c.kb == c.hi) cursor_set(c, c.item + ncl, parts, nkb);
}

__device__ __forceinline__ int gather_owner(const GatherArgs& ga, int item, int per_rank) {
  return (ga.rank + 1 + (item / ga.parts) / per_rank) % ga.world;
}
__device__ __forceinline__ int gather_srow(const GatherArgs& ga, int item, int per_rank) {
  return ((item / ga.parts) % per_rank) * 128;
}

__device__ void gather_rows(const GatherArgs& ga, const GemmParams& p, uint32_t slots, uint64_t* gbar, int cid,
                            int ncl) {
  const int nkb = (p.K + kBK - 1) / kBK;
  const int per_rank = ga.shard_rows / 128;
  const int items = ga.world * per_rank * ga.parts;
  GatherCursor ld, st;
  cursor_set(ld, cid, ga.parts, nkb);
  st = ld;
  int loaded = 0, stored = 0;
  bool ok = true;
  for (int s = 0; s < 2 && ld.item < items; ++s) {
    mbar_arrive_expect_tx(&gbar[s], kGatherSlotBytes);
    tma_load_3d_cta(slots + s * kGatherSlotBytes, &ga.shard[gather_owner(ga, ld.item, per_rank)], &gbar[s],
                    ld.kb * kBK, gather_srow(ga, ld.item, per_rank), 0);
    cursor_next(ld, ncl, ga.parts, nkb);
    ++loaded;
  }
  while (stored < loaded) {
    const int s = stored & 1;
    if (!mbar_wait_ns(&gbar[s], (stored >> 1) & 1, p.status, kStatusTimeoutOther, p.wait_ns)) {
      ok = false;
      break;
    }
    const int grow = gather_owner(ga, st.item, per_rank) * ga.shard_rows + gather_srow(ga, st.item, per_rank);
    tma_store_3d(&ga.g, slots + s * kGatherSlotBytes, st.kb * kBK, grow, 0);
    bulk_commit_group();
    bulk_wait_group_read0();  // the slot may be refilled
    if (st.kb + 1 == st.hi) {  // the item is complete once its stores are
      bulk_wait_group0();
      fence_proxy_async_global();
      red_release_gpu_add_u32(&ga.flags[grow / 128], 1u);
    }
    cursor_next(st, ncl, ga.parts, nkb);
    ++stored;
    if (ld.item < items) {
      mbar_arrive_expect_tx(&gbar[s], kGatherSlotBytes);
      tma_load_3d_cta(slots + s * kGatherSlotBytes, &ga.shard[gather_owner(ga, ld.item, per_rank)], &gbar[s],
                      ld.kb * kBK, gather_srow(ga, ld.item, per_rank), 0);
      cursor_next(ld, ncl, ga.parts, nkb);
      ++loaded;
    }
  }
  bulk_wait_group0();
  if (!ok) spin_ns(1000000ull);  // loads still in flight land before the CTA exits
}

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_gather_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_out,
                       const __grid_constant__ GatherArgs ga, const GemmParams p) {
  using CF = PairCfg<BN, kEpiStore>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ PairBars bars;
  __shared__ uint64_t gbar[2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  const int total = p.tiles_m * p.tiles_n;
  const int nkb = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < CF::kStages; ++s) {
      mbar_init(&bars.full[s], 1);
      mbar_init(&bars.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.acc_full[i], 1);
      mbar_init(&bars.acc_empty[i], 2 * kEpiWarps);
      mbar_init(&gbar[i], 1);
    }
    mbar_init(&bars.done, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars.tmem_base, CF::kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&ga.g);
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = cid; ok && t < total; t += ncl) {
        int mt, nt;
        gather_tile<BN>(t, p, ga, mt, nt);
        const int am = mt * 2 * kBM + static_cast<int>(crank) * kBM;
        const int bn = nt * BN + static_cast<int>(crank) * CF::kBHalf;  // this CTA's 128 weight rows
        const int owner = bn / ga.shard_rows;
        const CUtensorMap* mb = &ga.shard[owner];
        int by = bn - owner * ga.shard_rows;
        if (owner != ga.rank && static_cast<int>(ld_acquire_gpu_u32(&ga.flags[bn / 128]) - ga.target) >= 0) {
          fence_proxy_async_global();  // G's rows were written by other CTAs' TMA stores
          mb = &ga.g;
          by = bn;
        }
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CF::kStages;
          if (it >= CF::kStages && !mbar_wait_ns(&bars.empty[s], ((it / CF::kStages) - 1) & 1, p.status,
                                                 kStatusTimeoutEmpty, p.wait_ns)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem_u32(smem + s * CF::kStageBytes);
          const uint32_t sb = sa + CF::kABytes;
          const uint32_t fb = mapa_shared(smem_u32(&bars.full[s]), 0);
          if (leader) mbar_arrive_expect_tx(&bars.full[s], 2 * CF::kStageBytes);
          tma_load_3d_pair(sa, &map_a, fb, kb * kBK, am, 0);
          tma_load_3d_pair(sb, mb, fb, kb * kBK, by, 0);
        }
      }
      for (int j = max(0, it - CF::kStages); j < it; ++j) {
        if (!mbar_wait_ns(&bars.empty[j % CF::kStages], (j / CF::kStages) & 1, p.status, kStatusTimeoutKV,
                          p.wait_ns)) {
          spin_ns(1000000ull);
          break;
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      // ---------------------------------------------------------- MMA issuer (even CTA)
      const uint32_t idesc = idesc_bf16_f32(2 * kBM, BN, 0, 0);
      int it = 0, i = 0;
      bool ok = true;
      for (int t = cid; ok && t < total; t += ncl, ++i) {
        const int buf = i & 1;
        if (i >= 2 &&
            !mbar_wait_ns(&bars.acc_empty[buf], ((i >> 1) - 1) & 1, p.status, kStatusTimeoutO, p.wait_ns))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CF::kStages;
          if (!mbar_wait_ns(&bars.full[s], (it / CF::kStages) & 1, p.status, kStatusTimeoutKV, p.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * CF::kStageBytes);
          const uint32_t sb = sa + CF::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16_pair(acc, smem_desc(sa + kk * 32, 16, 1024, kLayoutSW128),
                          smem_desc(sb + kk * 32, 16, 1024, kLayoutSW128), idesc, (kb | kk) != 0 ? 1u : 0u);
          mma_commit_pair(&bars.empty[s], 0x3);
        }
        if (ok) mma_commit_pair(&bars.acc_full[buf], 0x3);
      }
      mma_commit_pair(&bars.done, 0x3);
    } else if (!leader && lane == 0) {
      // ---------------------------------------------------------- gatherer (odd CTA)
      gather_rows(ga, p, smem_u32(smem + CF::kStagingOffset + kEpiWarps * CF::kStagingPerWarp), gbar, cid, ncl);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int wq = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    Staging st{smem_u32(smem + CF::kStagingOffset) + static_cast<uint32_t>((warp - 2) * CF::kStagingPerWarp), 0u};
    int i = 0;
    for (int t = cid; t < total; t += ncl, ++i) {
      const int buf = i & 1;
      int mt, nt;
      gather_tile<BN>(t, p, ga, mt, nt);
      const int row0 = mt * 2 * kBM + static_cast<int>(crank) * kBM + wq * 32;
      const uint32_t tacc = tmem + lane_off + buf * BN;
      if (!warp_wait_ns(&bars.acc_full[buf], (i >> 1) & 1, p.status, kStatusTimeoutS, p.wait_ns)) break;
      tc_fence_after();
      epilogue_store_tma<BN>(p, &map_out, tacc, lane, row0, 0, nt * BN, half, st);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&bars.acc_empty[buf]), 0));
    }
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
    if (warp == 2 && lane == 0) mbar_wait_ns(&bars.done, 0, p.status, kStatusTimeoutOther, p.wait_ns);
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, CF::kTmemCols);
  }
}

template <int BN>
constexpr int gather_smem() {
  return PairCfg<BN, kEpiStore>::kSmem + 2 * kGatherSlotBytes;
}
static_assert(gather_smem<256>() + 1024 <= 232448, "the gather kernel's shared memory must fit one SM");

// ------------------------------------------------------------------------------------ host side
int* status_word(int device) {
  static int* words[64] = {nullptr};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (words[device] == nullptr) {
    C10_CUDA_CHECK(cudaMalloc(&words[device], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(words[device], 0, sizeof(int)));
  }
  return words[device];
}

// Number of CTA pairs that can be resident at once (the persistent grid), per device.
int resident_pairs(int device, const void* kernel, int smem) {
  static int cached[64] = {0};
  if (cached[device] > 0) return cached[device];
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  cfg.gridDim = dim3(sms & ~1);
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters <= 0) {
    (void)cudaGetLastError();
    clusters = sms / 2;
  }
  cached[device] = clusters;
  return clusters;
}

template <int BN, bool kAMn, bool kBMn, int kEpi, bool kOutF32>
void launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const CUtensorMap& mx,
                 const GemmParams& p, int device, cudaStream_t st) {
  using CF = PairCfg<BN, kEpi>;
  auto kernel = gemm_pair_kernel<BN, kAMn, kBMn, kEpi, kOutF32>;
  static bool attr[64] = {false};
  if (!attr[device]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kSmem));
    attr[device] = true;
  }
  const int pairs = std::min(resident_pairs(device, reinterpret_cast<const void*>(kernel), CF::kSmem),
                             p.batch * p.tiles_m * p.tiles_n);
  kernel<<<2 * pairs, kThreads, CF::kSmem, st>>>(ma, mb, mo, mx, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void check_operand(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && (t.dim() == 2 || t.dim() == 3) && t.stride(-1) == 1,
              name, ": bf16 CUDA matrix (or batch of matrices) with unit column stride");
  TORCH_CHECK((t.stride(-2) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0 &&
                  (t.dim() == 2 || (t.stride(0) * 2) % 16 == 0),
              name, ": 16-byte aligned base and strides");
}

// TMA map of one operand (2-D: a batch of one), rows x cols with a box of box_cols x box_rows.
CUtensorMap operand_map(const at::Tensor& t, int box_cols, int box_rows) {
  const int64_t rows = t.size(-2), cols = t.size(-1), ld = t.stride(-2);
  const int64_t batch = t.dim() == 3 ? t.size(0) : 1;
  const int64_t bstride = t.dim() == 3 ? t.stride(0) : rows * ld;
  return make_tmap_bf16_3d(t.data_ptr(), batch, rows, cols, ld, bstride, box_cols, box_rows);
}

template <int BN>
void dispatch_store(bool a_mn, bool b_mn, bool f32, const CUtensorMap& ma, const CUtensorMap& mb,
                    const CUtensorMap& mo, const GemmParams& p, int dev, cudaStream_t st) {
  const int code = (a_mn ? 4 : 0) | (b_mn ? 2 : 0) | (f32 ? 1 : 0);
  switch (code) {
    case 0: launch_pair<BN, false, false, kEpiStore, false>(ma, mb, mo, mo, p, dev, st); break;
    case 1: launch_pair<BN, false, false, kEpiStore, true>(ma, mb, mo, mo, p, dev, st); break;
    case 2: launch_pair<BN, false, true, kEpiStore, false>(ma, mb, mo, mo, p, dev, st); break;
    case 3: launch_pair<BN, false, true, kEpiStore, true>(ma, mb, mo, mo, p, dev, st); break;
    case 6: launch_pair<BN, true, true, kEpiStore, false>(ma, mb, mo, mo, p, dev, st); break;
    case 7: launch_pair<BN, true, true, kEpiStore, true>(ma, mb, mo, mo, p, dev, st); break;
    default: TORCH_CHECK(false, "unsupported operand layout: an M-major A needs an N-major B");
  }
}

// TMA map of a bf16 output written in [32 rows x 32 columns] chunks (64-byte swizzle); a map
// the kernel never uses (fp32 output, or an output read back as an addend) is left zero.
CUtensorMap output_map(const at::Tensor& t) {
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  if (t.scalar_type() != at::kBFloat16) return map;
  const int64_t rows = t.size(-2), cols = t.size(-1), ld = t.stride(-2);
  const int64_t batch = t.dim() == 3 ? t.size(0) : 1;
  const int64_t bstride = t.dim() == 3 ? t.stride(0) : rows * ld;
  return make_tmap_bf16_3d(t.data_ptr(), batch, rows, cols, ld, bstride, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
}

GemmParams base_params(int M, int N, int K, int BN, int64_t group_m, int64_t wait_ns, int64_t inject, int device) {
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.alpha = 1.f;
  p.beta = 0.f;
  p.tiles_m = (M + 2 * kBM - 1) / (2 * kBM);
  p.tiles_n = (N + BN - 1) / BN;
  p.group_m = static_cast<int>(std::max<int64_t>(1, group_m));
  p.batch = 1;
  p.status = status_word(device);
  p.wait_ns = wait_ns > 0 ? static_cast<unsigned long long>(wait_ns) : 2000000000ull;
  p.inject = static_cast<int>(inject);
  return p;
}

}  // namespace

// out[M, N] = alpha * op(a) @ op(b)^T (+ beta * add).  a: [M, K] (a_mn = false) or [K, M] (a_mn =
// true); b: [N, K] (b_mn = false) or [K, N] (b_mn = true).  `out` (bf16 or fp32) is allocated as
// bf16 when absent; `add` has out's dtype and may be `out` itself (in-place accumulation).  With
// 3-D operands ([batch, ...], every tensor the same batch) the problems run in one launch.
at::Tensor gemm(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn, c10::optional<at::Tensor> out,
                c10::optional<at::Tensor> add, double alpha, double beta, int64_t bn, int64_t group_m,
                int64_t wait_ns, int64_t inject) {
  check_operand(a, "a");
  check_operand(b, "b");
  TORCH_CHECK(a.dim() == b.dim(), "a and b must both be matrices or both batches");
  const bool batched = a.dim() == 3;
  const int64_t B = batched ? a.size(0) : 1;
  TORCH_CHECK(!batched || b.size(0) == B, "a and b batch sizes differ");
  const int64_t M = a_mn ? a.size(-1) : a.size(-2), K = a_mn ? a.size(-2) : a.size(-1);
  const int64_t N = b_mn ? b.size(-1) : b.size(-2);
  TORCH_CHECK((b_mn ? b.size(-2) : b.size(-1)) == K, "inner dimensions differ");
  TORCH_CHECK(!a_mn || b_mn, "an M-major A needs an N-major B");
  TORCH_CHECK(N % 32 == 0, "N must be a multiple of 32");  // inner extents are checked by the TMA maps
  TORCH_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31) && B < (1ll << 16), "dimensions out of range");
  const c10::cuda::CUDAGuard guard(a.device());
  at::Tensor o = out.has_value() ? *out : (batched ? at::empty({B, M, N}, a.options()) : at::empty({M, N}, a.options()));
  TORCH_CHECK(o.is_cuda() && o.dim() == a.dim() && o.size(-2) == M && o.size(-1) == N && o.stride(-1) == 1 &&
                  (!batched || o.size(0) == B) && (o.scalar_type() == at::kBFloat16 || o.scalar_type() == at::kFloat),
              "out: [(batch,) M, N] bf16 or fp32 with unit column stride");
  const bool f32 = o.scalar_type() == at::kFloat;
  TORCH_CHECK(reinterpret_cast<uintptr_t>(o.data_ptr()) % 16 == 0 && (o.stride(-2) * o.element_size()) % 16 == 0,
              "out: 16-byte aligned base and row stride");
  if (M == 0 || N == 0 || B == 0) return o;
  const int BN = bn == 128 ? 128 : 256;
  const int dev = a.device().index();
  GemmParams p = base_params(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), BN, group_m, wait_ns,
                             inject, dev);
  p.batch = static_cast<int>(B);
  p.out = o.data_ptr();
  p.ldo = o.stride(-2);
  p.bs_out = batched ? o.stride(0) : 0;
  p.alpha = static_cast<float>(alpha);
  if (add.has_value() && beta != 0.0) {
    const auto& d = *add;
    TORCH_CHECK(d.scalar_type() == o.scalar_type() && d.dim() == o.dim() && d.size(-2) == M && d.size(-1) == N &&
                    (!batched || d.size(0) == B) && d.stride(-1) == 1 &&
                    reinterpret_cast<uintptr_t>(d.data_ptr()) % 16 == 0 && (d.stride(-2) * d.element_size()) % 16 == 0,
                "add: same dtype and shape as out, 16-byte aligned");
    p.add = d.data_ptr();
    p.ldd = d.stride(-2);
    p.bs_add = batched ? d.stride(0) : 0;
    p.beta = static_cast<float>(beta);
  }
  if (K == 0) {  // no products: the result is the scaled addend (or zero)
    if (p.add != nullptr) o.copy_(add->mul(beta));
    else o.zero_();
    return o;
  }
  const CUtensorMap ma = a_mn ? operand_map(a, 64, kBK) : operand_map(a, kBK, kBM);
  const CUtensorMap mb = b_mn ? operand_map(b, 64, kBK) : operand_map(b, kBK, BN / 2);
  const CUtensorMap mo = output_map(o);
  auto st = at::cuda::getCurrentCUDAStream();
  if (BN == 256) dispatch_store<256>(a_mn, b_mn, f32, ma, mb, mo, p, dev, st);
  else dispatch_store<128>(a_mn, b_mn, f32, ma, mb, mo, p, dev, st);
  return o;
}

// Forward of a SwiGLU MLP's first projection: gu = x @ w_gu^T (w_gu = [gate rows; up rows],
// [2F, K]) and h = silu(gate) * up, both bf16.  Returns {h [M, F], gu [M, 2F]}.
std::vector<at::Tensor> gemm_swiglu(at::Tensor x, at::Tensor w_gu, int64_t group_m) {
  check_operand(x, "x");
  check_operand(w_gu, "w_gu");
  TORCH_CHECK(x.dim() == 2 && w_gu.dim() == 2, "x and w_gu must be matrices");
  const int64_t M = x.size(0), K = x.size(1), F = w_gu.size(0) / 2;
  TORCH_CHECK(w_gu.size(1) == K && w_gu.size(0) == 2 * F, "w_gu: [2F, K]");
  TORCH_CHECK(F % 128 == 0, "F must be a multiple of 128");
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor h = at::empty({M, F}, x.options());
  at::Tensor gu = at::empty({M, 2 * F}, x.options());
  if (M == 0) return {h, gu};
  constexpr int BN = 256;  // 128 gate + 128 up columns per tile: 128 columns of h
  const int dev = x.device().index();
  GemmParams p = base_params(static_cast<int>(M), static_cast<int>(F), static_cast<int>(K), BN, group_m, 0, 0, dev);
  p.tiles_n = static_cast<int>(F / (BN / 2));
  p.out = h.data_ptr();
  p.ldo = h.stride(0);
  p.aux = gu.data_ptr();
  p.ldx = gu.stride(0);
  p.ffn = static_cast<int>(F);
  const CUtensorMap ma = operand_map(x, kBK, kBM);
  const CUtensorMap mb = operand_map(w_gu, kBK, BN / 2);
  launch_pair<256, false, false, kEpiSwiGLU, false>(ma, mb, output_map(h), output_map(gu), p, dev,
                                                    at::cuda::getCurrentCUDAStream());
  return {h, gu};
}

// Input gradient of a SwiGLU MLP's down projection fused with the SwiGLU backward:
// dh = dy @ w_down (w_down = [D, F]), then d[gate|up] from the saved bf16 gate|up.  Returns
// dgu [M, 2F] bf16.
at::Tensor gemm_swiglu_bwd(at::Tensor dy, at::Tensor w_down, at::Tensor gu, int64_t group_m) {
  check_operand(dy, "dy");
  check_operand(w_down, "w_down");
  check_operand(gu, "gu");
  TORCH_CHECK(dy.dim() == 2 && w_down.dim() == 2 && gu.dim() == 2, "dy, w_down and gu must be matrices");
  const int64_t M = dy.size(0), D = dy.size(1), F = w_down.size(1);
  TORCH_CHECK(w_down.size(0) == D && gu.size(0) == M && gu.size(1) == 2 * F, "shapes: dy [M, D], w_down [D, F], gu [M, 2F]");
  TORCH_CHECK(F % 32 == 0, "F must be a multiple of 32");
  const c10::cuda::CUDAGuard guard(dy.device());
  at::Tensor dgu = at::empty({M, 2 * F}, dy.options());
  if (M == 0) return dgu;
  const int dev = dy.device().index();
  GemmParams p = base_params(static_cast<int>(M), static_cast<int>(F), static_cast<int>(D), 256, group_m, 0, 0, dev);
  p.out = dgu.data_ptr();
  p.ldo = dgu.stride(0);
  p.aux = gu.data_ptr();
  p.ldx = gu.stride(0);
  p.ffn = static_cast<int>(F);
  const CUtensorMap ma = operand_map(dy, kBK, kBM);
  const CUtensorMap mb = operand_map(w_down, 64, kBK);
  const CUtensorMap mo = output_map(dgu);
  launch_pair<256, false, true, kEpiSwiGLUBwd, false>(ma, mb, mo, mo, p, dev, at::cuda::getCurrentCUDAStream());
  return dgu;
}

// y = x @ W^T for a weight W [n_rows, K] sharded by rows over len(shard_ptrs) ranks of one node
// (rank k's rows at shard_ptrs[k], contiguous [n_rows / world, K] bf16, mapped on this GPU), with
// the whole of W gathered into `g` [n_rows, K] as a by-product.  `flags` (int32 [n_rows / 128],
// zero before the first call) persists across calls with the same `g`; `epoch` counts those
// calls from 1.  The shards must not change while any rank's call runs.
at::Tensor gemm_allgather(at::Tensor x, std::vector<int64_t> shard_ptrs, int64_t rank, at::Tensor g, at::Tensor flags,
                          int64_t epoch, int64_t wait_ns) {
  check_operand(x, "x");
  check_operand(g, "g");
  const int64_t world = static_cast<int64_t>(shard_ptrs.size());
  TORCH_CHECK(world >= 1 && world <= 8 && rank >= 0 && rank < world, "1 to 8 shards, 0 <= rank < world");
  TORCH_CHECK(x.dim() == 2 && g.dim() == 2 && g.is_contiguous(), "x [M, K], g [N, K] contiguous");
  const int64_t M = x.size(0), K = x.size(1), N = g.size(0);
  TORCH_CHECK(g.size(1) == K, "g: [N, K]");
  TORCH_CHECK(N % 256 == 0 && N % (world * 128) == 0, "N must be a multiple of 256 and of 128 x world");
  TORCH_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "dimensions out of range");
  TORCH_CHECK(flags.is_cuda() && flags.scalar_type() == at::kInt && flags.is_contiguous() && flags.numel() == N / 128,
              "flags: int32 [N / 128]");
  TORCH_CHECK(epoch >= 1, "epoch counts calls from 1");
  const int64_t S = N / world;
  for (int64_t p : shard_ptrs) TORCH_CHECK(p % 16 == 0, "shard pointers must be 16-byte aligned");
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor y = at::empty({M, N}, x.options());
  constexpr int BN = 256;
  const int dev = x.device().index();
  GemmParams p = base_params(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), BN, 1, wait_ns, 0, dev);
  p.out = y.data_ptr();
  p.ldo = y.stride(0);
  auto kernel = gemm_gather_kernel<BN>;
  constexpr int smem = gather_smem<BN>();
  static bool attr[64] = {false};
  if (!attr[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  // Every resident pair runs (a pair without tiles still gathers), so the split of the rows into
  // items, and with it the counters' step per call, depends only on the device and the shape.
  const int pairs = resident_pairs(dev, reinterpret_cast<const void*>(kernel), smem);
  const int nkb = static_cast<int>((K + kBK - 1) / kBK);
  const int blocks = static_cast<int>(N / 128);
  const int parts = std::max(1, std::min(nkb, (2 * pairs + blocks - 1) / blocks));
  GatherArgs ga;
  std::memset(&ga, 0, sizeof(ga));
  for (int64_t k = 0; k < world; ++k)
    ga.shard[k] = make_tmap_bf16_3d(reinterpret_cast<const void*>(shard_ptrs[k]), 1, S, K, K, S * K, kBK, 128);
  ga.g = make_tmap_bf16_3d(g.data_ptr(), 1, N, K, K, N * K, kBK, 128);
  ga.flags = reinterpret_cast<unsigned*>(flags.data_ptr());
  ga.target = static_cast<unsigned>(static_cast<uint64_t>(epoch) * static_cast<uint64_t>(parts));
  ga.rank = static_cast<int>(rank);
  ga.world = static_cast<int>(world);
  ga.shard_rows = static_cast<int>(S);
  ga.parts = parts;
  const CUtensorMap ma = M > 0 ? operand_map(x, kBK, kBM) : ga.g;  // without rows the pairs only gather
  const CUtensorMap mo = M > 0 ? output_map(y) : ga.g;
  kernel<<<2 * pairs, kThreads, smem, at::cuda::getCurrentCUDAStream()>>>(ma, mo, ga, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

// Reads and clears the dense GEMM kernels' status word of `device` (0 = every wait completed).
int64_t gemm_status(int64_t device) {
  int* w = status_word(static_cast<int>(device));
  int host = 0;
  C10_CUDA_CHECK(cudaMemcpy(&host, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (host != 0) C10_CUDA_CHECK(cudaMemset(w, 0, sizeof(int)));
  return host;
}
