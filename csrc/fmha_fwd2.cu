// Prefix-LM flash attention forward for sm_100a, two query tiles per CTA (tcgen05 + TMEM + TMA).
//
// Same semantics as fmha_fwd.cu (a query row at sequence position r sees keys [0, P) if r < P,
// keys [0, r] otherwise; GQA; optional sigmoid(gate) epilogue; log2-domain LSE), but one CTA
// owns 256 query rows (tiles A and B) of one head, so every K/V block loaded by TMA feeds four
// MMAs and two independent softmax warpgroups keep the tensor core busy in turn:
//
//   tensor core:  S_A(0) S_B(0) | PV_A(0) S_A(1) | PV_B(0) S_B(1) | PV_A(1) S_A(2) | ...
//   softmax A:          [ P_A(0) ]      ...       [ P_A(1) ]
//   softmax B:                     [ P_B(0) ]                     [ P_B(1) ]
//
// TMEM (512 columns): S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512).  P_X is written
// as packed bf16 into the first 64 columns of S_X (tcgen05.st) and read from there as the A
// operand of O_X += P_X V (tcgen05.mma with A in tensor memory), so P never touches shared
// memory.  A new S_X is issued only after the PV that reads P_X, and P_X is only rewritten after
// that PV has completed (o_done), so the aliasing is ordered both ways.
//
// Warps (320 threads; with 3 warps on two of the four SM sub-partitions the register cap is 168 per
// thread): 0 TMA producer, 1 TMEM owner + MMA issuer, 2..5 softmax/epilogue of tile
// A, 6..9 softmax/epilogue of tile B (warp w reaches TMEM lanes 32*(w%4)..+31).  Lazy O
// rescaling (only when a row max grows by more than 2^8).  Every mbarrier wait is bounded
// (common.cuh); a timeout records a status code and all roles fall through to a teardown that
// drains their asynchronous work and frees TMEM.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tma.cuh"

using namespace mimir;

int* fmha_status_ptr(const at::Device& dev);

namespace {

constexpr int kTile = 128;
constexpr int kPair = 2 * kTile;
constexpr int kHeadDim = 128;
constexpr int kThreads = 320;
constexpr uint32_t kTileBytes = kTile * kHeadDim * 2;  // 32 KB
constexpr uint32_t kChunkBytes = kTileBytes / 2;       // one 64-column half
constexpr float kRescaleThreshold = 8.0f;
// Every kPolyEvery-th exponential pair is computed on the FMA pipe (poly_exp2) instead of MUFU;
// the kernel is instantiated for 0 (off), 2, 4 and 8 and MIMIR_FMHA2_POLY_EVERY selects; the default is
// 0: with two softmax warpgroups MUFU is not the limit and the polynomial costs issue slots (measured).

struct Fwd2Params {
  __nv_bfloat16* y;
  __nv_bfloat16* o;
  const __nv_bfloat16* gate;
  int64_t gate_ld;
  int gate_col;
  float* lse;
  int64_t lse_ld;
  const int* cu_seqlens;
  const int* prefix_lens;
  const int2* tiles;   // (sequence, 256-row block)
  const int* ntiles;
  int H, KV;
  int q_col, k_col, v_col;
  int is_causal;
  float scale_log2;
  int* status;
};

struct __align__(8) Barriers {
  uint64_t q_full;
  uint64_t k_full[2];
  uint64_t v_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full[2];   // per tile
  uint64_t p_full[2];   // per tile
  uint64_t o_done[2];   // per tile
  uint64_t mma_done;
  uint32_t tmem_base;
  int pad;
};

constexpr uint32_t kSmemQ = 0;                       // Q_A, then Q_B
constexpr uint32_t kSmemKV = 2 * kTileBytes;         // stage s: K at +2s*32K, V at +(2s+1)*32K
constexpr uint32_t kSmemBar = 6 * kTileBytes;
constexpr uint32_t kSmemBytes = kSmemBar + sizeof(Barriers) + 1024;

__device__ __forceinline__ uint8_t* q_tile(uint8_t* b, int x) { return b + kSmemQ + x * kTileBytes; }
__device__ __forceinline__ uint8_t* k_stage(uint8_t* b, int s) { return b + kSmemKV + 2 * s * kTileBytes; }
__device__ __forceinline__ uint8_t* v_stage(uint8_t* b, int s) { return k_stage(b, s) + kTileBytes; }

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]  (A K-major in tensor memory: row m at lane m, 2 bf16 per column)
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// 32 columns of 32-bit words into this warp's 32 lanes, without waiting.
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st32_u(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

template <int kPolyEvery>
__global__ void __launch_bounds__(kThreads, 1)
    fmha_fwd2_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const Fwd2Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bar = reinterpret_cast<Barriers*>(smem + kSmemBar);

  const int tile = blockIdx.y;
  if (tile >= *p.ntiles) return;  // CTA-uniform, before any allocation
  const int h = blockIdx.x;
  const int2 tq = p.tiles[tile];
  const int seq = tq.x;
  const int q0 = tq.y * kPair;
  const int start = p.cu_seqlens[seq];
  const int L = p.cu_seqlens[seq + 1] - start;
  const int P = p.is_causal ? 0 : p.prefix_lens[seq];
  const bool has_b = q0 + kTile < L;
  // key blocks needed by each tile (row limits are non-decreasing in the row index)
  auto nkv_of = [&](int first_row) {
    const int last = min(first_row + kTile - 1, L - 1);
    const int mx = last >= P ? last : P - 1;
    return mx / kTile + 1;
  };
  const int nkv_a = nkv_of(q0);
  const int nkv_b = has_b ? nkv_of(q0 + kTile) : 0;
  const int nkv = max(nkv_a, nkv_b);
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
      mbar_init(&bar->p_full[s], 4);
      mbar_init(&bar->o_done[s], 1);
    }
    mbar_init(&bar->mma_done, 1);
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
  auto tS = [tmem](int x) -> uint32_t { return tmem + x * 128; };
  auto tO = [tmem](int x) -> uint32_t { return tmem + 256 + x * 128; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int qx = p.q_col + h * kHeadDim;
      const int kx = p.k_col + kvh * kHeadDim;
      const int vx = p.v_col + kvh * kHeadDim;
      mbar_arrive_expect_tx(&bar->q_full, has_b ? 2 * kTileBytes : kTileBytes);
      for (int x = 0; x < (has_b ? 2 : 1); ++x) {
        tma_load_2d(q_tile(smem, x), &map_q, &bar->q_full, qx, start + q0 + x * kTile);
        tma_load_2d(q_tile(smem, x) + kChunkBytes, &map_q, &bar->q_full, qx + 64, start + q0 + x * kTile);
      }
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&bar->kv_empty[s], ((j >> 1) - 1) & 1, p.status, kStatusTimeoutEmpty)) break;
        const int row = start + j * kTile;
        mbar_arrive_expect_tx(&bar->k_full[s], kTileBytes);
        tma_load_2d(k_stage(smem, s), &map_k, &bar->k_full[s], kx, row);
        tma_load_2d(k_stage(smem, s) + kChunkBytes, &map_k, &bar->k_full[s], kx + 64, row);
        mbar_arrive_expect_tx(&bar->v_full[s], kTileBytes);
        tma_load_2d(v_stage(smem, s), &map_v, &bar->v_full[s], vx, row);
        tma_load_2d(v_stage(smem, s) + kChunkBytes, &map_v, &bar->v_full[s], vx + 64, row);
        issued = j + 1;
      }
      // Teardown: no TMA write into this CTA's shared memory may still be in flight.
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
      auto issue_s = [&](int x, int j) {
        const uint32_t sq = smem_u32(q_tile(smem, x));
        const uint32_t sk = smem_u32(k_stage(smem, j & 1));
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kChunkBytes + (k & 3) * 32;
          mma_ss(tS(x), smem_desc(sq + off, 16, 1024, kLayoutSW128), smem_desc(sk + off, 16, 1024, kLayoutSW128),
                 idesc_qk, k > 0 ? 1u : 0u);
        }
        mma_commit(&bar->s_full[x]);
      };
      auto issue_pv = [&](int x, int j) {
        const uint32_t sv = smem_u32(v_stage(smem, j & 1));
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          // A = P_x: 16 keys = 8 packed columns of S_x; B = V (MN-major over head_dim):
          // 16 key rows = 2048 bytes, the second 64-wide head_dim half sits 16 KB further (LBO).
          mma_ts(tO(x), tS(x) + k * 8, smem_desc(sv + k * 2048, kChunkBytes, 1024, kLayoutSW128), idesc_pv,
                 (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&bar->o_done[x]);
      };
      bool ok = mbar_wait(&bar->q_full, 0, p.status, kStatusTimeoutQ) &&
                mbar_wait(&bar->k_full[0], 0, p.status, kStatusTimeoutKV);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        if (has_b) issue_s(1, 0);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int s = j & 1;
        bool v_ready = false, k_ready = false;
        for (int x = 0; x < 2 && ok; ++x) {
          const int nx = x == 0 ? nkv_a : nkv_b;
          if (j >= nx) continue;
          if (!mbar_wait(&bar->p_full[x], j & 1, p.status, kStatusTimeoutP)) { ok = false; break; }
          if (!v_ready && !mbar_wait(&bar->v_full[s], (j >> 1) & 1, p.status, kStatusTimeoutKV)) { ok = false; break; }
          v_ready = true;
          tc_fence_after();
          issue_pv(x, j);
          if (j + 1 < nx) {
            if (!k_ready && !mbar_wait(&bar->k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, p.status, kStatusTimeoutKV)) {
              ok = false;
              break;
            }
            k_ready = true;
            tc_fence_after();
            issue_s(x, j + 1);
          }
        }
        if (ok) mma_commit(&bar->kv_empty[s]);  // every MMA reading stage s has been issued
      }
      // Teardown: every MMA issued by this thread completes before TMEM is released.
      mma_commit(&bar->mma_done);
      mbar_wait(&bar->mma_done, 0, p.status, kStatusTimeoutOther);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (tile x)
    const int x = (warp - 2) >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const int row0 = q0 + x * kTile;
    const int qpos = row0 + r;
    const int lim = qpos < P ? P - 1 : qpos;
    const int min_lim = row0 < P ? P - 1 : row0;
    const int my_nkv = x == 0 ? nkv_a : nkv_b;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    float m_i = -INFINITY, l_i = 0.f;
    bool ok = true;
    for (int j = 0; j < my_nkv; ++j) {
      if (!warp_wait(&bar->s_full[x], j & 1, p.status, kStatusTimeoutS)) { ok = false; break; }
      tc_fence_after();
      float sv[128];
      {
        uint32_t raw[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32_nowait(tS(x) + lane_off + c * 32, raw[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(raw[c][i]);
      }
      const int k0 = j * kTile;
      if (k0 + kTile - 1 > min_lim) {
        const int rel = lim - k0;
#pragma unroll
        for (int c = 0; c < 128; ++c) sv[c] = c > rel ? -INFINITY : sv[c];
      }
      float mxp[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mxp[e] = sv[e];
#pragma unroll
      for (int c = 8; c < 128; c += 8)
#pragma unroll
        for (int e = 0; e < 8; ++e) mxp[e] = fmaxf(mxp[e], sv[c + e]);
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
      // P_x(j) overwrites the columns PV_x(j-1) reads, and a rescale touches O_x: both wait for it.
      if (j > 0) {
        if (!warp_wait(&bar->o_done[x], (j - 1) & 1, p.status, kStatusTimeoutO)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffff, rescale)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float ov[32];
            tmem_ld32(tO(x) + lane_off + c * 32, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= alpha;
            tmem_st32(tO(x) + lane_off + c * 32, ov);
          }
        }
      }
      tmem_st32_u(tS(x) + lane_off, pk);
      tmem_st32_u(tS(x) + lane_off + 32, pk + 32);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->p_full[x]);
    }
    if (ok && my_nkv > 0 && warp_wait(&bar->o_done[x], (my_nkv - 1) & 1, p.status, kStatusTimeoutO)) {
      tc_fence_after();
      const bool valid = qpos < L;
      const int64_t grow = (int64_t)start + qpos;
      const float inv_l = 1.f / l_i;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(tO(x) + lane_off + c * 32, ov);
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

// Tile schedule over 256-row query blocks, heaviest (most key blocks) first.
constexpr int kMaxBuckets = 1024;

__global__ void build_pair_tiles_kernel(const int* __restrict__ cu, const int* __restrict__ prefix, int nseq,
                                        int is_causal, int2* __restrict__ tiles, int* __restrict__ ntiles,
                                        int max_tiles) {
  __shared__ int hist[kMaxBuckets];
  __shared__ int total;
  for (int i = threadIdx.x; i < kMaxBuckets; i += blockDim.x) hist[i] = 0;
  if (threadIdx.x == 0) total = 0;
  __syncthreads();
  auto work = [&](int s, int qb) {
    const int L = cu[s + 1] - cu[s];
    const int P = is_causal ? 0 : prefix[s];
    const int last = min(qb * kPair + kPair - 1, L - 1);
    const int mx = last >= P ? last : P - 1;
    return min(mx / kTile + 1, kMaxBuckets) - 1;
  };
  for (int s = threadIdx.x; s < nseq; s += blockDim.x) {
    const int nq = (cu[s + 1] - cu[s] + kPair - 1) / kPair;
    for (int qb = 0; qb < nq; ++qb) atomicAdd(&hist[work(s, qb)], 1);
    atomicAdd(&total, nq);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = kMaxBuckets - 1; b >= 0; --b) {
      const int c = hist[b];
      hist[b] = acc;
      acc += c;
    }
    *ntiles = min(total, max_tiles);
  }
  __syncthreads();
  for (int s = threadIdx.x; s < nseq; s += blockDim.x) {
    const int nq = (cu[s + 1] - cu[s] + kPair - 1) / kPair;
    for (int qb = 0; qb < nq; ++qb) {
      const int pos = atomicAdd(&hist[work(s, qb)], 1);
      if (pos < max_tiles) tiles[pos] = make_int2(s, qb);
    }
  }
}

}  // namespace

std::vector<at::Tensor> fmha_plan2(at::Tensor cu_seqlens, at::Tensor prefix_lens, int64_t numseqs,
                                   int64_t total_tokens, bool is_causal) {
  TORCH_CHECK(cu_seqlens.is_cuda() && cu_seqlens.scalar_type() == at::kInt);
  TORCH_CHECK(prefix_lens.scalar_type() == at::kInt);
  c10::cuda::CUDAGuard guard(cu_seqlens.device());
  const int64_t max_tiles = (total_tokens + kPair - 1) / kPair + numseqs;
  auto tiles = at::empty({std::max<int64_t>(max_tiles, 1), 2}, cu_seqlens.options());
  auto ntiles = at::zeros({1}, cu_seqlens.options());
  if (numseqs > 0) {
    build_pair_tiles_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
        cu_seqlens.data_ptr<int>(), prefix_lens.data_ptr<int>(), (int)numseqs, is_causal ? 1 : 0,
        reinterpret_cast<int2*>(tiles.data_ptr<int>()), ntiles.data_ptr<int>(), (int)max_tiles);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {tiles, ntiles};
}

std::vector<at::Tensor> fmha_fwd2(at::Tensor q_src, int64_t q_col, at::Tensor k_src, int64_t k_col, at::Tensor v_src,
                                  int64_t v_col, c10::optional<at::Tensor> gate_src, int64_t gate_col, int64_t H,
                                  int64_t KV, bool is_causal, at::Tensor cu_seqlens, at::Tensor prefix_lens,
                                  int64_t numseqs, at::Tensor tiles, at::Tensor ntiles) {
  for (const at::Tensor* t : {&q_src, &k_src, &v_src}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 2 && t->stride(1) == 1,
                "fmha_fwd2: q/k/v sources must be 2-D bf16 row-major CUDA tensors");
  }
  TORCH_CHECK(H % KV == 0, "fmha_fwd2: H must be a multiple of KV");
  TORCH_CHECK(q_col % 8 == 0 && k_col % 8 == 0 && v_col % 8 == 0, "fmha_fwd2: column offsets must be 16-byte aligned");
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

  Fwd2Params prm{};
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
  prm.status = fmha_status_ptr(q_src.device());

  static const int poly = [] {
    const char* env = std::getenv("MIMIR_FMHA2_POLY_EVERY");
    const int v = env != nullptr ? std::atoi(env) : 0;
    TORCH_CHECK(v == 0 || v == 2 || v == 4 || v == 8, "MIMIR_FMHA2_POLY_EVERY must be 0, 2, 4 or 8");
    return v;
  }();
  auto kernel = poly == 0 ? fmha_fwd2_kernel<0> : poly == 2 ? fmha_fwd2_kernel<2>
              : poly == 8 ? fmha_fwd2_kernel<8> : fmha_fwd2_kernel<4>;
  static bool attr_set[16] = {false};
  if (!attr_set[q_src.device().index()]) {
    for (auto k : {fmha_fwd2_kernel<0>, fmha_fwd2_kernel<2>, fmha_fwd2_kernel<4>, fmha_fwd2_kernel<8>})
      C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    attr_set[q_src.device().index()] = true;
  }
  dim3 grid((unsigned)H, (unsigned)tiles.size(0));
  kernel<<<grid, kThreads, kSmemBytes, at::cuda::getCurrentCUDAStream()>>>(mq, mk, mv, prm);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return gated ? std::vector<at::Tensor>{y, lse, o} : std::vector<at::Tensor>{y, lse};
}
