// Single-pass prefix-LM flash attention backward for sm_100a (tcgen05 + TMEM + TMA).
//
// One CTA owns a 128-key block of one KV head of one packed sequence and loops over every
// (query head of its GQA group, 64-row query block) pair that can see those keys:
//   S^T  = K Q^T        (M=128 keys, N=64 queries)          -> TMEM
//   dP^T = V dO^T       (M=128 keys, N=64 queries)          -> TMEM
//   P^T  = exp2(S^T * scale*log2e - LSE2[q]) (masked), dS^T = P^T * (dP^T - Delta[q])  (softmax warps)
//   dV  += P^T dO       (M=128 keys, N=128, K=64)            TMEM accumulator
//   dK  += dS^T Q       (M=128 keys, N=128, K=64)            TMEM accumulator
//   dQ^T = K^T dS^T     (M=128 head dims, N=64 queries, K=128 keys) -> TMEM; the dQ warps
//          transpose it into a [64 x 128] fp32 smem tile that one TMA reduce-add folds into
//          the global dQ (L2-side line reductions instead of per-element atomics: reductions
//          issued straight from registers, 32 head dims per warp instruction, made the whole
//          backward 1.68 ms instead of 1.01 ms on the 16k-token bench shape).
// dK/dV are written once per CTA (bf16, no atomics) because the CTA covers all query heads
// that share its KV head.  TMEM: S^T 64 + dP^T 64 + dQ^T 64 + dV 128 + dK 128 = 448 columns.
//
// Warp roles (448 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA issuer,
// warps 2..9 softmax (thread = key row; warps w and w+4 split the 64 query columns, so each
// SM sub-partition runs two softmax warps), warps 10..13 dQ drain (thread = head dim).
// All waits are bounded (common.cuh) and the teardown drains async work before freeing TMEM.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tma.cuh"

using namespace mimir;

namespace {

constexpr int kKeys = 128;     // keys per CTA
constexpr int kQRows = 64;     // query rows per block
constexpr int kHeadDim = 128;
constexpr int kThreads = 448;  // 14 warps
constexpr uint32_t kKVBytes = kKeys * kHeadDim * 2;        // 32 KB
constexpr uint32_t kKVChunk = kKVBytes / 2;                // [128 keys][64 dims] = 16 KB
constexpr uint32_t kQBytes = kQRows * kHeadDim * 2;        // 16 KB
constexpr uint32_t kQChunk = kQBytes / 2;                  // [64 rows][64 dims] = 8 KB
constexpr uint32_t kPBytes = kKeys * kQRows * 2;           // 16 KB
constexpr int kStages = 3;                                  // Q/dO ring depth

struct BwdParams {
  float* dq;                   // [T, H*128] fp32, pre-zeroed; receives scale * dS K
  __nv_bfloat16* dk;           // [T, KV*128]
  __nv_bfloat16* dv;           // [T, KV*128]
  const float* lse;            // [H, lse_ld] log2 domain
  const float* delta;          // [H, lse_ld]
  int64_t lse_ld;
  const int* cu_seqlens;
  const int* prefix_lens;
  const int2* tiles;           // (sequence, key block)
  const int* ntiles;
  int H, KV;
  int q_col, k_col, v_col;
  int is_causal;
  float scale_log2;            // log2(e) / sqrt(128)
  float scale;                 // 1 / sqrt(128)
  int* status;
};

struct __align__(8) Barriers {
  uint64_t kv_full;
  uint64_t qdo_full[3];
  uint64_t qdo_empty[3];
  uint64_t sdp_full;
  uint64_t s_free;
  uint64_t ds_ready;
  uint64_t pds_free;
  uint64_t dq_full[2];     // per TMEM dQ^T buffer
  uint64_t dq_free[2];
  uint64_t acc_full;
  uint64_t mma_done;
  uint64_t dqs_full[2];    // 4 dQ warps wrote staging tile b
  uint64_t dqs_free[2];    // the TMA reduce finished reading staging tile b
  uint32_t tmem_base;
  int pad;
};

constexpr uint32_t kSmemK = 0;
constexpr uint32_t kSmemV = kKVBytes;
constexpr uint32_t kSmemQ0 = 2 * kKVBytes;                       // Q stage s at kSmemQ0 + s * 2 * kQBytes
constexpr uint32_t kSmemP = kSmemQ0 + 2 * kStages * kQBytes;
constexpr uint32_t kSmemDS = kSmemP + kPBytes;
constexpr uint32_t kSmemDQ = kSmemDS + kPBytes;                  // 2 x [32 rows][128] fp32 staging tiles
constexpr int kDqRows = 32;                                         // rows per TMA reduce
constexpr uint32_t kDqTileBytes = kDqRows * kHeadDim * 4;           // 16 KB
constexpr uint32_t kSmemBar = kSmemDQ + 2 * kDqTileBytes;
constexpr uint32_t kSmemBytes = kSmemBar + sizeof(Barriers) + 1024;

__device__ __forceinline__ uint8_t* q_stage(uint8_t* b, int s) { return b + kSmemQ0 + s * 2 * kQBytes; }
__device__ __forceinline__ uint8_t* do_stage(uint8_t* b, int s) { return q_stage(b, s) + kQBytes; }

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// tcgen05.ld of 32 columns for the 32 lanes of this warp's quarter (ld + wait fused).
__device__ __forceinline__ void ld32(uint32_t taddr, float (&v)[32]) { tmem_ld32(taddr, v); }

__global__ void __launch_bounds__(kThreads, 1)
    fmha_bwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_do,
                    const __grid_constant__ CUtensorMap map_dq, const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bar = reinterpret_cast<Barriers*>(smem + kSmemBar);

  const int tile = blockIdx.y;
  if (tile >= *p.ntiles) return;
  const int kvh = blockIdx.x;
  const int2 tk = p.tiles[tile];
  const int seq = tk.x;
  const int k0 = tk.y * kKeys;
  const int start = p.cu_seqlens[seq];
  const int L = p.cu_seqlens[seq + 1] - start;
  const int P = p.is_causal ? 0 : p.prefix_lens[seq];
  const int group = p.H / p.KV;
  // Query rows that can see any key of this block: all rows if the block touches the prompt,
  // otherwise rows >= k0 (causal).
  const int qfirst_block = (k0 < P) ? 0 : k0 / kQRows;
  const int nqb = (L + kQRows - 1) / kQRows - qfirst_block;
  const int n = group * max(nqb, 0);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bar->kv_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar->qdo_full[s], 1);
      mbar_init(&bar->qdo_empty[s], 1);
    }
    mbar_init(&bar->sdp_full, 1);
    mbar_init(&bar->s_free, 8);
    mbar_init(&bar->ds_ready, 8);
    mbar_init(&bar->pds_free, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar->dq_full[b], 1);
      mbar_init(&bar->dq_free[b], 4);
      mbar_init(&bar->dqs_full[b], 4);
      mbar_init(&bar->dqs_free[b], 1);
    }
    mbar_init(&bar->acc_full, 1);
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
    tma_prefetch_desc(&map_do);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  // TMEM columns: S^T 0-63, dP^T 64-127, dQ^T buffers 128-191 and 448-511, dV 192-319, dK 320-447.
  const uint32_t tS = tmem, tdP = tmem + 64, tdV = tmem + 192, tdK = tmem + 320;
  auto tdQb = [tmem](int b) -> uint32_t { return b ? tmem + 448 : tmem + 128; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int kx = p.k_col + kvh * kHeadDim, vx = p.v_col + kvh * kHeadDim;
      mbar_arrive_expect_tx(&bar->kv_full, 2 * kKVBytes);
      tma_load_2d(smem + kSmemK, &map_k, &bar->kv_full, kx, start + k0);
      tma_load_2d(smem + kSmemK + kKVChunk, &map_k, &bar->kv_full, kx + 64, start + k0);
      tma_load_2d(smem + kSmemV, &map_v, &bar->kv_full, vx, start + k0);
      tma_load_2d(smem + kSmemV + kKVChunk, &map_v, &bar->kv_full, vx + 64, start + k0);
      int issued = 0;
      for (int i = 0; i < n; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait(&bar->qdo_empty[s], ((i / kStages) - 1) & 1, p.status, kStatusTimeoutEmpty))
          break;
        const int hq = kvh * group + i / nqb;
        const int row = start + (qfirst_block + i % nqb) * kQRows;
        const int qx = p.q_col + hq * kHeadDim, dox = hq * kHeadDim;
        mbar_arrive_expect_tx(&bar->qdo_full[s], 2 * kQBytes);
        tma_load_2d(q_stage(smem, s), &map_q, &bar->qdo_full[s], qx, row);
        tma_load_2d(q_stage(smem, s) + kQChunk, &map_q, &bar->qdo_full[s], qx + 64, row);
        tma_load_2d(do_stage(smem, s), &map_do, &bar->qdo_full[s], dox, row);
        tma_load_2d(do_stage(smem, s) + kQChunk, &map_do, &bar->qdo_full[s], dox + 64, row);
        issued = i + 1;
      }
      mbar_wait(&bar->kv_full, 0, p.status, kStatusTimeoutKV);
      for (int i = max(0, issued - kStages); i < issued; ++i)
        mbar_wait(&bar->qdo_full[i % kStages], (i / kStages) & 1, p.status, kStatusTimeoutQ);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16_f32(128, 64, 0, 0);    // S^T, dP^T
      const uint32_t id_acc = idesc_bf16_f32(128, 128, 0, 1); // dV, dK (B MN-major)
      const uint32_t id_dq = idesc_bf16_f32(128, 64, 1, 1);   // dQ^T (A and B MN-major)
      const uint32_t sk = smem_u32(smem + kSmemK), sv = smem_u32(smem + kSmemV);
      const uint32_t sp = smem_u32(smem + kSmemP), sds = smem_u32(smem + kSmemDS);
      bool ok = mbar_wait(&bar->kv_full, 0, p.status, kStatusTimeoutKV);
      // S^T/dP^T of block i+1 are issued before dV/dK/dQ of block i, so the softmax warps work
      // on block i+1 while the tensor core runs block i's accumulations.
      auto issue_sdp = [&](int i) -> bool {
        const int s = i % kStages;
        if (!mbar_wait(&bar->qdo_full[s], (i / kStages) & 1, p.status, kStatusTimeoutQ)) return false;
        if (i > 0 && !mbar_wait(&bar->s_free, (i - 1) & 1, p.status, kStatusTimeoutS)) return false;
        tc_fence_after();
        const uint32_t sq = smem_u32(q_stage(smem, s)), sdo = smem_u32(do_stage(smem, s));
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t ka = (k >> 2) * kKVChunk + (k & 3) * 32;
          const uint32_t kb = (k >> 2) * kQChunk + (k & 3) * 32;
          mma_ss(tS, smem_desc(sk + ka, 16, 1024, kLayoutSW128), smem_desc(sq + kb, 16, 1024, kLayoutSW128), id_s,
                 k > 0);
          mma_ss(tdP, smem_desc(sv + ka, 16, 1024, kLayoutSW128), smem_desc(sdo + kb, 16, 1024, kLayoutSW128), id_s,
                 k > 0);
        }
        mma_commit(&bar->sdp_full);
        return true;
      };
      if (ok && n > 0) ok = issue_sdp(0);
      for (int i = 0; ok && i < n; ++i) {
        const int s = i % kStages;
        if (i + 1 < n && !issue_sdp(i + 1)) { ok = false; break; }
        if (!mbar_wait(&bar->ds_ready, i & 1, p.status, kStatusTimeoutP)) { ok = false; break; }
        if (i >= 2 && !mbar_wait(&bar->dq_free[i & 1], ((i >> 1) - 1) & 1, p.status, kStatusTimeoutO)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sq = smem_u32(q_stage(smem, s)), sdo = smem_u32(do_stage(smem, s));
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // K-dim = 64 queries
          const uint64_t a_p = smem_desc(sp + k * 32, 16, 1024, kLayoutSW128);
          const uint64_t a_ds = smem_desc(sds + k * 32, 16, 1024, kLayoutSW128);
          const uint64_t b_do = smem_desc(sdo + k * 2048, kQChunk, 1024, kLayoutSW128);
          const uint64_t b_q = smem_desc(sq + k * 2048, kQChunk, 1024, kLayoutSW128);
          mma_ss(tdV, a_p, b_do, id_acc, (i > 0 || k > 0));
          mma_ss(tdK, a_ds, b_q, id_acc, (i > 0 || k > 0));
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // K-dim = 128 keys
          const uint64_t a_kt = smem_desc(sk + k * 2048, kKVChunk, 1024, kLayoutSW128);
          const uint64_t b_ds = smem_desc(sds + k * 2048, kPBytes, 1024, kLayoutSW128);
          mma_ss(tdQb(i & 1), a_kt, b_ds, id_dq, k > 0);
        }
        mma_commit(&bar->dq_full[i & 1]);
        mma_commit(&bar->pds_free);
        mma_commit(&bar->qdo_empty[s]);
      }
      mma_commit(&bar->acc_full);
      mma_commit(&bar->mma_done);
      mbar_wait(&bar->mma_done, 0, p.status, kStatusTimeoutOther);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ softmax / dS (thread = key row)
    const int wq = warp & 3;
    const int half = (warp - 2) >> 2;        // which 32 query columns this warp owns
    const int r = wq * 32 + lane;
    const int key = k0 + r;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t col_off = half * 32;
    const uint32_t sP = smem_u32(smem + kSmemP);
    const uint32_t sDS = smem_u32(smem + kSmemDS);
    // LSE / Delta of this warp's 32 queries live in registers (lane l holds query 32*half + l)
    // and are fetched one iteration ahead to hide the global latency.
    auto fetch = [&](int i, float& lse2, float& dl) {
      const int hq = kvh * group + i / nqb;
      const int q0 = (qfirst_block + i % nqb) * kQRows;
      const int64_t idx = (int64_t)hq * p.lse_ld + start + min(q0 + (int)col_off + lane, L - 1);
      lse2 = p.lse[idx];
      dl = p.delta[idx];
    };
    float cur_lse = 0.f, cur_dl = 0.f, nxt_lse = 0.f, nxt_dl = 0.f;
    if (n > 0) fetch(0, cur_lse, cur_dl);
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int q0 = (qfirst_block + i % nqb) * kQRows;
      if (i + 1 < n) fetch(i + 1, nxt_lse, nxt_dl);
      if (!warp_wait(&bar->sdp_full, i & 1, p.status, kStatusTimeoutS)) { ok = false; break; }
      tc_fence_after();
      float sv[32], dpv[32];
      ld32(tS + lane_off + col_off, sv);
      ld32(tdP + lane_off + col_off, dpv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->s_free);
      uint32_t pk[16], dk[16];
      // Branch-free element loop: masked entries get an exponent argument of -inf (exp2 -> 0), so
      // the compiler keeps one basic block and interleaves the 32 independent element chains.
      const bool full = (q0 + kQRows <= L) && (k0 + kKeys - 1 <= (q0 < P ? P - 1 : q0));
      const int qbase = q0 + (int)col_off;
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        float pe[2], de[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = c + e;
          const float lse_c = __shfl_sync(0xffffffffu, cur_lse, col);
          const float dl_c = __shfl_sync(0xffffffffu, cur_dl, col);
          const int q = qbase + col;
          const int lim = q < P ? P - 1 : q;
          const bool vis = full | ((q < L) & (key <= lim));
          const float arg = vis ? fmaf(sv[col], p.scale_log2, -lse_c) : -INFINITY;
          const float pv = fast_exp2(arg);
          pe[e] = pv;
          de[e] = pv * (dpv[col] - dl_c);
        }
        pk[c >> 1] = pack_bf16x2(pe[0], pe[1]);
        dk[c >> 1] = pack_bf16x2(de[0], de[1]);
      }
      if (i > 0 && !warp_wait(&bar->pds_free, (i - 1) & 1, p.status, kStatusTimeoutP)) { ok = false; break; }
#pragma unroll
      for (int u4 = 0; u4 < 4; ++u4) {
        const int u = half * 4 + u4;  // 16-byte unit of the 128-byte row
        const uint32_t off = r * 128 + ((u ^ (r & 7)) << 4);
        st_shared_v4(sP + off, pk[4 * u4], pk[4 * u4 + 1], pk[4 * u4 + 2], pk[4 * u4 + 3]);
        st_shared_v4(sDS + off, dk[4 * u4], dk[4 * u4 + 1], dk[4 * u4 + 2], dk[4 * u4 + 3]);
      }
      fence_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->ds_ready);
      cur_lse = nxt_lse, cur_dl = nxt_dl;
    }
    // Epilogue: dK (scaled) and dV rows of this key block.
    if (ok && warp_wait(&bar->acc_full, 0, p.status, kStatusTimeoutO)) {
      tc_fence_after();
      const bool valid = key < L;
      const int64_t row = (int64_t)start + key;
      {
        const int which = half;  // half-0 warps write dK, half-1 warps write dV
        const uint32_t tacc = which == 0 ? tdK : tdV;
        __nv_bfloat16* out = which == 0 ? p.dk : p.dv;
        const float mul = which == 0 ? p.scale : 1.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          ld32(tacc + lane_off + c * 32, v);
          if (valid && n > 0) {
            uint4* dst = reinterpret_cast<uint4*>(out + row * (int64_t)p.KV * kHeadDim + kvh * kHeadDim + c * 32);
#pragma unroll
            for (int w = 0; w < 4; ++w)
              dst[w] = make_uint4(pack_bf16x2(v[8 * w] * mul, v[8 * w + 1] * mul),
                                  pack_bf16x2(v[8 * w + 2] * mul, v[8 * w + 3] * mul),
                                  pack_bf16x2(v[8 * w + 4] * mul, v[8 * w + 5] * mul),
                                  pack_bf16x2(v[8 * w + 6] * mul, v[8 * w + 7] * mul));
          } else if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(out + row * (int64_t)p.KV * kHeadDim + kvh * kHeadDim + c * 32);
#pragma unroll
            for (int w = 0; w < 4; ++w) dst[w] = make_uint4(0, 0, 0, 0);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ dQ drain (thread = head dim)
    const int wq = warp & 3;
    const int d = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t sdq_addr = smem_u32(smem + kSmemDQ);
    const bool issuer = (warp == 10 && lane == 0);
    bool pending = false;
    for (int i = 0; i < n; ++i) {
      const int hq = kvh * group + i / nqb;
      const int q0 = (qfirst_block + i % nqb) * kQRows;
      const int b = i & 1;
      if (!warp_wait(&bar->dq_full[b], (i >> 1) & 1, p.status, kStatusTimeoutO)) break;
      tc_fence_after();
      float a[32], c2[32];
      ld32(tdQb(b) + lane_off, a);
      ld32(tdQb(b) + lane_off + 32, c2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->dq_free[b]);
      // Two 32-row halves, alternating between two 16 KB staging tiles: transpose a half into
      // [query][dim] and fold it into global dQ with one TMA reduce-add; the reduce of the
      // previous half overlaps the staging of this one.
      bool issued_ok = true;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int ph = 2 * i + h2;   // staging phase
        const int sb = ph & 1;       // staging tile
        if (ph >= 2 && !warp_wait(&bar->dqs_free[sb], ((ph >> 1) - 1) & 1, p.status, kStatusTimeoutOther)) {
          issued_ok = false;
          break;
        }
        const uint32_t tile = sdq_addr + sb * kDqTileBytes;
        const float* src = h2 == 0 ? a : c2;
#pragma unroll
        for (int c = 0; c < 32; ++c)
            st_shared_f32(tile + (c * kHeadDim + d) * 4, (q0 + 32 * h2 + c < L) ? src[c] * p.scale : 0.f);
        fence_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->dqs_full[sb]);
        bool ok2 = true;
        if (issuer) {
          ok2 = mbar_wait(&bar->dqs_full[sb], (ph >> 1) & 1, p.status, kStatusTimeoutOther);
          if (ok2) {
            tma_reduce_add_2d(&map_dq, smem + kSmemDQ + sb * kDqTileBytes, hq * kHeadDim, start + q0 + 32 * h2);
            bulk_commit_group();
            pending = true;
            if (ph >= 1) {
              bulk_wait_group_read1();          // the previous phase's reduce has read its tile
              mbar_arrive(&bar->dqs_free[sb ^ 1]);
            }
          }
        }
        if (!__shfl_sync(0xffffffffu, ok2 ? 1 : 0, 0)) { issued_ok = false; break; }
      }
      if (!issued_ok) break;
    }
    if (issuer && pending) bulk_wait_group0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Key-block schedule for the backward: (sequence, key block) ordered by decreasing number of
// query blocks that see the block.
constexpr int kMaxBuckets = 2048;

__global__ void build_kv_tiles_kernel(const int* __restrict__ cu, const int* __restrict__ prefix, int nseq,
                                      int is_causal, int2* __restrict__ tiles, int* __restrict__ ntiles,
                                      int max_tiles) {
  __shared__ int hist[kMaxBuckets];
  __shared__ int total;
  for (int i = threadIdx.x; i < kMaxBuckets; i += blockDim.x) hist[i] = 0;
  if (threadIdx.x == 0) total = 0;
  __syncthreads();
  auto work = [&](int s, int kb) {
    const int L = cu[s + 1] - cu[s];
    const int P = is_causal ? 0 : prefix[s];
    const int k0 = kb * kKeys;
    const int first = k0 < P ? 0 : k0 / kQRows;
    const int nq = (L + kQRows - 1) / kQRows - first;
    return min(max(nq, 1), kMaxBuckets) - 1;
  };
  for (int s = threadIdx.x; s < nseq; s += blockDim.x) {
    const int L = cu[s + 1] - cu[s];
    const int nk = (L + kKeys - 1) / kKeys;
    for (int kb = 0; kb < nk; ++kb) atomicAdd(&hist[work(s, kb)], 1);
    atomicAdd(&total, nk);
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
    const int L = cu[s + 1] - cu[s];
    const int nk = (L + kKeys - 1) / kKeys;
    for (int kb = 0; kb < nk; ++kb) {
      const int pos = atomicAdd(&hist[work(s, kb)], 1);
      if (pos < max_tiles) tiles[pos] = make_int2(s, kb);
    }
  }
}

}  // namespace

int* fmha_status_ptr(const at::Device& dev);  // fmha_fwd.cu

std::vector<at::Tensor> fmha_bwd_plan(at::Tensor cu_seqlens, at::Tensor prefix_lens, int64_t numseqs,
                                      int64_t total_tokens, bool is_causal) {
  c10::cuda::CUDAGuard guard(cu_seqlens.device());
  const int64_t max_tiles = (total_tokens + kKeys - 1) / kKeys + numseqs;
  auto tiles = at::empty({std::max<int64_t>(max_tiles, 1), 2}, cu_seqlens.options());
  auto ntiles = at::zeros({1}, cu_seqlens.options());
  if (numseqs > 0) {
    build_kv_tiles_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
        cu_seqlens.data_ptr<int>(), prefix_lens.data_ptr<int>(), (int)numseqs, is_causal ? 1 : 0,
        reinterpret_cast<int2*>(tiles.data_ptr<int>()), ntiles.data_ptr<int>(), (int)max_tiles);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {tiles, ntiles};
}

// Returns {dq (fp32), dk (bf16), dv (bf16)}.
std::vector<at::Tensor> fmha_bwd(at::Tensor q_src, int64_t q_col, at::Tensor k_src, int64_t k_col, at::Tensor v_src,
                                 int64_t v_col, at::Tensor d_o, at::Tensor lse, at::Tensor delta, int64_t H,
                                 int64_t KV, bool is_causal, at::Tensor cu_seqlens, at::Tensor prefix_lens,
                                 int64_t numseqs, at::Tensor kv_tiles, at::Tensor kv_ntiles) {
  for (const at::Tensor* t : {&q_src, &k_src, &v_src, &d_o}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 2 && t->stride(1) == 1,
                "fmha_bwd: q/k/v/dO must be 2-D bf16 row-major CUDA tensors");
  }
  TORCH_CHECK(d_o.size(1) == H * kHeadDim && d_o.is_contiguous());
  TORCH_CHECK(q_col % 8 == 0 && k_col % 8 == 0 && v_col % 8 == 0);
  TORCH_CHECK(lse.scalar_type() == at::kFloat && delta.scalar_type() == at::kFloat && lse.size(1) == delta.size(1));
  c10::cuda::CUDAGuard guard(q_src.device());
  const int64_t T = q_src.size(0);
  auto dq = at::zeros({T, H * kHeadDim}, q_src.options().dtype(at::kFloat));
  auto dk = at::empty({T, KV * kHeadDim}, q_src.options());
  auto dv = at::empty({T, KV * kHeadDim}, q_src.options());
  if (T == 0 || numseqs == 0) return {dq, dk, dv};
  // Rows never covered by a key block (padding beyond the last sequence) stay zero.
  dk.zero_();
  dv.zero_();
  CUtensorMap mq = make_tmap_bf16_2d(q_src.data_ptr(), T, q_src.size(1), q_src.stride(0), 64, kQRows);
  CUtensorMap mk = make_tmap_bf16_2d(k_src.data_ptr(), T, k_src.size(1), k_src.stride(0), 64, kKeys);
  CUtensorMap mv = make_tmap_bf16_2d(v_src.data_ptr(), T, v_src.size(1), v_src.stride(0), 64, kKeys);
  CUtensorMap mdo = make_tmap_bf16_2d(d_o.data_ptr(), T, d_o.size(1), d_o.stride(0), 64, kQRows);
  CUtensorMap mdq = make_tmap_f32_2d(dq.data_ptr(), T, dq.size(1), dq.size(1), kHeadDim, kDqRows);
  BwdParams prm{};
  prm.dq = dq.data_ptr<float>();
  prm.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  prm.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  prm.lse = lse.data_ptr<float>();
  prm.delta = delta.data_ptr<float>();
  prm.lse_ld = lse.size(1);
  prm.cu_seqlens = cu_seqlens.data_ptr<int>();
  prm.prefix_lens = prefix_lens.data_ptr<int>();
  prm.tiles = reinterpret_cast<const int2*>(kv_tiles.data_ptr<int>());
  prm.ntiles = kv_ntiles.data_ptr<int>();
  prm.H = (int)H;
  prm.KV = (int)KV;
  prm.q_col = (int)q_col;
  prm.k_col = (int)k_col;
  prm.v_col = (int)v_col;
  prm.is_causal = is_causal ? 1 : 0;
  prm.scale_log2 = 1.4426950408889634f / sqrtf((float)kHeadDim);
  prm.scale = 1.f / sqrtf((float)kHeadDim);
  prm.status = fmha_status_ptr(q_src.device());
  static bool attr_set[16] = {false};
  if (!attr_set[q_src.device().index()]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(fmha_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    attr_set[q_src.device().index()] = true;
  }
  dim3 grid((unsigned)KV, (unsigned)kv_tiles.size(0));
  fmha_bwd_kernel<<<grid, kThreads, kSmemBytes, at::cuda::getCurrentCUDAStream()>>>(mq, mk, mv, mdo, mdq, prm);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dq, dk, dv};
}
