// Replicated-weight data parallelism over NVLink peer memory: one kernel per optimizer step
// reduce-scatters the ranks' bf16 gradients, applies AdamATan2 to this rank's fp32 master shard
// and all-gathers the new bf16 weights, all through direct loads/stores to the peers' buffers.
//
// Layout.  Every rank holds the full model twice in bf16 (weights and gradients), in one flat
// buffer each, allocated with cudaMalloc and exported with CUDA IPC so every peer can map it.
// Parameter p occupies [flat_p, flat_p + numel_p); rank r owns rows [r*c, min(R, (r+1)*c)) of p
// (c = ceil(R / world), the same split FSDP2 uses, so the fp32 shards checkpoint identically).
// The owned ranges of all parameters are the rank's "segments"; its fp32 master weights and
// moments are stored back to back in segment order.
//
// Kernel (persistent CTAs walking 8192-element chunks of the segments):
//   g   = sum_k grad_k[flat + i]   (peer loads, fixed rank order, fp32)
//   g  *= grad_scale               (global clipping coefficient or 1)
//   w   = w * (1 - lr*wd);  v = b2 v + (1-b2) g^2;  m += (1-b1)(g - m)
//   w  -= lr/bc1 * atan2(m, sqrt(v)/bc2_sqrt)     (or lr * atan2(g, .) without first moment)
//   ema += (1-d)(w - ema)
//   param_k[flat + i] = bf16(w) for every rank k  (peer stores)
// A reduce-only variant writes the fp32 reduced gradient shard and per-CTA sums of squares for
// global-norm clipping; the update variant can then read that shard instead of the peers.
//
// Segment kinds (one per parameter shard; the whole chunk takes one branch):
//   kAdamATan2   the update above.
//   kAdamEps     MuonAdamW's Adam for non-matrix parameters:
//                m = lerp(m, g, 1-b1);  v = lerp(v, g^2, 1-b2)
//                w = w (1 - lr wd) - lr * (m / bc1) / (sqrt(v / bc2) + 1e-8)
//   kMuonGather  Muon momentum on the fp32 shard, Nesterov input to the matrix's owner rank:
//                mom = lerp(mom, g, 1-beta);  u = lerp(g, mom, beta)
//                work_owner[dst + i] = u      (fp32 peer store; beta is carried in `bc1`)
//   kMuonApply   after the owner orthogonalised the gathered matrix in place:
//                O = work_owner[dst + i]      (fp32 peer load)
//                w = w (1 - lr wd) - lr O;  EMA;  bf16(w) to every rank
//
// The caller orders the step with the other ranks (a collective before: every rank's backward
// is complete; and after: every rank's stores have landed).  Nothing here waits on a peer.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kLeanThreads = 128;
constexpr int kVec = 8;                              // bf16 elements per 16-byte access
constexpr int kIters = 4;
constexpr int kChunk = kThreads * kVec * kIters;     // 8192 elements per CTA
constexpr int kMaxRanks = 8;

enum SegmentKind : int32_t { kAdamATan2 = 0, kAdamEps = 1, kMuonGather = 2, kMuonApply = 3 };
constexpr int32_t kLocalFlag = 256;  // OR-ed into `kind`: a rank-local (expert-parallel) parameter

struct Segment {
  int64_t flat;         // element offset in the flat bf16 weight/grad buffers
  int64_t shard;        // element offset in the fp32 shard buffers
  int64_t n;            // elements
  int64_t block_start;  // first chunk index
  float lr, wd, bc1, bc2_sqrt;  // kAdamEps: bc2_sqrt holds bc2 itself; kMuonGather: bc1 holds beta
  int32_t vec;          // flat % 8 == 0, shard % 8 == 0, n % 8 == 0 (and dst % 8 == 0 for Muon)
  int32_t kind;         // SegmentKind
  int64_t dst;          // Muon: element offset of this shard in the owner's fp32 workspace
  int32_t dst_rank;     // Muon: owner rank of the matrix
  int32_t has_m;        // kAdamEps: the parameter keeps a first moment (beta1 > 0)
};

struct Peers {
  uint64_t grad[kMaxRanks];
  uint64_t weight[kMaxRanks];
  uint64_t work[kMaxRanks];  // fp32 Muon workspaces (0 when unused)
};

struct StepArgs {
  const Segment* segs;
  int nsegs;
  int world;
  int rank;
  float* master;
  float* exp_avg;        // nullptr without a first moment
  float* exp_avg_sq;
  float* ema;            // nullptr without EMA
  const float* reduced;  // update variant: read gradients from here instead of the peers
  float* reduced_out;    // reduce variant: write the reduced gradient shard here
  float* sumsq_out;      // reduce variant: one partial sum of squares per chunk
  const float* grad_scale;  // device scalar (clip coefficient) or nullptr for 1
  float b1, b2, ema_decay;
};

__device__ __forceinline__ int find_segment(const Segment* segs, int n, int64_t b) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (segs[mid].block_start <= b) lo = mid;
    else hi = mid - 1;
  }
  return lo;
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

__device__ __forceinline__ void ld8(const float* p, float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
}

__device__ __forceinline__ void st8(float* p, const float (&f)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(f[4], f[5], f[6], f[7]);
}

__device__ __forceinline__ float reduce1(const Peers& peers, int r0, int world, int64_t flat) {
  float g = 0.f;
  for (int k = 0; k < world; ++k)
    g += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(peers.grad[r0 + k])[flat]);
  return g;
}

// torch.lerp's two-sided form (the same rounding as the per-parameter optimizers' lerp_).
__device__ __forceinline__ float lerpf(float a, float b, float t) {
  return fabsf(t) < 0.5f ? a + t * (b - a) : b - (b - a) * (1.f - t);
}

__device__ __forceinline__ float adam1(float g, float& w, float* m, float& v, float* e, const Segment& s,
                                       const StepArgs& a) {
  if ((s.kind & ~kLocalFlag) == kAdamEps) {
    w = w * (1.f - s.lr * s.wd);
    v = lerpf(v, g * g, 1.f - a.b2);
    float num = g;
    if (m != nullptr && s.has_m) {
      *m = lerpf(*m, g, 1.f - a.b1);
      num = *m / s.bc1;
    }
    w = w - s.lr * (num / (sqrtf(v / s.bc2_sqrt) + 1e-8f));
  } else {
    if (s.wd != 0.f) w = w * (1.f - s.lr * s.wd);
    v = a.b2 * v + (1.f - a.b2) * g * g;
    const float denom = sqrtf(v) / s.bc2_sqrt;
    if (m != nullptr) {
      *m = *m + (1.f - a.b1) * (g - *m);
      w = w - (s.lr / s.bc1) * atan2f(*m, denom);
    } else {
      w = w - s.lr * atan2f(g, denom);
    }
  }
  if (e != nullptr) *e = *e + (1.f - a.ema_decay) * (w - *e);
  return w;
}

// Muon: momentum on the fp32 shard (kept in the first-moment buffer) and the Nesterov input.
__device__ __forceinline__ float muon_gather1(float g, float* mom, float beta) {
  *mom = lerpf(*mom, g, 1.f - beta);
  return lerpf(g, *mom, beta);
}

// Muon: decoupled decay and the orthogonalised update, then the EMA.
__device__ __forceinline__ float muon_apply1(float o, float w, float* e, const Segment& s, const StepArgs& a) {
  w = w * (1.f - s.lr * s.wd);
  w = w - s.lr * o;
  if (e != nullptr) *e = *e + (1.f - a.ema_decay) * (w - *e);
  return w;
}

__device__ __forceinline__ float* work_ptr(const Peers& peers, const Segment& s) {
  return reinterpret_cast<float*>(peers.work[s.dst_rank]) + s.dst;
}

// Load the 8-element gradient group at flat offset `flat` of every rank (raw bf16 words).
__device__ __forceinline__ void load_grads(const Peers& peers, int r0, int world, int64_t flat,
                                           uint4 (&raw)[kMaxRanks]) {
#pragma unroll
  for (int k = 0; k < kMaxRanks; ++k)
    if (k < world)
      raw[k] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(peers.grad[r0 + k]) + flat);
}

__device__ __forceinline__ void sum_grads(const uint4 (&raw)[kMaxRanks], int world, float (&g)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) g[e] = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxRanks; ++k) {
    if (k < world) {
      float f[8];
      unpack8(raw[k], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) g[e] += f[e];
    }
  }
}

__device__ __forceinline__ void update8(const float (&gin)[8], float scale, int64_t sh, const Segment& s,
                                        const StepArgs& a, float (&w)[8]) {
  float v[8], m[8], e[8];
  ld8(a.master + sh, w);
  ld8(a.exp_avg_sq + sh, v);
  if (a.exp_avg != nullptr) ld8(a.exp_avg + sh, m);
  if (a.ema != nullptr) ld8(a.ema + sh, e);
#pragma unroll
  for (int k = 0; k < 8; ++k)
    adam1(gin[k] * scale, w[k], a.exp_avg != nullptr ? &m[k] : nullptr, v[k], a.ema != nullptr ? &e[k] : nullptr, s, a);
  st8(a.master + sh, w);
  st8(a.exp_avg_sq + sh, v);
  if (a.exp_avg != nullptr) st8(a.exp_avg + sh, m);
  if (a.ema != nullptr) st8(a.ema + sh, e);
}

// Persistent: CTA b handles chunks b, b + gridDim.x, ...  Within a chunk each thread walks its
// 8-element groups with the next group's gradient loads (peer loads over NVLink) issued before
// the current group is updated, so NVLink latency overlaps the HBM traffic of the update.
//
// Lean variant (kT = kLeanThreads): for an update that runs beside the backward's kernels.  128
// threads and at most 80 registers each, so a CTA fits in what a dense-GEMM CTA leaves of every
// SM sub-partition's register file; no gradient prefetch; launched with one CTA per chunk, so no
// CTA holds an SM longer than one chunk (a waiting attention or fused-SwiGLU CTA, which leaves no
// room beside it, is not delayed by more than that).
template <bool kFromPeers, int kT>
__global__ void __launch_bounds__(kT, kT == kThreads ? 2 : 6) dp_update_kernel(const __grid_constant__ Peers peers,
                                                                                 const StepArgs a, int64_t nchunks) {
  constexpr bool kPrefetch = kT == kThreads;
  const float scale = a.grad_scale != nullptr ? *a.grad_scale : 1.f;
  for (int64_t chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x) {
    const Segment s = a.segs[find_segment(a.segs, a.nsegs, chunk)];
    const int64_t start = (chunk - s.block_start) * kChunk;
    const int64_t end = min(start + int64_t(kChunk), s.n);
    // A rank-local segment (expert-parallel parameter) is reduced over and written to this rank only.
    const bool local = (s.kind & kLocalFlag) != 0;
    const int r0 = local ? a.rank : 0, nr = local ? 1 : a.world;
    const int kind = s.kind & ~kLocalFlag;
    const bool needs_grad = kind != kMuonApply;
    if (s.vec) {
      int64_t i = start + int64_t(threadIdx.x) * kVec;
      uint4 raw[kPrefetch ? kMaxRanks : 1];
      if constexpr (kPrefetch)
        if (kFromPeers && needs_grad && i < end) load_grads(peers, r0, nr, s.flat + i, raw);
      for (; i < end; i += int64_t(kT) * kVec) {
        float g[8];
        if (!needs_grad) {
        } else if constexpr (kFromPeers && kPrefetch) {
          sum_grads(raw, nr, g);
          const int64_t nxt = i + int64_t(kT) * kVec;
          if (nxt < end) load_grads(peers, r0, nr, s.flat + nxt, raw);
        } else if constexpr (kFromPeers) {
#pragma unroll
          for (int e = 0; e < 8; ++e) g[e] = 0.f;
          for (int k = 0; k < nr; ++k) {
            float f[8];
            unpack8(*reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(peers.grad[r0 + k]) +
                                                    s.flat + i),
                    f);
#pragma unroll
            for (int e = 0; e < 8; ++e) g[e] += f[e];
          }
        } else {
          ld8(a.reduced + s.shard + i, g);
        }
        float w[8];
        if (kind == kMuonGather) {
          float m[8];
          ld8(a.exp_avg + s.shard + i, m);
#pragma unroll
          for (int k = 0; k < 8; ++k) g[k] = muon_gather1(g[k] * scale, &m[k], s.bc1);
          st8(a.exp_avg + s.shard + i, m);
          st8(work_ptr(peers, s) + i, g);
          continue;
        }
        if (kind == kMuonApply) {
          float o[8], e[8];
          ld8(work_ptr(peers, s) + i, o);
          ld8(a.master + s.shard + i, w);
          if (a.ema != nullptr) ld8(a.ema + s.shard + i, e);
#pragma unroll
          for (int k = 0; k < 8; ++k) w[k] = muon_apply1(o[k], w[k], a.ema != nullptr ? &e[k] : nullptr, s, a);
          st8(a.master + s.shard + i, w);
          if (a.ema != nullptr) st8(a.ema + s.shard + i, e);
        } else {
          update8(g, scale, s.shard + i, s, a, w);
        }
        const uint4 packed = pack8(w);
#pragma unroll
        for (int k = 0; k < kMaxRanks; ++k)
          if (k < nr)
            *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peers.weight[r0 + k]) + s.flat + i) = packed;
      }
    } else {
      for (int64_t i = start + threadIdx.x; i < end; i += kT) {
        const int64_t sh = s.shard + i;
        float* e = a.ema != nullptr ? a.ema + sh : nullptr;
        float w = a.master[sh];
        if (kind == kMuonApply) {
          w = muon_apply1(work_ptr(peers, s)[i], w, e, s, a);
        } else {
          const float g = (kFromPeers ? reduce1(peers, r0, nr, s.flat + i) : a.reduced[sh]) * scale;
          if (kind == kMuonGather) {
            work_ptr(peers, s)[i] = muon_gather1(g, a.exp_avg + sh, s.bc1);
            continue;
          }
          float v = a.exp_avg_sq[sh];
          w = adam1(g, w, a.exp_avg != nullptr ? a.exp_avg + sh : nullptr, v, e, s, a);
          a.exp_avg_sq[sh] = v;
        }
        a.master[sh] = w;
        const __nv_bfloat16 b = __float2bfloat16(w);
        for (int k = 0; k < nr; ++k) reinterpret_cast<__nv_bfloat16*>(peers.weight[r0 + k])[s.flat + i] = b;
      }
    }
  }
  __threadfence_system();  // once per thread: its peer stores are visible before the closing collective
}

__global__ void __launch_bounds__(kThreads, 2) dp_reduce_kernel(const __grid_constant__ Peers peers,
                                                                   const StepArgs a, int64_t nchunks) {
  // One partial sum of squares per chunk (written by the CTA that owns the chunk), so the host
  // sums a fixed set of partials in a fixed order whatever the grid size.
  __shared__ float part[kThreads / 32];
  for (int64_t chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x) {
    const Segment s = a.segs[find_segment(a.segs, a.nsegs, chunk)];
    const int64_t start = (chunk - s.block_start) * kChunk;
    const int64_t end = min(start + int64_t(kChunk), s.n);
    const bool local = (s.kind & kLocalFlag) != 0;
    const int r0 = local ? a.rank : 0, nr = local ? 1 : a.world;
    float sq = 0.f;
    if (s.vec) {
      for (int64_t i = start + int64_t(threadIdx.x) * kVec; i < end; i += int64_t(kThreads) * kVec) {
        uint4 raw[kMaxRanks];
        float g[8];
        load_grads(peers, r0, nr, s.flat + i, raw);
        sum_grads(raw, nr, g);
        st8(a.reduced_out + s.shard + i, g);
#pragma unroll
        for (int k = 0; k < 8; ++k) sq += g[k] * g[k];
      }
    } else {
      for (int64_t i = start + threadIdx.x; i < end; i += kThreads) {
        const float g = reduce1(peers, r0, nr, s.flat + i);
        a.reduced_out[s.shard + i] = g;
        sq += g * g;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < kThreads / 32 ? part[threadIdx.x] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (threadIdx.x == 0) a.sumsq_out[chunk] = t;
    }
    __syncthreads();
  }
}

// Two resident CTAs per SM (the launch bounds), capped by the number of chunks.
unsigned persistent_grid(int64_t nchunks, int device) {
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  return static_cast<unsigned>(std::min<int64_t>(nchunks, int64_t(sms) * 2));
}

Peers make_peers(const std::vector<int64_t>& grads, const std::vector<int64_t>& weights,
                 const std::vector<int64_t>& work = {}) {
  TORCH_CHECK(grads.size() == weights.size() && grads.size() >= 1 && grads.size() <= kMaxRanks,
              "dp step supports 1..", kMaxRanks, " ranks");
  TORCH_CHECK(work.empty() || work.size() == grads.size(), "one Muon workspace per rank");
  Peers p{};
  for (size_t k = 0; k < grads.size(); ++k) {
    TORCH_CHECK(grads[k] % 16 == 0 && weights[k] % 16 == 0, "peer buffers must be 16-byte aligned");
    p.grad[k] = static_cast<uint64_t>(grads[k]);
    p.weight[k] = static_cast<uint64_t>(weights[k]);
    if (!work.empty()) {
      TORCH_CHECK(work[k] % 32 == 0, "Muon workspaces must be 32-byte aligned");
      p.work[k] = static_cast<uint64_t>(work[k]);
    }
  }
  return p;
}

StepArgs make_args(at::Tensor segs, int64_t world, at::Tensor master, c10::optional<at::Tensor> exp_avg,
                   at::Tensor exp_avg_sq, c10::optional<at::Tensor> ema, c10::optional<at::Tensor> grad_scale,
                   double b1, double b2, double ema_decay) {
  TORCH_CHECK(segs.is_cuda() && segs.dtype() == at::kByte && segs.numel() % sizeof(Segment) == 0, "bad segment table");
  for (const at::Tensor* t : {&master, &exp_avg_sq})
    TORCH_CHECK(t->is_cuda() && t->dtype() == at::kFloat && t->is_contiguous(), "fp32 contiguous shard buffers");
  StepArgs a{};
  a.segs = reinterpret_cast<const Segment*>(segs.data_ptr());
  a.nsegs = static_cast<int>(segs.numel() / sizeof(Segment));
  a.world = static_cast<int>(world);
  a.master = master.data_ptr<float>();
  a.exp_avg = exp_avg ? exp_avg->data_ptr<float>() : nullptr;
  a.exp_avg_sq = exp_avg_sq.data_ptr<float>();
  a.ema = ema ? ema->data_ptr<float>() : nullptr;
  a.grad_scale = grad_scale ? grad_scale->data_ptr<float>() : nullptr;
  a.b1 = static_cast<float>(b1);
  a.b2 = static_cast<float>(b2);
  a.ema_decay = static_cast<float>(ema_decay);
  return a;
}

}  // namespace

// Segment table entry size (bytes), for the host-side packer.
int64_t dp_segment_bytes() { return sizeof(Segment); }

int64_t dp_chunk_elements() { return kChunk; }

void dp_step(std::vector<int64_t> peer_grads, std::vector<int64_t> peer_weights, at::Tensor segs, int64_t nblocks,
             at::Tensor master, c10::optional<at::Tensor> exp_avg, at::Tensor exp_avg_sq, c10::optional<at::Tensor> ema,
             c10::optional<at::Tensor> reduced, c10::optional<at::Tensor> grad_scale, double b1, double b2,
             double ema_decay, std::vector<int64_t> peer_work, int64_t rank, bool lean) {
  const c10::cuda::CUDAGuard guard(master.device());
  const Peers peers = make_peers(peer_grads, peer_weights, peer_work);
  StepArgs a = make_args(segs, peer_grads.size(), master, exp_avg, exp_avg_sq, ema, grad_scale, b1, b2, ema_decay);
  TORCH_CHECK(rank >= 0 && rank < a.world, "bad rank");
  a.rank = static_cast<int>(rank);
  if (nblocks == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (reduced) a.reduced = reduced->data_ptr<float>();
  if (lean) {  // one short CTA per chunk, beside the backward's kernels
    TORCH_CHECK(!reduced && nblocks < (int64_t(1) << 31), "the lean update reads the peers' gradients");
    dp_update_kernel<true, kLeanThreads><<<static_cast<unsigned>(nblocks), kLeanThreads, 0, stream>>>(peers, a, nblocks);
  } else {
    const unsigned grid = persistent_grid(nblocks, master.device().index());
    if (reduced) dp_update_kernel<false, kThreads><<<grid, kThreads, 0, stream>>>(peers, a, nblocks);
    else dp_update_kernel<true, kThreads><<<grid, kThreads, 0, stream>>>(peers, a, nblocks);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_reduce(std::vector<int64_t> peer_grads, at::Tensor segs, int64_t nblocks, at::Tensor reduced_out,
               at::Tensor sumsq_out, int64_t rank) {
  const c10::cuda::CUDAGuard guard(reduced_out.device());
  const Peers peers = make_peers(peer_grads, peer_grads);
  TORCH_CHECK(reduced_out.dtype() == at::kFloat && sumsq_out.dtype() == at::kFloat && sumsq_out.numel() >= nblocks,
              "dp_reduce outputs");
  StepArgs a{};
  a.segs = reinterpret_cast<const Segment*>(segs.data_ptr());
  a.nsegs = static_cast<int>(segs.numel() / sizeof(Segment));
  a.world = static_cast<int>(peer_grads.size());
  TORCH_CHECK(rank >= 0 && rank < a.world, "bad rank");
  a.rank = static_cast<int>(rank);
  a.reduced_out = reduced_out.data_ptr<float>();
  a.sumsq_out = sumsq_out.data_ptr<float>();
  if (nblocks == 0) return;
  dp_reduce_kernel<<<persistent_grid(nblocks, reduced_out.device().index()), kThreads, 0,
                     at::cuda::getCurrentCUDAStream()>>>(peers, a, nblocks);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ CUDA IPC buffers
// A device buffer from cudaMalloc (IPC handles need allocation-granular memory, which the
// caching allocator does not guarantee), returned as a uint8 tensor that frees it on release.
std::vector<at::Tensor> ipc_alloc(int64_t nbytes, int64_t device) {
  TORCH_CHECK(nbytes > 0, "ipc_alloc: empty buffer");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, static_cast<size_t>(nbytes)));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, static_cast<size_t>(nbytes)));
  cudaIpcMemHandle_t handle;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&handle, ptr));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device);
  at::Tensor buf = torch::from_blob(ptr, {nbytes}, [device](void* p) {
    c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
    cudaFree(p);
  }, opts);
  at::Tensor h = at::empty({static_cast<int64_t>(sizeof(handle))}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(h.data_ptr(), &handle, sizeof(handle));
  return {buf, h};
}

int64_t ipc_open(at::Tensor handle_bytes, int64_t device) {
  TORCH_CHECK(handle_bytes.numel() == sizeof(cudaIpcMemHandle_t) && !handle_bytes.is_cuda(), "bad IPC handle");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t handle;
  std::memcpy(&handle, handle_bytes.contiguous().data_ptr(), sizeof(handle));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, handle, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

void ipc_close(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

// Zeroes a contiguous device tensor with one driver memset on the current stream (the gradient
// buffer between steps: a plain store stream at the copy engine's rate, one call for any size).
void zero_bytes(at::Tensor t) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "zero_bytes: contiguous CUDA tensor");
  if (t.numel() == 0) return;
  const c10::cuda::CUDAGuard guard(t.device());
  C10_CUDA_CHECK(cudaMemsetAsync(t.data_ptr(), 0, t.nbytes(), at::cuda::getCurrentCUDAStream()));
}

bool peer_access_possible(int64_t device, int64_t peer) {
  int ok = 0;
  C10_CUDA_CHECK(cudaDeviceCanAccessPeer(&ok, static_cast<int>(device), static_cast<int>(peer)));
  return ok != 0;
}
