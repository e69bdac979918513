// Allocation-free entry point of the prefix-LM attention forward.
//
// This entry point has no counterpart in the reference implementation; it exists for callers
// that must not allocate device memory while they run attention:
//   * engines that capture their whole decode/prefill step into a CUDA graph and forbid
//     cudaMalloc inside the capture (an allocation during capture fails or invalidates it);
//   * inference runtimes and plugin interfaces that own all device memory and call kernels
//     through an "enqueue" hook with no workspace argument;
//   * latency-critical loops where an allocator call (and its possible device synchronisation)
//     is not acceptable.
// The usual entry (`mimir_b200._C.fmha_fwd`) needs a scratch tile schedule that its caller
// allocates through PyTorch.  This variant keeps that scratch in a fixed, file-scope device
// array instead, so it calls no cudaMalloc, cudaFree or allocating library routine.
//
// Limits and sharing rules:
//   * at most MIMIR_FMHA_NOALLOC_MAX_TILES query tiles per call, where the tile count is
//     ceil(total_tokens / 128) + numseqs; larger calls are rejected with
//     MIMIR_NOALLOC_ERR_TOO_LARGE before anything is launched;
//   * the scratch array is shared by every call in the process on a given device and keeps
//     the previous call's contents; the entry point rewrites everything it reads, but two
//     calls that overlap on the GPU (different streams, no ordering between them) race on it;
//   * the first call on each device looks up the scratch address (cudaGetSymbolAddress) and
//     sets the kernel's shared-memory limit; make that first call before any stream capture.
//   * every GPU that loads the library holds the scratch array until the process exits.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define MIMIR_FMHA_NOALLOC_MAX_TILES 16384   /* 16384 x 8 bytes = 128 KiB of scratch per device */

#define MIMIR_NOALLOC_OK 0
#define MIMIR_NOALLOC_ERR_ARGS (-1)
#define MIMIR_NOALLOC_ERR_TOO_LARGE (-2)
#define MIMIR_NOALLOC_ERR_CUDA (-3)

#ifdef __cplusplus
extern "C" {
#endif

// out = attention(q, k, v) per head (head_dim 128, bf16), lse = per-row log2-sum-exp (fp32).
//   q: [total_tokens, q_ld] bf16 row-major, head h at columns [128h, 128h+128)
//   k, v: [total_tokens, k_ld / v_ld] bf16, KV heads; H must be a multiple of KV
//   out: [total_tokens, H*128] bf16; lse: [H, lse_ld] fp32 with lse_ld >= total_tokens
//   cu_seqlens: numseqs + 1 int32 offsets on the device; prefix_lens: numseqs int32 (device)
//   is_causal != 0 ignores the prompt lengths (plain causal attention).
// Returns MIMIR_NOALLOC_OK or a negative error code; launches are asynchronous on `stream`.
int mimir_fmha_fwd_noalloc(const void* q, int64_t q_ld, const void* k, int64_t k_ld, const void* v, int64_t v_ld,
                           void* out, float* lse, int64_t lse_ld, const int* cu_seqlens, const int* prefix_lens,
                           int numseqs, int64_t total_tokens, int num_heads, int num_kv_heads, int is_causal,
                           cudaStream_t stream);

#ifdef __cplusplus
}
#endif
