// Allocation-free entry point of the prefix-LM attention forward.
//
// This entry point has no counterpart in the reference implementation.  It is for callers
// that are not allowed to allocate device memory at the point where they run attention:
//   * inference runtimes and plugin interfaces that own every byte of device memory
//     themselves and call kernels through an "enqueue" hook that has no workspace argument;
//   * code running under a memory manager that forbids allocation after start-up (a fixed
//     budget carved out at load time), where cudaMalloc would fail or break the budget;
//   * latency-critical loops where an allocator call, and the device synchronisation that
//     cudaMalloc/cudaFree can imply, is not acceptable.
// The regular entry (`mimir_b200._C.fmha_fwd`) needs a scratch tile schedule that its caller
// allocates through PyTorch.  This variant keeps that scratch in a fixed, file-scope device
// array instead, so it calls no cudaMalloc, cudaFree or allocating library routine.  The
// caller still passes every input and output buffer.
//
// Limits and sharing rules:
//   * at most MIMIR_FMHA_NOALLOC_MAX_TILES query tiles per call, where the tile count is
//     ceil(total_tokens / 128) + numseqs; larger calls are rejected with
//     MIMIR_NOALLOC_ERR_TOO_LARGE before anything is launched;
//   * the scratch array is shared by every call in the process on a given device and keeps
//     the previous call's contents; each call rewrites the tile schedule it reads, but two
//     calls that overlap on the GPU (different streams, no ordering between them) race on it;
//   * the first call on each device (of either function below) looks up the scratch address
//     with cudaGetSymbolAddress and sets the kernel's shared-memory limit, with that device
//     current; make that first call before any stream capture;
//   * every GPU that loads the library holds the scratch array (128 KiB plus a status word)
//     until the process exits.
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
//   q, k, v, out: 16-byte aligned, row strides a multiple of 8 elements
//   out: [total_tokens, H*128] bf16; lse: [H, lse_ld] fp32 with lse_ld >= total_tokens
//   cu_seqlens: numseqs + 1 int32 offsets on the device; prefix_lens: numseqs int32 (device)
//   is_causal != 0 ignores the prompt lengths (plain causal attention).
// Returns MIMIR_NOALLOC_OK or a negative error code; launches are asynchronous on `stream`.
int mimir_fmha_fwd_noalloc(const void* q, int64_t q_ld, const void* k, int64_t k_ld, const void* v, int64_t v_ld,
                           void* out, float* lse, int64_t lse_ld, const int* cu_seqlens, const int* prefix_lens,
                           int numseqs, int64_t total_tokens, int num_heads, int num_kv_heads, int is_causal,
                           cudaStream_t stream);

// Reads the kernel status of the current device into *status_out and clears it.  0 means every
// call since the previous read finished normally; a positive code means a bounded wait inside
// the kernel gave up (a protocol error), and the output rows of that call are not valid.  The
// status is sticky: it holds the first failure until it is read.  Synchronises `stream`.
int mimir_fmha_noalloc_status(cudaStream_t stream, int* status_out);

#ifdef __cplusplus
}
#endif
