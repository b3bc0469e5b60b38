// Allocation-free C entry point of the paged structured-mask attention.
//
// This entry point has no counterpart in the reference (D3D has no native
// code at all); it exists for callers of this library that must not allocate
// GPU memory while they run:
//   * code that is being recorded into a CUDA graph, where an allocation would
//     either be refused or silently synchronize the device;
//   * plugins of other inference runtimes whose per-call hook is required to
//     run with the memory the host framework already owns;
//   * serving loops that reserved the whole device for their own pool up
//     front, so a cudaMalloc would fail or fragment that pool mid-request.
// Such callers still pass every input and output buffer; the only memory the
// kernel needs beyond them (the per-chunk partial results of the split-KV
// softmax) comes from a fixed array compiled into the library.
//
// Contract:
//   * Scratch capacity is D3D_ATTN_NOALLOC_SCRATCH_BYTES (16 MiB) per GPU,
//     reserved on every GPU that loads the library for as long as the process
//     lives.  It holds n_chunks * B*q_len * Hq * (head_dim + 2) floats when
//     n_chunks > 1 (none when n_chunks == 1); larger requests are rejected
//     with D3D_NOALLOC_ERR_TOO_LARGE before anything is launched.
//   * The first call on each device looks up the device address of that array
//     (cudaGetSymbolAddress) with the device current, and sets the kernels'
//     shared-memory limit.  Make that first call outside any stream capture;
//     later calls only enqueue kernels.
//   * All calls share the one array, and it keeps what the last call left in
//     it.  Nothing in it has to start at zero: every partial a call reads was
//     written earlier in the same call.  Calls whose kernels overlap on the
//     GPU (different streams, or different host threads on one device) race
//     on the array and must be serialized by the caller.
//   * No cudaMalloc, cudaFree or other allocating routine is called.
//
// Arguments mirror the allocating binding: q [B*q_len, Hq, D] bf16,
// k_cache / v_cache [num_slots, Hkv, D] bf16, block_table [B, bt_stride]
// int32, rows [B*q_len, 3] int32 (lim, lo, hi), kv_end [B] int32, out like q.
// Shape rules (violations return D3D_NOALLOC_ERR_BAD_ARG, nothing launched):
//   * page_size divides 64 (a 64-key tile spans whole pages); chunk is a
//     multiple of 64 and of page_size;
//   * 1 <= n_chunks <= D3D_ATTN_NOALLOC_MAX_CHUNKS.
// The caller's duty, not checked: n_chunks * chunk >= kv_end[b] for every
// sequence b.  Chunk c covers keys [c*chunk, (c+1)*chunk); keys at or beyond
// n_chunks * chunk are not attended to.
// Returns 0 on success, a D3D_NOALLOC_ERR_* code, or the cudaError_t of this
// call's own kernel launches (errors of earlier, unrelated work are not
// reported here).
#pragma once
#include <cuda_runtime.h>

#define D3D_ATTN_NOALLOC_SCRATCH_BYTES (16u << 20)
#define D3D_ATTN_NOALLOC_MAX_CHUNKS 512

#define D3D_NOALLOC_ERR_TOO_LARGE 1001
#define D3D_NOALLOC_ERR_BAD_ARG 1002
#define D3D_NOALLOC_ERR_SYMBOL 1003

#ifdef __cplusplus
extern "C" {
#endif

__attribute__((visibility("default"))) int d3d_attention_noalloc(
    const void* q, const void* k_cache, const void* v_cache, long long num_slots, const int* block_table,
    int bt_stride, const int* rows, const int* kv_end, int B, int q_len, int Hq, int Hkv, int head_dim,
    int page_size, float scale, int chunk, int n_chunks, void* out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
