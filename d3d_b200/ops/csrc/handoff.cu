// Cross-GPU handoff over NVLink peer memory (sm_100a).  It replaces the
// reference's host Pipe between the drafter and the verifier process
// (single/eval_async_packed.py:216-346, serving/target_process.py:9-139).
//
// A mailbox is a device allocation [flag (int64, own 128-byte line) |
// payload] owned by the receiving GPU and mapped into the sender's process
// through CUDA IPC (no multicast object is ever created).  The sender's
// kernel stores the payload with plain st.global through the peer pointer,
// then publishes a monotonically increasing sequence number with a
// system-scope release store; the receiver's kernel spins with system-scope
// acquire loads until the sequence number arrives.  Every spin is bounded by
// a globaltimer limit and reports ERR_TIMEOUT_FLAG in a status word instead
// of hanging.
//
// accept_send fuses the end of target verification with the
// handoff: greedy acceptance (commit length, correction token) plus the
// hidden state that produced the correction and the posterior row are
// written straight into the drafter GPU's mailbox, followed by the flag.
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace d3d {

__device__ __forceinline__ void st_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int64_t ld_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Copy nbytes (multiple of 16) from local src to (peer) dst, then publish
// seq.  Each block fences its own stores at system scope and takes a ticket;
// the last block to finish (no block ever waits for another) resets the
// ticket counter and publishes the flag with a release store.
__global__ void handoff_put_kernel(const uint4* __restrict__ src, uint4* dst, size_t n16, int64_t* flag,
                                   int64_t seq, unsigned int* ticket) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  if (gridDim.x > 1) {
    const unsigned int t = atomicAdd(ticket, 1u);
    if (t != gridDim.x - 1) return;
    *ticket = 0;
    __threadfence_system();
  }
  st_release_sys(flag, seq);
}

void handoff_put(const void* src, void* dst_peer, size_t nbytes, int64_t* flag_peer, int64_t seq,
                 unsigned int* ticket, cudaStream_t st) {
  if (nbytes % 16) throw std::runtime_error("handoff payload must be a multiple of 16 bytes");
  const size_t n16 = nbytes / 16;
  int blocks = static_cast<int>((n16 + 1023) / 1024);
  blocks = blocks < 1 ? 1 : (blocks > 132 ? 132 : blocks);
  if (blocks > 1 && ticket == nullptr) blocks = 1;
  handoff_put_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst_peer), n16,
                                             flag_peer, seq, ticket);
}

// Wait until *flag >= seq (bounded), then copy the payload to dst and write
// the outcome to *status (0 = arrived, ERR_TIMEOUT_FLAG = gave up).  dst and
// status may be pinned host memory (written through the unified address
// space), so the host reads the message right after a stream synchronize;
// status is a plain store by one thread, never a device atomic.
__global__ void handoff_wait_kernel(const int64_t* flag, int64_t seq, const uint4* src, uint4* __restrict__ dst,
                                    size_t n16, int* status, unsigned long long limit_ns) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(flag) < seq) {
      if (globaltimer_ns() - t0 > limit_ns) {
        ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (ok && dst != nullptr) {
    // __ldcv: fetch from memory, not from a line this SM may have cached earlier
    for (size_t i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = __ldcv(src + i);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && status) *reinterpret_cast<volatile int*>(status) = ok ? 0 : ERR_TIMEOUT_FLAG;
}

void handoff_wait(const int64_t* flag, int64_t seq, const void* src, void* dst, size_t nbytes, int* status,
                  unsigned long long limit_ns, cudaStream_t st) {
  handoff_wait_kernel<<<1, 256, 0, st>>>(flag, seq, static_cast<const uint4*>(src), static_cast<uint4*>(dst),
                                         nbytes / 16, status, limit_ns);
}

// Greedy acceptance fused with the handoff.  Writes one reply message into
// the peer's mailbox slot:
//   out_i64[0..3]              header (2 = verify, B, K, H)
//   out_i64[8 + b*(2+K) + 0]   commit length of sequence b
//   out_i64[8 + b*(2+K) + 1]   correction token
//   out_i64[8 + b*(2+K) + 2..] posterior (target argmax at each block row)
//   hid_out[b*H ..]            bf16 hidden state that produced the correction
// and then publishes seq.  One block; the commit scan is K steps per row.
__global__ void accept_send_kernel(const int64_t* __restrict__ blocks, const int64_t* __restrict__ post, int B, int K,
                                   const __nv_bfloat16* __restrict__ hidden, int H, int64_t* out_i64,
                                   __nv_bfloat16* hid_out, int64_t* flag, int64_t seq) {
  __shared__ int s_commit;
  if (threadIdx.x == 0) {
    out_i64[0] = 2;
    out_i64[1] = B;
    out_i64[2] = K;
    out_i64[3] = H;
  }
  int64_t* res = out_i64 + 8;
  for (int b = 0; b < B; ++b) {
    if (threadIdx.x == 0) {
      int n = 1;
      while (n < K && blocks[static_cast<size_t>(b) * K + n] == post[static_cast<size_t>(b) * K + n - 1]) ++n;
      s_commit = n;
      int64_t* o = res + static_cast<size_t>(b) * (2 + K);
      o[0] = n;
      o[1] = post[static_cast<size_t>(b) * K + n - 1];
    }
    __syncthreads();
    for (int j = threadIdx.x; j < K; j += blockDim.x)
      res[static_cast<size_t>(b) * (2 + K) + 2 + j] = post[static_cast<size_t>(b) * K + j];
    if (hidden && hid_out) {
      const size_t src = (static_cast<size_t>(b) * K + s_commit - 1) * H;
      for (int i = threadIdx.x; i < H; i += blockDim.x) hid_out[static_cast<size_t>(b) * H + i] = hidden[src + i];
    }
    __syncthreads();
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) st_release_sys(flag, seq);
}

void accept_send(const int64_t* blocks, const int64_t* post, int B, int K, const __nv_bfloat16* hidden, int H,
                 int64_t* out_peer, __nv_bfloat16* hid_peer, int64_t* flag_peer, int64_t seq, cudaStream_t st) {
  accept_send_kernel<<<1, 256, 0, st>>>(blocks, post, B, K, hidden, H, out_peer, hid_peer, flag_peer, seq);
}

// ---------------------------------------------------------------- CUDA IPC
void* mailbox_alloc(size_t nbytes) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, nbytes);
  if (e != cudaSuccess) throw std::runtime_error(std::string("mailbox cudaMalloc: ") + cudaGetErrorString(e));
  e = cudaMemset(p, 0, nbytes);
  if (e != cudaSuccess) throw std::runtime_error(std::string("mailbox memset: ") + cudaGetErrorString(e));
  return p;
}

void mailbox_free(void* p) { cudaFree(p); }

void ipc_get_handle(void* p, unsigned char* out64) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  memcpy(out64, &h, sizeof(h));
}

void* ipc_open_handle(const unsigned char* in64) {
  cudaIpcMemHandle_t h;
  memcpy(&h, in64, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  return p;
}

void ipc_close_handle(void* p) { cudaIpcCloseMemHandle(p); }

}  // namespace d3d
