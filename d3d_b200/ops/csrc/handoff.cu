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
                                   __nv_bfloat16* hid_out, int64_t* flag, int64_t seq, const int* gate) {
  __shared__ int s_commit;
  // an armed verify whose request did not match ran on placeholder inputs:
  // nothing is sent (the host answers the message that did arrive)
  if (gate != nullptr && *reinterpret_cast<const volatile int*>(gate) == 0) return;
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
                 int64_t* out_peer, __nv_bfloat16* hid_peer, int64_t* flag_peer, int64_t seq, const int* gate,
                 cudaStream_t st) {
  accept_send_kernel<<<1, 256, 0, st>>>(blocks, post, B, K, hidden, H, out_peer, hid_peer, flag_peer, seq, gate);
}

// ------------------------------------------------------- armed verify (target)
// The target enqueues the next verify before its request exists: this kernel
// (first on the stream, ahead of the verify graph) waits -- bounded -- for
// message ``seq`` of every source inbox, copies each message's first
// ``head_words`` into pinned host memory for the host's bookkeeping, and, when
// every source sent a VERIFY of the expected shape and sequences whose
// positions lie inside the KV pages reserved for them, writes the verify
// graph's integer inputs (token ids, positions, KV slots, causal row limits,
// key ends) straight from the messages -- the host never touches the request
// on the critical path.  Otherwise the inputs become placeholders (every KV
// store goes to one scratch slot, keys end at K) and ``gate`` is cleared, so
// the reply kernels after the graph send nothing and the host handles the
// messages.  Status per source (pinned): 0 matched, 1 another message
// arrived, 2 nothing arrived in time; [n_src] is 0 when the verify is valid.
// On a tensor-parallel target every rank runs the same graphs, so rank 0
// alone decides (its bounded waits and checks above) and publishes the
// decision into each other rank's memory with peer stores and a release
// flag stamped with the arm's epoch; the other ranks wait (bounded) for it
// and for their own copies of the messages it saw, and follow it.  A
// follower that gets no decision, or whose messages disagree with it,
// reports status 3 and its host ends serving.
__global__ void verify_arm_kernel(ArmArgs a) {
  __shared__ int arrived[ARM_MAX_SRC];
  __shared__ int lead_st[ARM_MAX_SRC];
  __shared__ int valid, lost;
  const int tid = threadIdx.x;
  if (a.role == 2) {
    // follower: take rank 0's decision (bounded, well above rank 0's own
    // bound), then wait for the messages rank 0 saw arrive in this inbox
    if (tid == 0) {
      lost = 0;
      valid = 0;
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(a.dec_in) < a.epoch) {
        if (globaltimer_ns() - t0 > 3 * a.limit_ns) {
          lost = 1;
          break;
        }
      }
      for (int d = 0; d < a.n_src; ++d) {
        lead_st[d] = lost ? 2 : static_cast<int>(reinterpret_cast<const volatile int64_t*>(a.dec_in)[1 + d]);
        arrived[d] = 0;
      }
      if (!lost) valid = static_cast<int>(reinterpret_cast<const volatile int64_t*>(a.dec_in)[1 + a.n_src]);
      for (int d = 0; d < a.n_src && !lost; ++d) {
        if (lead_st[d] == 2) continue;
        const uint64_t t1 = globaltimer_ns();
        while (ld_acquire_sys(a.flag[d]) < a.seq[d]) {
          if (globaltimer_ns() - t1 > a.limit_ns) {
            lost = 1;
            break;
          }
        }
        arrived[d] = !lost;
      }
      if (lost) valid = 0;
    }
  } else if (tid < a.n_src) {
    arrived[tid] = 1;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(a.flag[tid]) < a.seq[tid]) {
      if (globaltimer_ns() - t0 > a.limit_ns) {
        arrived[tid] = 0;
        break;
      }
    }
  }
  __syncthreads();
  for (int d = 0; d < a.n_src; ++d) {
    if (!arrived[d]) continue;
    const uint4* src = reinterpret_cast<const uint4*>(a.msg[d]);
    uint4* dst = reinterpret_cast<uint4*>(a.head[d]);
    for (int i = tid; i < a.head_words / 2; i += blockDim.x) dst[i] = __ldcv(src + i);
  }
  const int B = a.row0[a.n_src - 1] + a.nb[a.n_src - 1];
  const int64_t* exp_sid = a.tab;
  const int64_t* reserved = a.tab + B;
  if (tid == 0) {
    // the follower checks too (memory safety): a follower that finds the
    // messages unlike its leader's decision reports the group as lost
    int ok = a.role == 2 ? valid : 1;
    for (int d = 0; d < a.n_src && ok; ++d) {
      const volatile int64_t* m = a.msg[d];
      if (!arrived[d] || m[0] != 2 || m[1] != a.nb[d] || m[2] != a.K) {
        ok = 0;
        break;
      }
      for (int b = 0; b < a.nb[d]; ++b) {
        const int r = a.row0[d] + b;
        const int64_t p = m[8 + 2 * b + 1];
        if (m[8 + 2 * b] != exp_sid[r] || p < 0 || p + a.K > reserved[r]) {
          ok = 0;
          break;
        }
      }
    }
    if (a.role == 2 && valid && !ok) lost = 1;
    valid = ok;
    if (a.role == 1) {
      // publish the decision to every follower before this rank's graph runs
      for (int f = 0; f < a.n_follow; ++f) {
        int64_t* rec = a.dec_out[f];
        for (int d = 0; d < a.n_src; ++d) rec[1 + d] = arrived[d] ? (ok ? 0 : 1) : 2;
        rec[1 + a.n_src] = ok;
      }
      __threadfence_system();
      for (int f = 0; f < a.n_follow; ++f) st_release_sys(a.dec_out[f], a.epoch);
    }
  }
  __syncthreads();
  const int T = B * a.K;
  for (int t = tid; t < T; t += blockDim.x) {
    const int r = t / a.K, i = t - r * a.K;
    if (valid) {
      int d = 0;
      while (d + 1 < a.n_src && r >= a.row0[d + 1]) ++d;
      const int b = r - a.row0[d];
      const int64_t* m = a.msg[d];
      const int64_t p = __ldcv(m + 8 + 2 * b + 1) + i;
      const int64_t row = a.seq_rows[r];
      a.ids[t] = __ldcv(m + 8 + 2 * a.nb[d] + static_cast<int64_t>(b) * a.K + i);
      a.pos[t] = p;
      const int64_t page = a.block_table[row * a.bt_stride + p / a.page];
      a.slots[t] = page * a.page + p % a.page;
      a.rows[3 * t] = static_cast<int32_t>(p + 1);
      if (i == 0) a.kv_end[r] = static_cast<int32_t>(p + a.K);
    } else {
      a.ids[t] = 0;
      a.pos[t] = i;
      a.slots[t] = a.scratch_slot;
      a.rows[3 * t] = i + 1;
      if (i == 0) a.kv_end[r] = a.K;
    }
    a.rows[3 * t + 1] = 0;
    a.rows[3 * t + 2] = 0;
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    const bool gone = a.role == 2 && lost;
    *a.gate = valid;
    for (int d = 0; d < a.n_src; ++d) {
      int st = 2;
      if (gone) st = 3;
      else if (arrived[d]) st = valid ? 0 : 1;
      reinterpret_cast<volatile int*>(a.status)[d] = st;
    }
    __threadfence_system();
    reinterpret_cast<volatile int*>(a.status)[a.n_src] = gone ? 3 : (valid ? 0 : 1);
  }
}

void verify_arm(const ArmArgs& a, cudaStream_t st) {
  if (a.n_src < 1 || a.n_src > ARM_MAX_SRC) throw std::runtime_error("verify_arm: 1..8 sources");
  if (a.head_words % 2) throw std::runtime_error("verify_arm: head_words must be even");
  verify_arm_kernel<<<1, 256, 0, st>>>(a);
}

// ------------------------------------------------ device branch select (drafter)
// The drafter enqueues this behind its packed forward, before the target's
// reply exists: it waits -- bounded -- for reply ``rseq``, copies its first
// ``head_words`` into pinned host memory (the host's receive reads it there),
// and for every row looks up the drafted branch keyed by the outcome
// (commit length, and the correction token unless the whole block was
// accepted or no anchor branches are drafted).  When every row continues
// (commit below its finishing limit, correction not a stop token) and has a
// branch, it writes the next VERIFY request -- correction + the branch's
// drafts 1..K-1 (from the forward's top-1 ids, or the controlled-acceptance
// drafts of the row's positions) -- into the target rank(s)' inboxes with
// peer stores and raises their flags.  Otherwise it sends nothing and the
// host takes the step.  status (pinned): [0] 0 reply arrived / 2 not in time,
// [1] 1 request sent / 0 not.
__global__ void select_send_kernel(SelectArgs a) {
  __shared__ int ok, arrived;
  __shared__ int sn[SEL_MAX_ROWS], sj[SEL_MAX_ROWS];
  __shared__ int64_t scorr[SEL_MAX_ROWS];
  const int tid = threadIdx.x;
  const int B = a.B, K = a.K;
  if (tid == 0) {
    arrived = 1;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(a.rflag) < a.rseq) {
      if (globaltimer_ns() - t0 > a.limit_ns) {
        arrived = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (arrived) {
    const uint4* src = reinterpret_cast<const uint4*>(a.reply);
    uint4* dst = reinterpret_cast<uint4*>(a.reply_host);
    for (int i = tid; i < a.head_words / 2; i += blockDim.x) dst[i] = __ldcv(src + i);
  }
  const int64_t* sid = a.tab;
  const int64_t* prefix = a.tab + B;
  const int64_t* n_limit = a.tab + 2 * B;
  const int64_t* keys = a.tab + 3 * B;
  const int64_t* key_rows = keys + static_cast<size_t>(B) * a.nk * 2;
  const int64_t* eos = key_rows + static_cast<size_t>(B) * a.nk;
  const int64_t* ctrl = eos + a.n_eos;
  if (tid == 0) {
    const volatile int64_t* r = a.reply;
    int good = arrived && B <= SEL_MAX_ROWS && r[0] == 2 && r[1] == B && r[2] == K;
    for (int b = 0; b < B && good; ++b) {
      const int64_t n = r[8 + static_cast<int64_t>(b) * (2 + K)];
      const int64_t corr = r[8 + static_cast<int64_t>(b) * (2 + K) + 1];
      if (n < 1 || n > K || n >= n_limit[b]) good = 0;
      for (int e = 0; e < a.n_eos && good; ++e)
        if (corr == eos[e]) good = 0;
      const int64_t key = (n == K || a.a0) ? -1 : corr;
      int j = -1;   // the last branch with this key, as the host's key -> branch map keeps
      for (int q = 0; q < a.nk && good; ++q) {
        const int64_t* kq = keys + (static_cast<size_t>(b) * a.nk + q) * 2;
        if (kq[0] == n && kq[1] == key) j = q;
      }
      if (j < 0) good = 0;
      sn[b] = static_cast<int>(n);
      sj[b] = j;
      scorr[b] = corr;
    }
    ok = good;
  }
  __syncthreads();
  if (ok) {
    const int words = 8 + 2 * B + B * K;
    for (int w = tid; w < words; w += blockDim.x) {
      int64_t v = 0;
      if (w < 8) {
        v = w == 0 ? 2 : (w == 1 ? B : (w == 2 ? K : 0));
      } else if (w < 8 + 2 * B) {
        const int b = (w - 8) >> 1;
        v = ((w - 8) & 1) ? prefix[b] + sn[b] : sid[b];
      } else {
        const int idx = w - 8 - 2 * B;
        const int b = idx / K, i = idx - b * K;
        if (i == 0) v = scorr[b];
        else if (a.ctrl) v = ctrl[static_cast<size_t>(b) * 2 * K + sn[b] + i - 1];
        else v = a.top[(key_rows[static_cast<size_t>(b) * a.nk + sj[b]] + i) * a.top_stride];
      }
      for (int o = 0; o < a.n_out; ++o) a.out_slot[o][w] = v;
    }
    __threadfence_system();
  }
  __syncthreads();
  if (tid == 0) {
    if (ok)
      for (int o = 0; o < a.n_out; ++o) st_release_sys(a.out_flag[o], a.out_seq[o]);
    reinterpret_cast<volatile int*>(a.status)[0] = arrived ? 0 : 2;
    __threadfence_system();
    reinterpret_cast<volatile int*>(a.status)[1] = ok;
  }
}

void select_send(const SelectArgs& a, cudaStream_t st) {
  if (a.n_out < 1 || a.n_out > ARM_MAX_SRC) throw std::runtime_error("select_send: 1..8 destinations");
  if (a.B < 1 || a.B > SEL_MAX_ROWS) throw std::runtime_error("select_send: 1..64 rows");
  if (a.head_words % 2) throw std::runtime_error("select_send: head_words must be even");
  select_send_kernel<<<1, 256, 0, st>>>(a);
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
