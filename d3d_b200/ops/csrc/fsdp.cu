// Sharded-optimizer step fused with its collectives over NVLink (sm_100a).
// The reference shards with FSDP2 through Accelerate (train/runtime.py:70-114).
//
// Every rank keeps its full fp32 gradient and its full bf16 parameter copy in
// device buffers that all peers have mapped through CUDA IPC.  Rank r owns
// elements [lo_r, lo_r + shard) of the flattened model:
//
//   fsdp_reduce   waits (bounded) until every rank has published "gradients of
//                 step e ready", then reads its shard from every rank's
//                 gradient buffer (peer loads, summed in rank order -- a
//                 reduce-scatter), stores the reduced shard locally and
//                 accumulates its squared norm (for clipping);
//   fsdp_update   AdamW on the fp32 master shard with the reduced gradient
//                 times one scale (1/world and the clip factor), casts to bf16
//                 and stores the new shard into every rank's parameter buffer
//                 (peer stores -- an all-gather); the last CTA raises "shard
//                 of step e written" on every rank;
//   fsdp_wait     bounded wait for every rank's "written" flag.
//
// That replaces NCCL reduce-scatter + AdamW + NCCL all-gather.  A rank never
// rewrites a buffer a peer may still read: gradients of step e+1 are written
// after fsdp_wait of step e, which follows every rank's fsdp_reduce of step e.
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"

namespace d3d {

__device__ __forceinline__ void fs_release(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int64_t fs_acquire(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// thread 0 of the block: wait until flags[j] >= e for every rank j
__device__ bool fs_wait(const int64_t* flags, int world, int64_t e, int* status, unsigned long long limit) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int j = 0; j < world && ok; ++j)
      while (fs_acquire(flags + j) < e) {
        if (globaltimer_ns() - t0 > limit) {
          set_error(status, ERR_TIMEOUT_FLAG);
          ok = 0;
          break;
        }
      }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void fsdp_signal_kernel(FsdpArgs a, int phase, int64_t e) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  for (int j = 0; j < a.world; ++j) fs_release(a.flags[j] + phase * FSDP_MAX + a.rank, e);
}

__global__ void fsdp_reduce_kernel(FsdpArgs a, int64_t e, float* __restrict__ gshard, float* __restrict__ sumsq) {
  if (!fs_wait(a.flags[a.rank] + 0 * FSDP_MAX, a.world, e, a.status, a.timeout_ns)) return;
  float acc = 0.f;
  const size_t n4 = a.shard / 4;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float4 v[FSDP_MAX];
#pragma unroll
    for (int j = 0; j < FSDP_MAX; ++j)
      if (j < a.world) v[j] = __ldcv(reinterpret_cast<const float4*>(a.grads[j] + a.lo) + i);
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < FSDP_MAX; ++j)
      if (j < a.world) {
        s.x += v[j].x;
        s.y += v[j].y;
        s.z += v[j].z;
        s.w += v[j].w;
      }
    reinterpret_cast<float4*>(gshard)[i] = s;
    acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
  }
  acc = warp_sum(acc);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) atomicAdd(sumsq, t);
  }
}

__global__ void fsdp_update_kernel(FsdpArgs a, int64_t e, const float* __restrict__ gshard, float* __restrict__ p,
                                   float* __restrict__ m, float* __restrict__ v, float lr, float b1, float b2,
                                   float eps, float wd, float bc1, float bc2, float scale, unsigned int* ticket) {
  const size_t n = a.shard;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float gi = gshard[i] * scale;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float pi = p[i] * (1.f - lr * wd);
    pi -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    p[i] = pi;
    const __nv_bfloat16 o = __float2bfloat16(pi);
    for (int j = 0; j < a.world; ++j) a.params[j][a.lo + i] = o;   // the all-gather, by peer stores
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int t = atomicAdd(ticket, 1u);
    if (t == gridDim.x - 1) {
      *ticket = 0;
      __threadfence_system();
      for (int j = 0; j < a.world; ++j) fs_release(a.flags[j] + 1 * FSDP_MAX + a.rank, e);
    }
  }
}

__global__ void fsdp_wait_kernel(FsdpArgs a, int phase, int64_t e) {
  fs_wait(a.flags[a.rank] + phase * FSDP_MAX, a.world, e, a.status, a.timeout_ns);
}

static void check(const FsdpArgs& a) {
  if (a.world < 1 || a.world > FSDP_MAX) throw std::runtime_error("fsdp: world size 1..8");
  if (a.shard % 4 || a.lo % 4) throw std::runtime_error("fsdp: shard size and offset must be multiples of 4");
}

void fsdp_signal(const FsdpArgs& a, int phase, int64_t e, cudaStream_t st) {
  check(a);
  fsdp_signal_kernel<<<1, 32, 0, st>>>(a, phase, e);
}

void fsdp_reduce(const FsdpArgs& a, int64_t e, float* gshard, float* sumsq, cudaStream_t st) {
  check(a);
  size_t blocks = (a.shard / 4 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  fsdp_reduce_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(a, e, gshard, sumsq);
}

void fsdp_update(const FsdpArgs& a, int64_t e, const float* gshard, float* p, float* m, float* v, float lr, float b1,
                 float b2, float eps, float wd, int step, float scale, unsigned int* ticket, cudaStream_t st) {
  check(a);
  const float bc1 = 1.f - powf(b1, static_cast<float>(step));
  const float bc2 = 1.f - powf(b2, static_cast<float>(step));
  size_t blocks = (a.shard + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  fsdp_update_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(a, e, gshard, p, m, v, lr, b1, b2, eps, wd, bc1,
                                                                     bc2, scale, ticket);
}

void fsdp_wait(const FsdpArgs& a, int phase, int64_t e, cudaStream_t st) {
  check(a);
  fsdp_wait_kernel<<<1, 32, 0, st>>>(a, phase, e);
}

// Parameter all-gather of sharded (FSDP-style) layers: dst[r * n + i] =
// params[r][off + i] for every rank r -- rank r's shard of one layer, read
// over NVLink from its parameter buffer (peer loads, 16-byte vectors when
// the offsets allow).  Shards change only in the optimizer step, which the
// trainer orders before the next forward on every rank, so no flag is needed.
__global__ void fsdp_gather_kernel(FsdpArgs a, size_t off, size_t n, __nv_bfloat16* __restrict__ dst) {
  griddep_launch();
  griddep_wait();
  const int r = blockIdx.y;
  const __nv_bfloat16* src = a.params[r] + off;
  __nv_bfloat16* out = dst + static_cast<size_t>(r) * n;
  const bool vec = ((off | n) & 7) == 0;
  if (vec) {
    const size_t n8 = n / 8;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
      reinterpret_cast<uint4*>(out)[i] = __ldcv(reinterpret_cast<const uint4*>(src) + i);
  } else {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
      out[i] = src[i];
  }
}

void fsdp_gather(const FsdpArgs& a, size_t off, size_t n, __nv_bfloat16* dst, cudaStream_t st) {
  if (n == 0) return;
  size_t per = (n / 8 + 255) / 256;
  const int bx = static_cast<int>(per < 64 ? (per == 0 ? 1 : per) : 64);
  launch_pdl(fsdp_gather_kernel, dim3(bx, a.world), dim3(256), 0, st, a, off, n, dst);
}

}  // namespace d3d
