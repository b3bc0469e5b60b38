// Tensor-parallel exchange kernels (sm_100a, one process per GPU).  The
// reference's tensor-parallel layers exist but run at tp_size=1
// (serving/vendor/ssd/layers/linear.py:68-199, embed_head.py:9-116).
//
// The target's row-parallel GEMMs (o_proj, down_proj) push their fp32
// split-K partials from the GEMM epilogue into every rank's exchange region
// (peer stores over NVLink into buffers mapped through CUDA IPC; see the
// tensor-parallel branch of gemm_tcgen05.cu), and the GEMM's last CTA
// publishes "exchange x of forward e is ready" on every rank with a
// system-scope release store.  The consumer -- add_rmsnorm_tp, the residual
// add + RMSNorm of the next sublayer -- waits (bounded, acquire) for all
// ranks' flags, then sums the TP x S partials of each element from local
// memory in a fixed order (rank-major, then split).  That is an all-reduce
// fused into the GEMM epilogue and into the reduction the single-GPU path
// already does, with the same batch-invariant order.  (tp_signal remains for
// producers that are not GEMMs.)  The vocab-parallel LM head exchanges per-rank top-k
// candidates the same way (topk_merge_tp).
//
// Exchange regions are double-buffered by exchange parity: rank A rewrites a
// buffer two exchanges after a peer read it, and the peer's read is ordered
// before that by the flags of the exchange in between.  The forward's epoch
// (a device counter bumped at the start of every forward) is the flag value,
// so captured graphs need no host-side arguments per call.
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"

namespace d3d {

__device__ __forceinline__ void st_release_sys_i64(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int64_t ld_acquire_sys_i64(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void tp_epoch_bump_kernel(int64_t* epoch) {
  griddep_launch();
  griddep_wait();
  if (threadIdx.x == 0) *epoch += 1;
}

// flag arrays: flags_r[x * tp + src] on rank r = epoch at which src published exchange x
__global__ void tp_signal_kernel(const TpArgs a, int x) {
  griddep_launch();
  griddep_wait();
  if (threadIdx.x != 0) return;
  const int64_t e = *a.epoch;
  __threadfence_system();
  for (int j = 0; j < a.tp; ++j) st_release_sys_i64(a.flags[j] + static_cast<size_t>(x) * a.tp + a.rank, e);
}

// Bounded wait (thread 0) for every rank's flag of exchange x; false on timeout.
__device__ __forceinline__ bool tp_wait_all(const TpArgs& a, int x) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const int64_t e = *a.epoch;
    const int64_t* f = a.flags[a.rank] + static_cast<size_t>(x) * a.tp;
    const uint64_t t0 = globaltimer_ns();
    for (int j = 0; j < a.tp && ok; ++j) {
      while (ld_acquire_sys_i64(f + j) < e) {
        if (globaltimer_ns() - t0 > a.timeout_ns) {
          set_error(a.status, ERR_TIMEOUT_FLAG);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__device__ __forceinline__ float4 ldcv4(const float* p) { return __ldcv(reinterpret_cast<const float4*>(p)); }

// candidate slot layout: n float values, then n int64 ids at the next 8-byte boundary
__host__ __device__ inline size_t cand_ids_off(int n) { return (static_cast<size_t>(n) * 4 + 7) & ~size_t(7); }

// x = bf16(residual + bf16(sum_{rank, split} P)); residual <- x; out = w * bf16(x * rstd)
template <int V>
__global__ void __launch_bounds__(512) add_rmsnorm_tp_kernel(const TpArgs a, int x, size_t part_off, int nsplit, int pull,
                                                             __nv_bfloat16* __restrict__ residual,
                                                             const __nv_bfloat16* __restrict__ w,
                                                             __nv_bfloat16* __restrict__ out, int M, int N,
                                                             float eps) {
  griddep_launch();
  griddep_wait();
  const int m = blockIdx.x;
  if (!tp_wait_all(a, x) || m >= M) return;
  __shared__ float red[32];
  float xv[V][4];
  float ss = 0.f;
  const size_t stride = static_cast<size_t>(M) * N;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int n = 4 * (threadIdx.x + i * blockDim.x);
#pragma unroll
    for (int j = 0; j < 4; ++j) xv[i][j] = 0.f;
    if (n < N) {
      const size_t off = static_cast<size_t>(m) * N + n;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      // slots [rank][split]: all in this rank's buffer (pushed by the peers'
      // GEMMs), or slot rank r in rank r's buffer (read over NVLink: pull)
      for (int r = 0; r < a.tp; ++r) {
        const float* base = reinterpret_cast<const float*>(a.parts[pull ? r : a.rank] + part_off) +
                            static_cast<size_t>(r) * nsplit * stride;
        float4 v[16];
#pragma unroll
        for (int s = 0; s < 16; ++s)
          if (s < nsplit) v[s] = ldcv4(base + s * stride + off);
#pragma unroll
        for (int s = 0; s < 16; ++s)
          if (s < nsplit) {
            acc[0] += v[s].x;
            acc[1] += v[s].y;
            acc[2] += v[s].z;
            acc[3] += v[s].w;
          }
      }
      const uint2 raw = *reinterpret_cast<const uint2*>(residual + off);
      const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&raw);
      __align__(8) __nv_bfloat16 o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xv[i][j] = bf16r(__bfloat162float(rb[j]) + bf16r(acc[j]));
        o[j] = __float2bfloat16(xv[i][j]);
      }
      *reinterpret_cast<uint2*>(residual + off) = *reinterpret_cast<const uint2*>(o);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) ss += xv[i][j] * xv[i][j];
  }
  ss = warp_sum(ss);
  const int wid = threadIdx.x >> 5, lid = threadIdx.x & 31;
  if (lid == 0) red[wid] = ss;
  __syncthreads();
  if (wid == 0) {
    float t = lid < (blockDim.x >> 5) ? red[lid] : 0.f;
    t = warp_sum(t);
    if (lid == 0) red[0] = t;
  }
  __syncthreads();
  const float rs = rsqrtf(red[0] / N + eps);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int n = 4 * (threadIdx.x + i * blockDim.x);
    if (n < N) {
      const uint2 raw = *reinterpret_cast<const uint2*>(w + n);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&raw);
      __align__(8) __nv_bfloat16 o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = __float2bfloat16(bf16r(xv[i][j] * rs) * __bfloat162float(wb[j]));
      *reinterpret_cast<uint2*>(out + static_cast<size_t>(m) * N + n) = *reinterpret_cast<const uint2*>(o);
    }
  }
}

// Candidates of rank r at cand_off in its region: [M][k] float values then
// [M][k] int64 indices (already global vocabulary ids).  Every rank merges all
// ranks' lists in rank order (descending value, ties to the lower id).
__global__ void topk_merge_tp_kernel(const TpArgs a, int x, size_t cand_off, int M, int k, float* __restrict__ ov,
                                     int64_t* __restrict__ oi) {
  griddep_launch();
  griddep_wait();
  if (!tp_wait_all(a, x)) return;
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  float bv[4];
  int64_t bi[4];
  for (int q = 0; q < 4; ++q) {
    bv[q] = -INFINITY;
    bi[q] = INT64_MAX;
  }
  for (int r = 0; r < a.tp; ++r) {
    const float* vals = reinterpret_cast<const float*>(a.parts[r] + cand_off);
    const int64_t* ids = reinterpret_cast<const int64_t*>(a.parts[r] + cand_off + cand_ids_off(M * k));
    for (int c = 0; c < k; ++c) {
      float v = __ldcv(vals + static_cast<size_t>(m) * k + c);
      int64_t id = __ldcv(reinterpret_cast<const long long*>(ids) + static_cast<size_t>(m) * k + c);
      for (int q = 0; q < k; ++q) {
        if (v > bv[q] || (v == bv[q] && id < bi[q])) {
          const float t1 = bv[q];
          const int64_t t2 = bi[q];
          bv[q] = v;
          bi[q] = id;
          v = t1;
          id = t2;
        }
      }
    }
  }
  for (int q = 0; q < k; ++q) {
    if (ov) ov[static_cast<size_t>(m) * k + q] = bv[q];
    oi[static_cast<size_t>(m) * k + q] = bi[q];
  }
}

// Local top-k (already merged over this rank's vocabulary tiles) -> this
// rank's candidate slot, with local ids shifted to global vocabulary ids.
__global__ void tp_publish_topk_kernel(const float* __restrict__ lv, const int64_t* __restrict__ li, int M, int k,
                                       int64_t id_offset, uint8_t* cand) {
  griddep_launch();
  griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int n = M * k;
  if (i >= n) return;
  float* vals = reinterpret_cast<float*>(cand);
  int64_t* ids = reinterpret_cast<int64_t*>(cand + cand_ids_off(n));
  vals[i] = lv[i];
  ids[i] = li[i] + id_offset;
}

void tp_epoch_bump(int64_t* epoch, cudaStream_t st) { launch_pdl(tp_epoch_bump_kernel, dim3(1), dim3(32), 0, st, epoch); }

void tp_signal(const TpArgs& a, int x, cudaStream_t st) {
  if (a.tp > TP_MAX) throw std::runtime_error("tp_signal: tp size too large");
  launch_pdl(tp_signal_kernel, dim3(1), dim3(32), 0, st, a, x);
}

void add_rmsnorm_tp(const TpArgs& a, int x, size_t part_off, int nsplit, int pull, __nv_bfloat16* residual,
                    const __nv_bfloat16* w, __nv_bfloat16* out, int M, int N, float eps, cudaStream_t st) {
  if (M == 0) return;
  if (N % 4) throw std::runtime_error("add_rmsnorm_tp: hidden size must be a multiple of 4");
  if (nsplit < 1 || nsplit > 16) throw std::runtime_error("add_rmsnorm_tp: 1..16 splits");
  const int vec = N / 4;
  const int threads = vec >= 512 ? 512 : (vec + 31) / 32 * 32;
  const int v = (vec + threads - 1) / threads;
  if (v <= 1)
    launch_pdl(add_rmsnorm_tp_kernel<1>, dim3(M), dim3(threads), 0, st, a, x, part_off, nsplit, pull, residual, w, out, M,
               N, eps);
  else if (v <= 2)
    launch_pdl(add_rmsnorm_tp_kernel<2>, dim3(M), dim3(threads), 0, st, a, x, part_off, nsplit, pull, residual, w, out, M,
               N, eps);
  else if (v <= 4)
    launch_pdl(add_rmsnorm_tp_kernel<4>, dim3(M), dim3(threads), 0, st, a, x, part_off, nsplit, pull, residual, w, out, M,
               N, eps);
  else
    throw std::runtime_error("add_rmsnorm_tp: hidden size above 8192");
}

void tp_publish_topk(const float* lv, const int64_t* li, int M, int k, int64_t id_offset, uint8_t* cand,
                     cudaStream_t st) {
  const int n = M * k;
  launch_pdl(tp_publish_topk_kernel, dim3((n + 255) / 256), dim3(256), 0, st, lv, li, M, k, id_offset, cand);
}

void topk_merge_tp(const TpArgs& a, int x, size_t cand_off, int M, int k, float* ov, int64_t* oi, cudaStream_t st) {
  if (k > 4) throw std::runtime_error("topk_merge_tp: k <= 4");
  launch_pdl(topk_merge_tp_kernel, dim3((M + 127) / 128), dim3(128), 0, st, a, x, cand_off, M, k, ov, oi);
}

}  // namespace d3d
