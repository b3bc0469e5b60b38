// Training kernels (sm_100a): distillation loss over vocabulary chunks and
// the sharded AdamW update (reference: train/objective_kernels.py:7-37 full-vocab
// KL in PyTorch, train/losses.py:209-315 chunked CE, AdamW via FSDP2 in
// train/runtime.py:70-114).
//
// The LM-head loss never materialises [N, V] logits.  The vocabulary is
// walked in chunks of C columns; for each chunk the teacher and student
// logit tiles are produced by the tcgen05 GEMM (fp32, [N, C]) and folded into
// per-row running statistics by kl_ce_stats_kernel in one pass (online max,
// fixed chunk and lane order, so the result is deterministic):
//   M_t, S_t = max and sum of exp(z_t - M_t)               (teacher LSE)
//   A_tt     = sum exp(z_t - M_t) * z_t
//   A_ts     = sum exp(z_t - M_t) * z_s
//   M_s, S_s = max and sum of exp(z_s - M_s)               (student LSE)
//   z_s[target]
// from which forward KL(p_t || p_s) = (A_tt - A_ts)/S_t - LSE_t + LSE_s and
// CE = LSE_s - z_s[target].  The backward recomputes the chunk logits and
// kl_ce_grad_kernel writes dz = w_kl (softmax(z_s) - p_t) + w_ce (softmax(z_s)
// - onehot(target)) in bf16, both [N, C] and transposed [C, N] (the layouts
// of the two gradient GEMMs).
#include "common.cuh"
#include "kernels.h"

namespace d3d {

constexpr int ST_M_T = 0, ST_S_T = 1, ST_A_TT = 2, ST_A_TS = 3, ST_M_S = 4, ST_S_S = 5, ST_ZTGT = 6, ST_N = 8;

__device__ __forceinline__ void lse_merge(float& m, float& s, float om, float os) {
  if (om == -INFINITY) return;
  if (m == -INFINITY) {
    m = om;
    s = os;
    return;
  }
  const float nm = fmaxf(m, om);
  s = s * __expf(m - nm) + os * __expf(om - nm);
  m = nm;
}

// Online fold of one logit into a lane's running (max, sum of exp) -- and,
// for the teacher, the exp-weighted sums of its own and the student's logit.
// The sums are rescaled only when the running max rises.
__device__ __forceinline__ void fold_student(float y, float& ms, float& ss) {
  if (y > ms) {
    ss = ss * __expf(ms - y) + 1.f;
    ms = y;
  } else {
    ss += __expf(y - ms);
  }
}
__device__ __forceinline__ void fold_teacher(float x, float y, float& mt, float& st, float& att, float& ats) {
  if (x > mt) {
    const float f = __expf(mt - x);
    st = st * f + 1.f;
    att = att * f + x;
    ats = ats * f + y;
    mt = x;
  } else {
    const float e = __expf(x - mt);
    st += e;
    att += e * x;
    ats += e * y;
  }
}
// Merge another lane's state (m, s[, a, b]) into this one.
__device__ __forceinline__ void merge_state(float& m, float& s, float& a, float& b, float om, float os, float oa,
                                            float ob) {
  const float nm = fmaxf(m, om);
  if (nm == -INFINITY) return;
  const float f1 = m == -INFINITY ? 0.f : __expf(m - nm);
  const float f2 = om == -INFINITY ? 0.f : __expf(om - nm);
  s = s * f1 + os * f2;
  a = a * f1 + oa * f2;
  b = b * f1 + ob * f2;
  m = nm;
}

// One warp per row, one pass over the chunk (every logit read once; float4
// loads when VEC).  zt/zs: [N, ldz] fp32 chunk logits (columns [0, C)); the
// chunk covers vocabulary ids [v0, v0 + C).  zt may be null (CE only).
// Lanes fold their columns (lane-strided), then a fixed butterfly merges the
// lane states, so the result is deterministic.
template <bool VEC>
__global__ void kl_ce_stats_kernel(const float* __restrict__ zt, const float* __restrict__ zs, int N, int C,
                                   int ldz, int v0, const int64_t* __restrict__ target, float* __restrict__ st) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= N) return;
  const float* a = zt ? zt + static_cast<size_t>(row) * ldz : nullptr;
  const float* b = zs + static_cast<size_t>(row) * ldz;
  float mt = -INFINITY, s_t = 0.f, att = 0.f, ats = 0.f, ms = -INFINITY, s_s = 0.f;
  if (VEC) {
    for (int c = lane * 4; c < C; c += 128) {
      const float4 y4 = __ldcs(reinterpret_cast<const float4*>(b + c));
      const float y[4] = {y4.x, y4.y, y4.z, y4.w};
      if (a) {
        const float4 x4 = __ldcs(reinterpret_cast<const float4*>(a + c));
        const float x[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) fold_teacher(x[j], y[j], mt, s_t, att, ats);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) fold_student(y[j], ms, s_s);
    }
  } else {
    for (int c = lane; c < C; c += 32) {
      const float y = b[c];
      if (a) fold_teacher(a[c], y, mt, s_t, att, ats);
      fold_student(y, ms, s_s);
    }
  }
  float dummy0 = 0.f, dummy1 = 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float omt = __shfl_xor_sync(0xffffffffu, mt, o), ost = __shfl_xor_sync(0xffffffffu, s_t, o);
    const float oatt = __shfl_xor_sync(0xffffffffu, att, o), oats = __shfl_xor_sync(0xffffffffu, ats, o);
    const float oms = __shfl_xor_sync(0xffffffffu, ms, o), oss = __shfl_xor_sync(0xffffffffu, s_s, o);
    merge_state(mt, s_t, att, ats, omt, ost, oatt, oats);
    merge_state(ms, s_s, dummy0, dummy1, oms, oss, 0.f, 0.f);
  }
  if (lane == 0) {
    float* r = st + static_cast<size_t>(row) * ST_N;
    if (a && mt != -INFINITY) {
      // rescale the running teacher accumulators to the new maximum
      float M = r[ST_M_T];
      const float nm = fmaxf(M, mt);
      const float f_old = M == -INFINITY ? 0.f : __expf(M - nm);
      const float f_new = __expf(mt - nm);
      r[ST_S_T] = r[ST_S_T] * f_old + s_t * f_new;
      r[ST_A_TT] = r[ST_A_TT] * f_old + att * f_new;
      r[ST_A_TS] = r[ST_A_TS] * f_old + ats * f_new;
      r[ST_M_T] = nm;
    }
    float m = r[ST_M_S], s = r[ST_S_S];
    lse_merge(m, s, ms, s_s);
    r[ST_M_S] = m;
    r[ST_S_S] = s;
    const int64_t t = target ? target[row] : -1;
    if (t >= v0 && t < v0 + C) r[ST_ZTGT] = b[t - v0];
  }
}

void kl_ce_stats(const float* zt, const float* zs, int N, int C, int ldz, int v0, const int64_t* target, float* st,
                 cudaStream_t s) {
  if (N == 0) return;
  const bool vec = C % 4 == 0 && ldz % 4 == 0 && (reinterpret_cast<uintptr_t>(zs) & 15) == 0 &&
                   (zt == nullptr || (reinterpret_cast<uintptr_t>(zt) & 15) == 0);
  if (vec) kl_ce_stats_kernel<true><<<(N * 32 + 255) / 256, 256, 0, s>>>(zt, zs, N, C, ldz, v0, target, st);
  else kl_ce_stats_kernel<false><<<(N * 32 + 255) / 256, 256, 0, s>>>(zt, zs, N, C, ldz, v0, target, st);
}

// dz[n, c] = w_kl[n] (softmax_s - p_t) + w_ce[n] (softmax_s - onehot); lse_t/lse_s per row.
__global__ void kl_ce_grad_kernel(const float* __restrict__ zt, const float* __restrict__ zs, int N, int C, int ldz,
                                  int v0, const int64_t* __restrict__ target, const float* __restrict__ lse_t,
                                  const float* __restrict__ lse_s, const float* __restrict__ w_kl,
                                  const float* __restrict__ w_ce, __nv_bfloat16* __restrict__ dz, int ld_dz,
                                  __nv_bfloat16* __restrict__ dzT, int ld_dzT) {
  const size_t total = static_cast<size_t>(N) * C;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    // column-fastest within a row keeps the zt/zs reads coalesced
    const int n = static_cast<int>(i / C), c = static_cast<int>(i % C);
    const float ps = __expf(zs[static_cast<size_t>(n) * ldz + c] - lse_s[n]);
    float g = 0.f;
    if (w_kl && zt) g += w_kl[n] * (ps - __expf(zt[static_cast<size_t>(n) * ldz + c] - lse_t[n]));
    if (w_ce) g += w_ce[n] * (ps - (target && target[n] == v0 + c ? 1.f : 0.f));
    const __nv_bfloat16 gb = __float2bfloat16(g);
    if (dz) dz[static_cast<size_t>(n) * ld_dz + c] = gb;
    if (dzT) dzT[static_cast<size_t>(c) * ld_dzT + n] = gb;
  }
}

void kl_ce_grad(const float* zt, const float* zs, int N, int C, int ldz, int v0, const int64_t* target,
                const float* lse_t, const float* lse_s, const float* w_kl, const float* w_ce, __nv_bfloat16* dz,
                int ld_dz, __nv_bfloat16* dzT, int ld_dzT, cudaStream_t s) {
  const size_t total = static_cast<size_t>(N) * C;
  if (total == 0) return;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  kl_ce_grad_kernel<<<blocks, 256, 0, s>>>(zt, zs, N, C, ldz, v0, target, lse_t, lse_s, w_kl, w_ce, dz, ld_dz, dzT,
                                            ld_dzT);
}

// --------------------------------------------------------------- AdamW
// Decoupled-weight-decay Adam on an fp32 master shard; the updated value is
// also written in bf16 (the compute copy that is all-gathered).  grad_scale
// folds the data-parallel mean and the global-norm clip coefficient.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ out, size_t n, float lr, float b1,
                             float b2, float eps, float wd, float bc1, float bc2, float grad_scale) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float gi = g[i] * grad_scale;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float pi = p[i] * (1.f - lr * wd);
    pi -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    p[i] = pi;
    if (out) out[i] = __float2bfloat16(pi);
  }
}

void adamw(float* p, const float* g, float* m, float* v, __nv_bfloat16* out, size_t n, float lr, float b1, float b2,
           float eps, float wd, int step, float grad_scale, cudaStream_t s) {
  if (n == 0) return;
  const float bc1 = 1.f - powf(b1, static_cast<float>(step));
  const float bc2 = 1.f - powf(b2, static_cast<float>(step));
  size_t blocks = (n + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  adamw_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(p, g, m, v, out, n, lr, b1, b2, eps, wd, bc1, bc2,
                                                             grad_scale);
}

// Sum of squares of an fp32 buffer, accumulated into out[0] (one atomic per block).
__global__ void sumsq_kernel(const float* __restrict__ x, size_t n, float* __restrict__ out) {
  float acc = 0.f;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    acc += x[i] * x[i];
  acc = warp_sum(acc);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 8) {
    float t = red[threadIdx.x];
    t += __shfl_xor_sync(0xffu, t, 4);
    t += __shfl_xor_sync(0xffu, t, 2);
    t += __shfl_xor_sync(0xffu, t, 1);
    if (threadIdx.x == 0) atomicAdd(out, t);
  }
}

void sumsq(const float* x, size_t n, float* out, cudaStream_t s) {
  if (n == 0) return;
  size_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  sumsq_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, n, out);
}

}  // namespace d3d
