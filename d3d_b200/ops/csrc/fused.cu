// Memory-bound fused kernels of the decoder layer (sm_100a).
//
// Each GEMM of the layer writes fp32 split-K partials; the kernel that consumes
// them reduces the splits in a fixed order and fuses what follows the matmul:
//
//   qkv partials  -> per-head QK-RMSNorm + rotate-half RoPE -> q out,
//                    k/v scattered into the paged KV cache          (qkv_rope_kv)
//   o / down      -> + residual (bf16 rounding like two bf16 ops)
//                    -> RMSNorm of the next sublayer               (add_rmsnorm)
//   gate|up       -> SiLU(gate) * up                              (swiglu)
//
// plus the embedding gather (with the optional drafter conditioning add), the
// LM-head top-k merge and greedy acceptance.  Rounding points mirror the
// Hugging Face Qwen3 module order (bf16 after every op) except RoPE, which is
// evaluated in fp32 and rounded once.
#include "common.cuh"
#include "kernels.h"

namespace d3d {

// ----------------------------------------------------------------- helpers
// Sum of the split-K partials of one element, in split order (loads issued
// four at a time; the additions stay in split order).
__device__ __forceinline__ float load_split_sum(const float* p, int nsplit, size_t stride, size_t off) {
  float s = 0.f;
  int i = 0;
  for (; i + 4 <= nsplit; i += 4) {
    const float a = __ldg(p + (i + 0) * stride + off), b = __ldg(p + (i + 1) * stride + off);
    const float c = __ldg(p + (i + 2) * stride + off), d = __ldg(p + (i + 3) * stride + off);
    s += a;
    s += b;
    s += c;
    s += d;
  }
  for (; i < nsplit; ++i) s += __ldg(p + i * stride + off);
  return s;
}

// ------------------------------------------------------- add + RMSNorm
// x = bf16(residual + bf16(sum_s P[s])) (or x = residual when P is null);
// residual <- x; out = w * bf16(x * rsqrt(mean(x^2) + eps)).
template <int VPT>
__global__ void add_rmsnorm_kernel(const float* __restrict__ part, int nsplit, __nv_bfloat16* __restrict__ residual,
                                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int M, int N,
                                   float eps) {
  griddep_launch();
  griddep_wait();
  const int m = blockIdx.x;
  if (m >= M) return;
  __shared__ float red[32];
  float xv[VPT];
  float ss = 0.f;
  const size_t stride = static_cast<size_t>(M) * N;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int n = threadIdx.x + i * blockDim.x;
    float x = 0.f;
    if (n < N) {
      const size_t off = static_cast<size_t>(m) * N + n;
      x = __bfloat162float(residual[off]);
      if (part) {
        const float y = bf16r(load_split_sum(part, nsplit, stride, off));
        x = bf16r(x + y);
        residual[off] = __float2bfloat16(x);
      }
    }
    xv[i] = x;
    ss += x * x;
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
  const float r = rsqrtf(red[0] / N + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int n = threadIdx.x + i * blockDim.x;
    if (n < N) {
      const float y = bf16r(xv[i] * r) * __bfloat162float(w[n]);
      out[static_cast<size_t>(m) * N + n] = __float2bfloat16(y);
    }
  }
}

void add_rmsnorm(const float* part, int nsplit, __nv_bfloat16* residual, const __nv_bfloat16* w, __nv_bfloat16* out,
                 int M, int N, float eps, cudaStream_t st) {
  if (M == 0) return;
  const int threads = N >= 4096 ? 1024 : (N >= 1024 ? 256 : 128);
  const int vpt = (N + threads - 1) / threads;
  if (vpt <= 2) launch_pdl(add_rmsnorm_kernel<2>, dim3(M), dim3(threads), 0, st, part, nsplit, residual, w, out, M, N, eps);
  else if (vpt <= 4) launch_pdl(add_rmsnorm_kernel<4>, dim3(M), dim3(threads), 0, st, part, nsplit, residual, w, out, M, N, eps);
  else if (vpt <= 8) launch_pdl(add_rmsnorm_kernel<8>, dim3(M), dim3(threads), 0, st, part, nsplit, residual, w, out, M, N, eps);
  else launch_pdl(add_rmsnorm_kernel<16>, dim3(M), dim3(threads), 0, st, part, nsplit, residual, w, out, M, N, eps);
}

// ------------------------------------------------------------------ SwiGLU
// P[s][m][0:I] = gate, P[s][m][I:2I] = up  ->  h[m][i] = bf16(bf16(silu(g)) * u)
__global__ void swiglu_kernel(const float* __restrict__ part, int nsplit, __nv_bfloat16* __restrict__ h, int M, int I) {
  griddep_launch();
  griddep_wait();
  const size_t total = static_cast<size_t>(M) * I;
  const size_t stride = static_cast<size_t>(M) * 2 * I;
  for (size_t t = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t m = t / I, i = t % I;
    const size_t off = m * 2 * I + i;
    const float g = bf16r(load_split_sum(part, nsplit, stride, off));
    const float u = bf16r(load_split_sum(part, nsplit, stride, off + I));
    const float s = bf16r(g / (1.f + expf(-g)));
    h[t] = __float2bfloat16(s * u);
  }
}

void swiglu(const float* part, int nsplit, __nv_bfloat16* h, int M, int I, cudaStream_t st) {
  if (M == 0) return;
  const size_t total = static_cast<size_t>(M) * I;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  launch_pdl(swiglu_kernel, dim3(blocks), dim3(256), 0, st, part, nsplit, h, M, I);
}

// ------------------------------------------- QK-norm + RoPE + paged KV write
// One warp per (token, head) for heads [0, Hq + 2*Hkv): q heads, k heads, v heads.
template <int E>  // elements per lane = head_dim / 32
__global__ void qkv_rope_kv_kernel(QkvRopeArgs a) {
  griddep_launch();
  griddep_wait();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int H = a.Hq + 2 * a.Hkv;
  if (gw >= a.M * H) return;
  const int m = gw / H, h = gw % H;
  constexpr int D = E * 32;
  const int N = H * D;
  const size_t stride = static_cast<size_t>(a.M) * N;
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const size_t off = static_cast<size_t>(m) * N + h * D + lane * E + e;
    x[e] = bf16r(a.part ? load_split_sum(a.part, a.nsplit, stride, off) : __bfloat162float(a.y[off]));
  }
  const int64_t slot = a.slots[m];
  if (h >= a.Hq + a.Hkv) {  // v head: straight to the cache
    const int hv = h - a.Hq - a.Hkv;
    __nv_bfloat16* dst = a.v_cache + (slot * a.Hkv + hv) * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = __float2bfloat16(x[e]);
    return;
  }
  const bool is_q = h < a.Hq;
  const __nv_bfloat16* nw = is_q ? a.q_norm : a.k_norm;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) ss += x[e] * x[e];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + a.eps);
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = bf16r(bf16r(x[e] * r) * __bfloat162float(nw[lane * E + e]));
  // rotate-half RoPE: element d pairs with d +- D/2, held by lane ^ 16
  const float pos = static_cast<float>(a.positions[m]);
  float y[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int d = lane * E + e;
    const int fi = d % (D / 2);
    const float ang = pos * a.inv_freq[fi];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const float rot = d < D / 2 ? -partner : partner;
    y[e] = x[e] * cs + rot * sn;
  }
  if (is_q) {
    __nv_bfloat16* dst = a.q_out + (static_cast<size_t>(m) * a.Hq + h) * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = __float2bfloat16(y[e]);
  } else {
    const int hk = h - a.Hq;
    __nv_bfloat16* dst = a.k_cache + (slot * a.Hkv + hk) * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = __float2bfloat16(y[e]);
  }
}

void qkv_rope_kv(const QkvRopeArgs& a, cudaStream_t st) {
  if (a.M == 0) return;
  const int warps = a.M * (a.Hq + 2 * a.Hkv);
  const int blocks = (warps * 32 + 255) / 256;
  switch (a.head_dim) {
    case 32: launch_pdl(qkv_rope_kv_kernel<1>, dim3(blocks), dim3(256), 0, st, a); break;
    case 64: launch_pdl(qkv_rope_kv_kernel<2>, dim3(blocks), dim3(256), 0, st, a); break;
    case 128: launch_pdl(qkv_rope_kv_kernel<4>, dim3(blocks), dim3(256), 0, st, a); break;
    default: break;
  }
}

// --------------------------------------------------------------- embedding
// out[m] = table[ids[m]] (+ cond[m / q_len] where cond_rows[m])
__global__ void embed_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             const __nv_bfloat16* __restrict__ cond, const unsigned char* __restrict__ cond_rows,
                             int q_len, __nv_bfloat16* __restrict__ out, int M, int H) {
  griddep_launch();
  griddep_wait();
  const int m = blockIdx.x;
  const int64_t id = ids[m];
  const bool add = cond != nullptr && cond_rows != nullptr && cond_rows[m];
  const int b = m / q_len;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(table + id * H + i);
    if (!add) {
      *reinterpret_cast<uint4*>(out + static_cast<size_t>(m) * H + i) = raw;
    } else {
      const __nv_bfloat16* t = reinterpret_cast<const __nv_bfloat16*>(&raw);
      __align__(16) __nv_bfloat16 o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        o[j] = __float2bfloat16(__bfloat162float(t[j]) + __bfloat162float(cond[static_cast<size_t>(b) * H + i + j]));
      *reinterpret_cast<uint4*>(out + static_cast<size_t>(m) * H + i) = *reinterpret_cast<uint4*>(o);
    }
  }
}

void embed(const int64_t* ids, const __nv_bfloat16* table, const __nv_bfloat16* cond, const unsigned char* cond_rows,
           int q_len, __nv_bfloat16* out, int M, int H, cudaStream_t st) {
  if (M == 0) return;
  launch_pdl(embed_kernel, dim3(M), dim3(128), 0, st, ids, table, cond, cond_rows, q_len, out, M, H);
}

// ---------------------------------------------------------- top-k merge
// tile partials [M][ntiles][kt] (desc, ties -> lower index) -> [M][k]
template <int KT>
__global__ void topk_merge_kernel(const float* __restrict__ tv, const int* __restrict__ ti, int ntiles, int k,
                                  float* __restrict__ ov, int64_t* __restrict__ oi, int M) {
  griddep_launch();
  griddep_wait();
  const int m = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (m >= M) return;
  float bv[KT];
  int bi[KT];
#pragma unroll
  for (int r = 0; r < KT; ++r) {
    bv[r] = -INFINITY;
    bi[r] = 0x7fffffff;
  }
  const size_t base = static_cast<size_t>(m) * ntiles * KT;
  for (int c = lane; c < ntiles * KT; c += 32) {
    float cv = tv[base + c];
    int ci = ti[base + c];
#pragma unroll
    for (int q = 0; q < KT; ++q) {
      if (cv > bv[q] || (cv == bv[q] && ci < bi[q])) {
        const float t1 = bv[q];
        const int t2 = bi[q];
        bv[q] = cv;
        bi[q] = ci;
        cv = t1;
        ci = t2;
      }
    }
  }
  // warp merge: k rounds of arg-max over the lanes' sorted heads
  int head = 0;
  for (int r = 0; r < k; ++r) {
    float v = head < KT ? bv[0] : -INFINITY;
    int i = head < KT ? bi[0] : 0x7fffffff;
    // the list is consumed from the front by shifting
    float best = v;
    int besti = i;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi2 = __shfl_xor_sync(0xffffffffu, besti, o);
      if (ov2 > best || (ov2 == best && oi2 < besti)) {
        best = ov2;
        besti = oi2;
      }
    }
    if (lane == 0) {
      if (ov) ov[static_cast<size_t>(m) * k + r] = best;
      oi[static_cast<size_t>(m) * k + r] = besti;
    }
    if (head < KT && bi[0] == besti && bv[0] == best) {
#pragma unroll
      for (int q = 0; q + 1 < KT; ++q) {
        bv[q] = bv[q + 1];
        bi[q] = bi[q + 1];
      }
      bv[KT - 1] = -INFINITY;
      bi[KT - 1] = 0x7fffffff;
      ++head;
    }
  }
}

void topk_merge(const float* tv, const int* ti, int ntiles, int kt, int k, float* ov, int64_t* oi, int M,
                cudaStream_t st) {
  if (M == 0) return;
  const int blocks = (M + 7) / 8;
  if (kt == 1) launch_pdl(topk_merge_kernel<1>, dim3(blocks), dim3(256), 0, st, tv, ti, ntiles, k, ov, oi, M);
  else if (kt == 2) launch_pdl(topk_merge_kernel<2>, dim3(blocks), dim3(256), 0, st, tv, ti, ntiles, k, ov, oi, M);
  else launch_pdl(topk_merge_kernel<4>, dim3(blocks), dim3(256), 0, st, tv, ti, ntiles, k, ov, oi, M);
}

// -------------------------------------------------------- greedy acceptance
// blocks [B][K] (anchor + drafts), posterior [B][K] (target argmax after each
// block token).  commit[b] = 1 + leading matches; corr[b] = posterior[commit-1];
// the hidden row that produced corr is copied to hid_out[b] (H bf16).
__global__ void greedy_accept_kernel(const int64_t* __restrict__ blocks, const int64_t* __restrict__ post, int K,
                                     int64_t* __restrict__ commit, int64_t* __restrict__ corr,
                                     const __nv_bfloat16* __restrict__ hidden, __nv_bfloat16* __restrict__ hid_out,
                                     int H) {
  griddep_launch();
  griddep_wait();
  const int b = blockIdx.x;
  __shared__ int s_commit;
  if (threadIdx.x == 0) {
    int n = 1;
    while (n < K && blocks[static_cast<size_t>(b) * K + n] == post[static_cast<size_t>(b) * K + n - 1]) ++n;
    s_commit = n;
    commit[b] = n;
    corr[b] = post[static_cast<size_t>(b) * K + n - 1];
  }
  __syncthreads();
  if (hidden && hid_out) {
    const size_t src = (static_cast<size_t>(b) * K + s_commit - 1) * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) hid_out[static_cast<size_t>(b) * H + i] = hidden[src + i];
  }
}

void greedy_accept(const int64_t* blocks, const int64_t* post, int B, int K, int64_t* commit, int64_t* corr,
                   const __nv_bfloat16* hidden, __nv_bfloat16* hid_out, int H, cudaStream_t st) {
  if (B == 0) return;
  launch_pdl(greedy_accept_kernel, dim3(B), dim3(128), 0, st, blocks, post, K, commit, corr, hidden, hid_out, H);
}

}  // namespace d3d
