// Memory-bound fused kernels of the decoder layer (sm_100a).
// Reference counterparts: serving/vendor/ssd/layers/layernorm.py:5-98 (add +
// RMSNorm), rotary_embedding.py:6-73, activation.py:6-14 (SiLU-mul), the
// head-wise QK-norm of serving/vendor/ssd/models/qwen3.py, and the greedy match of
// single/eval_async_packed.py:170-175.
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
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"

namespace d3d {

// ----------------------------------------------------------------- helpers
// Sum of the split-K partials of one element (or of 4 consecutive elements),
// in split order.  Every load is issued before the first addition, so a
// thread waits for one memory round trip whatever the split count.
constexpr int MAX_SPLITS = 16;

template <int S = MAX_SPLITS>
__device__ __forceinline__ float load_split_sum(const float* p, int nsplit, size_t stride, size_t off) {
  float v[S];
#pragma unroll
  for (int i = 0; i < S; ++i)
    if (i < nsplit) v[i] = __ldg(p + i * stride + off);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < S; ++i)
    if (i < nsplit) s += v[i];
  return s;
}

template <int S>
__device__ __forceinline__ float4 load_split_sum4(const float* p, int nsplit, size_t stride, size_t off) {
  float4 v[S];
#pragma unroll
  for (int i = 0; i < S; ++i)
    if (i < nsplit) v[i] = __ldg(reinterpret_cast<const float4*>(p + i * stride + off));
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < S; ++i)
    if (i < nsplit) {
      s.x += v[i].x;
      s.y += v[i].y;
      s.z += v[i].z;
      s.w += v[i].w;
    }
  return s;
}

__device__ __forceinline__ void ld_bf16x4(const __nv_bfloat16* p, float* f) {
  const uint2 raw = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) f[j] = __bfloat162float(b[j]);
}

__device__ __forceinline__ void st_bf16x4(__nv_bfloat16* p, const float* f) {
  __align__(8) __nv_bfloat16 b[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) b[j] = __float2bfloat16(f[j]);
  *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(b);
}

// ------------------------------------------------------- add + RMSNorm
// x = bf16(residual + bf16(sum_s P[s])) (or x = residual when P is null);
// residual <- x; out = w * bf16(x * rsqrt(mean(x^2) + eps)).
// One block per row, 4 consecutive elements per thread and vector.
template <int V, int S>
__global__ void __launch_bounds__(512) add_rmsnorm_kernel(const float* __restrict__ part, int nsplit, __nv_bfloat16* __restrict__ residual,
                                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int M, int N,
                                   float eps) {
  griddep_launch();
  griddep_wait();
  const int m = blockIdx.x;
  if (m >= M) return;
  __shared__ float red[32];
  float xv[V][4];
  float ss = 0.f;
  const size_t stride = static_cast<size_t>(M) * N;
  float4 ps[V];
  if (part) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int n = 4 * (threadIdx.x + i * blockDim.x);
      if (n < N) ps[i] = load_split_sum4<S>(part, nsplit, stride, static_cast<size_t>(m) * N + n);
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int n = 4 * (threadIdx.x + i * blockDim.x);
#pragma unroll
    for (int j = 0; j < 4; ++j) xv[i][j] = 0.f;
    if (n < N) {
      const size_t off = static_cast<size_t>(m) * N + n;
      ld_bf16x4(residual + off, xv[i]);
      if (part) {
        const float y[4] = {ps[i].x, ps[i].y, ps[i].z, ps[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[i][j] = bf16r(xv[i][j] + bf16r(y[j]));
        st_bf16x4(residual + off, xv[i]);
      }
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
  const float r = rsqrtf(red[0] / N + eps);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int n = 4 * (threadIdx.x + i * blockDim.x);
    if (n < N) {
      float wv[4], y[4];
      ld_bf16x4(w + n, wv);
#pragma unroll
      for (int j = 0; j < 4; ++j) y[j] = bf16r(xv[i][j] * r) * wv[j];
      st_bf16x4(out + static_cast<size_t>(m) * N + n, y);
    }
  }
}

// S: compile-time bound on the split count (registers for the in-flight loads)
#define D3D_SPLIT_DISPATCH(nsplit, CALL)                       \
  do {                                                         \
    if ((nsplit) <= 4) { constexpr int S = 4; CALL; }          \
    else if ((nsplit) <= 8) { constexpr int S = 8; CALL; }     \
    else { constexpr int S = MAX_SPLITS; CALL; }               \
  } while (0)

void add_rmsnorm(const float* part, int nsplit, __nv_bfloat16* residual, const __nv_bfloat16* w, __nv_bfloat16* out,
                 int M, int N, float eps, cudaStream_t st) {
  if (M == 0) return;
  if (N % 4) throw std::runtime_error("add_rmsnorm: hidden size must be a multiple of 4");
  if (nsplit > MAX_SPLITS) throw std::runtime_error("add_rmsnorm: too many splits");
  const int vec = N / 4;
  const int threads = vec >= 512 ? 512 : (vec + 31) / 32 * 32;
  const int v = (vec + threads - 1) / threads;
  const int ns = part ? nsplit : 1;
  if (v <= 1) D3D_SPLIT_DISPATCH(ns, launch_pdl(add_rmsnorm_kernel<1, S>, dim3(M), dim3(threads), 0, st, part, nsplit, residual, w, out, M, N, eps));
  else if (v <= 2) D3D_SPLIT_DISPATCH(ns, launch_pdl(add_rmsnorm_kernel<2, S>, dim3(M), dim3(threads), 0, st, part, nsplit, residual, w, out, M, N, eps));
  else if (v <= 4) D3D_SPLIT_DISPATCH(ns, launch_pdl(add_rmsnorm_kernel<4, S>, dim3(M), dim3(threads), 0, st, part, nsplit, residual, w, out, M, N, eps));
  else if (v <= 8) D3D_SPLIT_DISPATCH(ns, launch_pdl(add_rmsnorm_kernel<8, S>, dim3(M), dim3(threads), 0, st, part, nsplit, residual, w, out, M, N, eps));
  else throw std::runtime_error("add_rmsnorm: hidden size above 16384");
}

// ------------------------------------------------------------------ SwiGLU
// P[s][m][0:I] = gate, P[s][m][I:2I] = up  ->  h[m][i] = bf16(bf16(silu(g)) * u)
// With ``interleaved`` the columns come from the interleaved gate|up weight
// (ops.pack_gate_up): h[i] takes gate column 128t + 32w + l and up column
// 128t + 32w + 16 + l for i = 64t + 16w + l.  Four consecutive columns per
// thread (they stay consecutive under the interleave).
// RMSNorm row scale from per-tile sums of squares (tiles of 128 columns):
// r = rsqrt(sum_t rsq[t][m] / n + eps).  Every lane of the calling warp gets
// the same value; the summation order (lane-strided, then a butterfly) is
// fixed, so a row's scale does not depend on the other rows of the launch.
__device__ __forceinline__ float row_scale(const float* rsq, int tiles, int M, int m, int n, float eps) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
  for (int t = lane; t < tiles; t += 32) s += rsq[static_cast<size_t>(t) * M + m];
  s = warp_sum(s);
  return rsqrtf(s / n + eps);
}

template <int S>
__global__ void __launch_bounds__(256)
    swiglu_rowscale_kernel(const float* __restrict__ part, int nsplit, __nv_bfloat16* __restrict__ h, int M, int I,
                           const float* __restrict__ rsq, int rsq_tiles, int rsq_n, float eps) {
  griddep_launch();
  griddep_wait();
  const int m = blockIdx.y;
  const float r = row_scale(rsq, rsq_tiles, M, m, rsq_n, eps);
  const size_t stride = static_cast<size_t>(M) * 2 * I;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) * 4; i < I; i += gridDim.x * blockDim.x * 4) {
    const size_t gcol = static_cast<size_t>(i / 64) * 128 + ((i % 64) / 16) * 32 + (i % 16);
    const float4 g4 = load_split_sum4<S>(part, nsplit, stride, static_cast<size_t>(m) * 2 * I + gcol);
    const float4 u4 = load_split_sum4<S>(part, nsplit, stride, static_cast<size_t>(m) * 2 * I + gcol + 16);
    const float g[4] = {g4.x, g4.y, g4.z, g4.w}, u[4] = {u4.x, u4.y, u4.z, u4.w};
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gb = bf16r(g[j] * r);
      const float sl = bf16r(gb / (1.f + expf(-gb)));
      o[j] = sl * bf16r(u[j] * r);
    }
    st_bf16x4(h + static_cast<size_t>(m) * I + i, o);
  }
}

void swiglu_rowscale(const float* part, int nsplit, __nv_bfloat16* h, int M, int I, const float* rsq, int rsq_tiles,
                     int rsq_n, float eps, cudaStream_t st) {
  if (M == 0) return;
  if (I % 64) throw std::runtime_error("swiglu_rowscale: interleaved gate|up needs I % 64 == 0");
  if (nsplit > MAX_SPLITS) throw std::runtime_error("swiglu_rowscale: too many splits");
  const int bx = (I / 4 + 255) / 256;
  D3D_SPLIT_DISPATCH(nsplit, launch_pdl(swiglu_rowscale_kernel<S>, dim3(bx, M), dim3(256), 0, st, part, nsplit, h,
                                        M, I, rsq, rsq_tiles, rsq_n, eps));
}

// Split-K reduction into the residual with per-tile row sums of squares, one
// warp per (row, 128-column tile): the stand-alone form of the GEMM's
// in-kernel reduction (same per-element and per-tile order, so the results
// are bit-identical whichever of the two a forward uses).
__global__ void residual_split_reduce_kernel(const float* __restrict__ part, int nsplit, __nv_bfloat16* x, int M,
                                             int N, float* __restrict__ sumsq) {
  griddep_launch();
  griddep_wait();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int tiles = (N + 127) / 128;
  if (w >= tiles * M) return;
  split_reduce_row(part, nsplit, static_cast<size_t>(M) * N, N, x, N, sumsq, M, w % M, w / M, lane);
}

void residual_split_reduce(const float* part, int nsplit, __nv_bfloat16* x, int M, int N, float* sumsq,
                           cudaStream_t st) {
  if (M == 0) return;
  if (nsplit > MAX_SPLITS) throw std::runtime_error("residual_split_reduce: too many splits");
  const int warps = ((N + 127) / 128) * M;
  launch_pdl(residual_split_reduce_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0, st, part, nsplit, x, M, N,
             sumsq);
}

__global__ void tile_sumsq_kernel(const __nv_bfloat16* __restrict__ x, int M, int N, float* __restrict__ out) {
  griddep_launch();
  griddep_wait();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int tiles = (N + 127) / 128;
  if (w >= tiles * M) return;
  const int t = w / M, m = w % M;
  float s = 0.f;
  for (int j = 0; j < 4; ++j) {
    const int n = t * 128 + j * 32 + lane;
    if (n < N) {
      const float v = __bfloat162float(x[static_cast<size_t>(m) * N + n]);
      s += v * v;
    }
  }
  s = warp_sum(s);
  if (lane == 0) out[static_cast<size_t>(t) * M + m] = s;
}

void tile_sumsq(const __nv_bfloat16* x, int M, int N, float* out, cudaStream_t st) {
  if (M == 0) return;
  const int warps = ((N + 127) / 128) * M;
  launch_pdl(tile_sumsq_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0, st, x, M, N, out);
}

template <int S>
__global__ void __launch_bounds__(256, 2)
    swiglu_kernel(const float* __restrict__ part, int nsplit, __nv_bfloat16* __restrict__ h, int M, int I,
                  bool interleaved) {
  griddep_launch();
  griddep_wait();
  const int I4 = I / 4;
  const size_t total = static_cast<size_t>(M) * I4;
  const size_t stride = static_cast<size_t>(M) * 2 * I;
  for (size_t t = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t m = t / I4, i = (t % I4) * 4;
    const size_t gcol = interleaved ? (i / 64) * 128 + ((i % 64) / 16) * 32 + (i % 16) : i;
    const size_t ucol = interleaved ? gcol + 16 : i + I;
    const float4 g4 = load_split_sum4<S>(part, nsplit, stride, m * 2 * I + gcol);
    const float4 u4 = load_split_sum4<S>(part, nsplit, stride, m * 2 * I + ucol);
    const float g[4] = {g4.x, g4.y, g4.z, g4.w}, u[4] = {u4.x, u4.y, u4.z, u4.w};
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gb = bf16r(g[j]);
      const float sl = bf16r(gb / (1.f + expf(-gb)));
      o[j] = sl * bf16r(u[j]);
    }
    st_bf16x4(h + m * I + i, o);
  }
}

void swiglu(const float* part, int nsplit, __nv_bfloat16* h, int M, int I, bool interleaved, cudaStream_t st) {
  if (M == 0) return;
  if (I % 4) throw std::runtime_error("swiglu: intermediate size must be a multiple of 4");
  if (interleaved && I % 64) throw std::runtime_error("swiglu: interleaved gate|up needs I % 64 == 0");
  if (nsplit > MAX_SPLITS) throw std::runtime_error("swiglu: too many splits");
  const size_t total = static_cast<size_t>(M) * (I / 4);
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  D3D_SPLIT_DISPATCH(nsplit, launch_pdl(swiglu_kernel<S>, dim3(blocks), dim3(256), 0, st, part, nsplit, h, M, I, interleaved));
}

// ------------------------------------------- QK-norm + RoPE + paged KV write
// One warp per (token, head) for heads [0, Hq + 2*Hkv): q heads, k heads, v heads.
template <int E, int S>  // E: elements per lane = head_dim / 32; S: split bound
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
  const size_t off0 = static_cast<size_t>(m) * N + h * D + lane * E;
  // RMSNorm scale of the GEMM input row when its norm weight is folded into qkv
  const float rs = a.rsq ? row_scale(a.rsq, a.rsq_tiles, a.M, m, a.rsq_n, a.eps) : 1.f;
  if constexpr (E == 4) {
    if (a.part) {
      const float4 s4 = load_split_sum4<S>(a.part, a.nsplit, stride, off0);
      x[0] = bf16r(s4.x * rs);
      x[1] = bf16r(s4.y * rs);
      x[2] = bf16r(s4.z * rs);
      x[3] = bf16r(s4.w * rs);
    } else {
      ld_bf16x4(a.y + off0, x);
#pragma unroll
      for (int e = 0; e < E; ++e) x[e] = a.rsq ? bf16r(x[e] * rs) : x[e];
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e)
      x[e] = bf16r((a.part ? load_split_sum<S>(a.part, a.nsplit, stride, off0 + e) : __bfloat162float(a.y[off0 + e])) *
                   rs);
  }
  const int64_t slot = a.slots[m];
  if (h >= a.Hq && !D3D_IN_BOUNDS(slot, a.num_slots, a.status)) return;   // debug builds only
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
  if (a.part && a.nsplit > MAX_SPLITS) throw std::runtime_error("qkv_rope_kv: too many splits");
  const int ns = a.part ? a.nsplit : 1;
  switch (a.head_dim) {
    case 32: D3D_SPLIT_DISPATCH(ns, launch_pdl(qkv_rope_kv_kernel<1, S>, dim3(blocks), dim3(256), 0, st, a)); break;
    case 64: D3D_SPLIT_DISPATCH(ns, launch_pdl(qkv_rope_kv_kernel<2, S>, dim3(blocks), dim3(256), 0, st, a)); break;
    case 128: D3D_SPLIT_DISPATCH(ns, launch_pdl(qkv_rope_kv_kernel<4, S>, dim3(blocks), dim3(256), 0, st, a)); break;
    default: throw std::runtime_error("qkv_rope_kv: head_dim must be 32, 64 or 128");
  }
}

// --------------------------------------------------------------- embedding
// out[m] = table[ids[m]] (+ cond[m / q_len] where cond_rows[m])
__global__ void embed_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             const __nv_bfloat16* __restrict__ cond, const unsigned char* __restrict__ cond_rows,
                             int q_len, __nv_bfloat16* __restrict__ out, int M, int H, long long vocab, int* status) {
  griddep_launch();
  griddep_wait();
  const int m = blockIdx.x;
  int64_t id = ids[m];
  if (!D3D_IN_BOUNDS(id, vocab, status)) id = 0;   // debug builds only
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
           int q_len, __nv_bfloat16* out, int M, int H, cudaStream_t st, long long vocab, int* status) {
  if (M == 0) return;
  launch_pdl(embed_kernel, dim3(M), dim3(128), 0, st, ids, table, cond, cond_rows, q_len, out, M, H, vocab, status);
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
