// Paged-KV attention with structured masks (sm_100a).  Reference
// counterparts: serving/vendor/ssd/layers/attention.py:8-53 (FlashAttention-2
// and dense-mask SDPA calls) and the mask builders of single/eval_sync.py:194-275.
//
// One kernel serves every attention of the framework: target prefill and
// verify (causal over the block), drafter prefill (causal / block-causal),
// recovery drafting, and the packed all-outcome forward.  Each query row
// carries three int32 numbers (lim, lo, hi): it sees key slots
// ``k < lim  or  lo <= k < hi``.  Key tiles that no row of a CTA can see are
// skipped without being loaded, which is what makes the packed forward (one
// pending block + up to 46 branch segments) cheap: a branch row reads the
// prefix, the accepted pending tokens and its own 16-token segment only.
//
// Layout: a CTA owns 64 "packed rows" of one (sequence, kv head): row r is
// token r / g and query head h*g + r % g (g = GQA group), so K/V tiles are
// loaded once for the whole group.  Four warps each run 16 rows through
// mma.sync m16n8k16 (bf16 -> fp32) for S = QK^T and O += PV with an online
// exp2 softmax.  Keys are split into chunks of ``chunk`` slots at fixed
// absolute boundaries (grid z); a combine kernel merges the chunks in index
// order.  Because chunk boundaries, the tile order inside a chunk and the
// per-row arithmetic do not depend on how many queries share a launch, a
// row's output is bit-identical whether it is verified in a block of 16 or
// decoded alone — required for greedy token identity with AR decoding.
#include <atomic>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace d3d {

constexpr int AT_ROWS = 64;
constexpr int AT_KEYS = 64;
constexpr int AT_MAX_PAGES = 1024;  // chunk / page_size + 1 must fit

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ bool visible(int k, int lim, int lo, int hi) { return k < lim || (k >= lo && k < hi); }

template <int D>
__global__ void __launch_bounds__(128, 4) attn_kernel(const AttnArgs a) {
  // Row descriptors, kv_end and the block table are step inputs copied in
  // before the forward starts, so they are read before the grid dependency
  // resolves; q and the KV cache (written by earlier kernels) after it.
  griddep_launch();
  constexpr int LD = D + 8;  // padded smem row (bank-conflict-free ldmatrix)
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* Kb = Qs + AT_ROWS * LD;       // [AT_KEYS][LD]
  __nv_bfloat16* Vb = Kb + AT_KEYS * LD;       // [AT_KEYS][LD]
  __shared__ int s_rows[AT_ROWS][3];
  __shared__ int s_range[3];
  __shared__ int s_pages[AT_MAX_PAGES];   // page ids of this CTA's key chunk

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = a.Hq / a.Hkv;
  const int b = blockIdx.y / a.Hkv, h = blockIdx.y % a.Hkv;
  const int chunk_id = blockIdx.z;
  const int R0 = blockIdx.x * AT_ROWS;
  const int T = a.B * a.q_len;
  const int kv_end = a.kv_end[b];

  // ---- rows: descriptors, key range of this CTA
  if (tid < AT_ROWS) {
    const int R = R0 + tid;
    const int t = R / g;
    int lim = 0, lo = 0, hi = 0;
    if (t < a.q_len) {
      const int* rr = a.rows + static_cast<size_t>(b * a.q_len + t) * 3;
      lim = min(rr[0], kv_end);
      lo = rr[1];
      hi = min(rr[2], kv_end);
      if (hi <= lo) lo = hi = 0;
    }
    s_rows[tid][0] = lim;
    s_rows[tid][1] = lo;
    s_rows[tid][2] = hi;
  }
  if (tid == 0) {
    s_range[0] = 0;
    s_range[1] = 0x7fffffff;
    s_range[2] = 0;
  }
  __syncthreads();
  if (tid < AT_ROWS) {
    atomicMax(&s_range[0], s_rows[tid][0]);
    if (s_rows[tid][2] > s_rows[tid][1]) {
      atomicMin(&s_range[1], s_rows[tid][1]);
      atomicMax(&s_range[2], s_rows[tid][2]);
    }
  }
  // page ids of this CTA's key chunk (clamped to the block-table row)
  const int kbeg = chunk_id * a.chunk;
  const int* bt = a.block_table + static_cast<size_t>(b) * a.bt_stride;
  const int pg0 = kbeg / a.page_size;
  const int npg_all = min((a.chunk + a.page_size - 1) / a.page_size + 1, a.bt_stride - pg0);
  for (int i = tid; i < npg_all && i < AT_MAX_PAGES; i += 128) s_pages[i] = bt[pg0 + i];
  __syncthreads();
  const int max_lim = s_range[0], min_lo = s_range[1], max_hi = s_range[2];
  griddep_wait();

  // ---- Q tile (async, lands with the first K/V tile)
  for (int c = tid; c < AT_ROWS * (D / 8); c += 128) {
    const int r = c / (D / 8), dc = (c % (D / 8)) * 8;
    const int R = R0 + r;
    const int t = R / g;
    if (t < a.q_len) {
      const int qh = h * g + R % g;
      cp_async16(smem_u32(Qs + r * LD + dc), a.q + (static_cast<size_t>(b * a.q_len + t) * a.Hq + qh) * D + dc);
    } else {
      *reinterpret_cast<uint4*>(Qs + r * LD + dc) = make_uint4(0, 0, 0, 0);
    }
  }

  // per-thread rows of the mma fragments
  const int ra = warp * 16 + (lane >> 2), rb = ra + 8;
  const int limA = s_rows[ra][0], loA = s_rows[ra][1], hiA = s_rows[ra][2];
  const int limB = s_rows[rb][0], loB = s_rows[rb][1], hiB = s_rows[rb][2];

  // Q fragments are re-read from shared memory for every key tile (ldmatrix)
  // instead of being pinned in registers: that keeps the kernel at <= 128
  // registers, so four CTAs (16 warps) share an SM and hide mma latency.
  const uint32_t q_base = smem_u32(Qs + (warp * 16 + (lane & 15)) * LD + (lane >> 4) * 8);

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  const float sl2 = a.scale * 1.4426950408889634f;  // scale * log2(e)

  const int kend = min(kbeg + a.chunk, kv_end);

  auto needed = [&](int k0) { return k0 < max_lim || (k0 + AT_KEYS > min_lo && k0 < max_hi); };
  auto next_needed = [&](int k0) {
    while (k0 < kend && !needed(k0)) k0 += AT_KEYS;
    return k0;
  };
  // issue the async copy of one K/V tile into buffer `buf` (zeros beyond kv_end)
  auto load_tile = [&](int k0) {
    __nv_bfloat16* Ks = Kb;
    __nv_bfloat16* Vs = Vb;
    for (int c = tid; c < AT_KEYS * (D / 8); c += 128) {
      const int kr = c / (D / 8), dc = (c % (D / 8)) * 8;
      const int s = k0 + kr;
      const int64_t page = s < kv_end ? s_pages[s / a.page_size - pg0] : 0;
      const int64_t krow = page * a.page_size + s % a.page_size;
      if (s < kv_end && D3D_IN_BOUNDS(krow, a.num_slots, a.status)) {
        const size_t off = (krow * a.Hkv + h) * static_cast<size_t>(D) + dc;
        cp_async16(smem_u32(Ks + kr * LD + dc), a.k_cache + off);
        cp_async16(smem_u32(Vs + kr * LD + dc), a.v_cache + off);
      } else {
        *reinterpret_cast<uint4*>(Ks + kr * LD + dc) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(Vs + kr * LD + dc) = make_uint4(0, 0, 0, 0);
      }
    }
  };

  // One K/V tile buffer per CTA: latency is hidden by the other CTAs of the SM.
  int k0 = next_needed(kbeg);
  if (k0 >= kend) {
    cp_async_commit();
    cp_async_wait_all();
  }
  while (k0 < kend) {
    load_tile(k0);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    const __nv_bfloat16* Ks = Kb;
    const __nv_bfloat16* Vs = Vb;

    // ---- S = Q K^T (16 rows x 64 keys per warp)
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t qf[4];
      ldsm_x4(q_base + kk * 32, qf[0], qf[1], qf[2], qf[3]);
#pragma unroll
      for (int nb = 0; nb < 8; nb += 2) {
        const int key = nb * 8 + (lane & 7) + (lane >> 4) * 8;
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(Ks + key * LD + col), b0, b1, b2, b3);
        mma16816(s[nb], qf, b0, b1);
        mma16816(s[nb + 1], qf, b2, b3);
      }
    }
    // ---- mask + online softmax (per-element masking only when some row of
    // this warp sees part of the tile)
    float tmA = -INFINITY, tmB = -INFINITY;
    const int k1e = k0 + AT_KEYS;
    const bool fullA = k1e <= kend && (k1e <= limA || (k0 >= loA && k1e <= hiA));
    const bool fullB = k1e <= kend && (k1e <= limB || (k0 >= loB && k1e <= hiB));
    if (__all_sync(0xffffffffu, fullA && fullB)) {
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          s[nb][e] *= sl2;
          s[nb][2 + e] *= sl2;
          tmA = fmaxf(tmA, s[nb][e]);
          tmB = fmaxf(tmB, s[nb][2 + e]);
        }
      }
    } else {
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = k0 + nb * 8 + (lane & 3) * 2 + e;
          const bool inb = key < kend;
          s[nb][e] = (inb && visible(key, limA, loA, hiA)) ? s[nb][e] * sl2 : -INFINITY;
          s[nb][2 + e] = (inb && visible(key, limB, loB, hiB)) ? s[nb][2 + e] * sl2 : -INFINITY;
          tmA = fmaxf(tmA, s[nb][e]);
          tmB = fmaxf(tmB, s[nb][2 + e]);
        }
      }
    }
    tmA = fmaxf(tmA, __shfl_xor_sync(0xffffffffu, tmA, 1));
    tmA = fmaxf(tmA, __shfl_xor_sync(0xffffffffu, tmA, 2));
    tmB = fmaxf(tmB, __shfl_xor_sync(0xffffffffu, tmB, 1));
    tmB = fmaxf(tmB, __shfl_xor_sync(0xffffffffu, tmB, 2));
    const float nmA = fmaxf(mA, tmA), nmB = fmaxf(mB, tmB);
    const float alA = (nmA == -INFINITY) ? 1.f : exp2f(mA - nmA);
    const float alB = (nmB == -INFINITY) ? 1.f : exp2f(mB - nmB);
    float sumA = 0.f, sumB = 0.f;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float pa = s[nb][e] == -INFINITY ? 0.f : exp2f(s[nb][e] - nmA);
        const float pb = s[nb][2 + e] == -INFINITY ? 0.f : exp2f(s[nb][2 + e] - nmB);
        s[nb][e] = pa;
        s[nb][2 + e] = pb;
        sumA += pa;
        sumB += pb;
      }
    }
    sumA += __shfl_xor_sync(0xffffffffu, sumA, 1);
    sumA += __shfl_xor_sync(0xffffffffu, sumA, 2);
    sumB += __shfl_xor_sync(0xffffffffu, sumB, 1);
    sumB += __shfl_xor_sync(0xffffffffu, sumB, 2);
    lA = lA * alA + sumA;
    lB = lB * alB + sumB;
    mA = nmA;
    mB = nmB;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alA;
      o[i][1] *= alA;
      o[i][2] *= alB;
      o[i][3] *= alB;
    }
    // ---- O += P V
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kb][0], s[2 * kb][1]);
      pa[1] = pack_bf16(s[2 * kb][2], s[2 * kb][3]);
      pa[2] = pack_bf16(s[2 * kb + 1][0], s[2 * kb + 1][1]);
      pa[3] = pack_bf16(s[2 * kb + 1][2], s[2 * kb + 1][3]);
#pragma unroll
      for (int nd = 0; nd < D / 8; nd += 2) {
        const int key = kb * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = nd * 8 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(Vs + key * LD + col), b0, b1, b2, b3);
        mma16816(o[nd], pa, b0, b1);
        mma16816(o[nd + 1], pa, b2, b3);
      }
    }
    __syncthreads();
    k0 = next_needed(k0 + AT_KEYS);
  }

  // ---- write partial (or final) results
  const int RA = R0 + ra, RB = R0 + rb;
  const int tA = RA / g, tB = RB / g;
  const int qhA = h * g + RA % g, qhB = h * g + RB % g;
  const bool vA = tA < a.q_len, vB = tB < a.q_len;
  const size_t tokA = static_cast<size_t>(b * a.q_len + tA), tokB = static_cast<size_t>(b * a.q_len + tB);
  if (a.n_chunks == 1) {
    const float iA = lA > 0.f ? 1.f / lA : 0.f, iB = lB > 0.f ? 1.f / lB : 0.f;
#pragma unroll
    for (int nd = 0; nd < D / 8; ++nd) {
      const int d = nd * 8 + (lane & 3) * 2;
      if (vA)
        *reinterpret_cast<__nv_bfloat162*>(a.out + (tokA * a.Hq + qhA) * D + d) =
            __floats2bfloat162_rn(o[nd][0] * iA, o[nd][1] * iA);
      if (vB)
        *reinterpret_cast<__nv_bfloat162*>(a.out + (tokB * a.Hq + qhB) * D + d) =
            __floats2bfloat162_rn(o[nd][2] * iB, o[nd][3] * iB);
    }
  } else {
    const size_t cbase = static_cast<size_t>(chunk_id) * T * a.Hq;
#pragma unroll
    for (int nd = 0; nd < D / 8; ++nd) {
      const int d = nd * 8 + (lane & 3) * 2;
      if (vA)
        *reinterpret_cast<float2*>(a.part_o + (cbase + tokA * a.Hq + qhA) * D + d) = make_float2(o[nd][0], o[nd][1]);
      if (vB)
        *reinterpret_cast<float2*>(a.part_o + (cbase + tokB * a.Hq + qhB) * D + d) = make_float2(o[nd][2], o[nd][3]);
    }
    if ((lane & 3) == 0) {
      if (vA) *reinterpret_cast<float2*>(a.part_ml + (cbase + tokA * a.Hq + qhA) * 2) = make_float2(mA, lA);
      if (vB) *reinterpret_cast<float2*>(a.part_ml + (cbase + tokB * a.Hq + qhB) * 2) = make_float2(mB, lB);
    }
  }
}

// Merge key chunks: O = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c.  The
// order of every sum is fixed by the chunk index (lane-strided, then a
// butterfly), and chunks without visible keys contribute exact zeros, so the
// result does not depend on how many (empty) chunks a launch had.
constexpr int MAX_CHUNKS = 512;
template <int D>
__global__ void attn_combine_kernel(const AttnArgs a) {
  griddep_launch();
  griddep_wait();
  __shared__ float wts[8][MAX_CHUNKS];
  const int T = a.B * a.q_len;
  const int wl = threadIdx.x >> 5;
  const int w = blockIdx.x * 8 + wl;
  const int lane = threadIdx.x & 31;
  if (w >= T * a.Hq) return;
  const int tok = w / a.Hq, qh = w % a.Hq;
  const int b = tok / a.q_len;
  const int nc = min(min(a.n_chunks, MAX_CHUNKS), (a.kv_end[b] + a.chunk - 1) / a.chunk);
  float M = -INFINITY;
  for (int c = lane; c < nc; c += 32)
    M = fmaxf(M, a.part_ml[((static_cast<size_t>(c) * T + tok) * a.Hq + qh) * 2]);
  M = warp_max(M);
  float L = 0.f;
  for (int c = lane; c < nc; c += 32) {
    const size_t idx = (static_cast<size_t>(c) * T + tok) * a.Hq + qh;
    const float mc = a.part_ml[idx * 2];
    const float f = (mc == -INFINITY || M == -INFINITY) ? 0.f : exp2f(mc - M);
    wts[wl][c] = f;
    L += a.part_ml[idx * 2 + 1] * f;
  }
  L = warp_sum(L);
  __syncwarp();
  constexpr int E = D / 32;
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
#pragma unroll 4
  for (int c = 0; c < nc; ++c) {
    const float f = wts[wl][c];
    const float* src = a.part_o + ((static_cast<size_t>(c) * T + tok) * a.Hq + qh) * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] += src[e] * f;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e)
    a.out[(static_cast<size_t>(tok) * a.Hq + qh) * D + lane * E + e] = __float2bfloat16(acc[e] * inv);
}

template <int D>
constexpr size_t attn_split_smem() {
  return static_cast<size_t>(AT_ROWS + 2 * AT_KEYS) * (D + 8) * 2;
}

// The dynamic shared-memory limit is a per-device property of a kernel: it
// is raised once on every device (bit ``dev`` of a per-kernel atomic mask;
// two threads racing on the first call both set the same value).
template <int D>
static cudaError_t ensure_attn_split_attr() {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(attn_split_smem<D>()));
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

template <int D>
static cudaError_t launch_attn_split(const AttnArgs& a, cudaStream_t st) {
  cudaError_t e = ensure_attn_split_attr<D>();
  if (e != cudaSuccess) return e;
  const int g = a.Hq / a.Hkv;
  dim3 grid((a.q_len * g + AT_ROWS - 1) / AT_ROWS, a.B * a.Hkv, a.n_chunks);
  e = launch_pdl(attn_kernel<D>, grid, dim3(128), attn_split_smem<D>(), st, a);
  if (e != cudaSuccess || a.n_chunks <= 1) return e;
  const int warps = a.B * a.q_len * a.Hq;
  return launch_pdl(attn_combine_kernel<D>, dim3((warps + 7) / 8), dim3(256), 0, st, a);
}

cudaError_t attention_combine(const AttnArgs& a, cudaStream_t st) {
  if (a.n_chunks <= 1) return cudaSuccess;
  if (a.n_chunks > MAX_CHUNKS) return cudaErrorInvalidValue;
  const int warps = a.B * a.q_len * a.Hq;
  const dim3 grid((warps + 7) / 8);
  switch (a.head_dim) {
    case 32: return launch_pdl(attn_combine_kernel<32>, grid, dim3(256), 0, st, a);
    case 64: return launch_pdl(attn_combine_kernel<64>, grid, dim3(256), 0, st, a);
    case 128: return launch_pdl(attn_combine_kernel<128>, grid, dim3(256), 0, st, a);
    default: return cudaErrorInvalidValue;
  }
}

// Split-KV attention with fp32 partials and a combine kernel.  Returns the
// status of its own launches (not a sticky error of earlier, unrelated work).
cudaError_t attention_split(const AttnArgs& a, cudaStream_t st) {
  if (a.B == 0 || a.q_len == 0) return cudaSuccess;
  if (a.n_chunks > MAX_CHUNKS) return cudaErrorInvalidValue;
  switch (a.head_dim) {
    case 32: return launch_attn_split<32>(a, st);
    case 64: return launch_attn_split<64>(a, st);
    case 128: return launch_attn_split<128>(a, st);
    default: return cudaErrorInvalidValue;
  }
}


// ===========================================================================
// Cluster attention (the default path).
//
// A thread-block cluster of CL = 8 CTAs owns one (row tile, sequence, kv
// head).  Keys are cut into chunks of 64 slots at fixed absolute boundaries;
// chunk c belongs to the CTA of cluster rank c % CL, which runs its chunks in
// increasing order through the same mma.sync online softmax as above, with
// an NT-deep ring of cp.async K/V tiles so several tiles are in flight.  The
// CTAs then merge their (m, l, O) states through distributed shared memory:
// rank r combines rows 8r..8r+7 over ranks 0..7 in rank order and writes the
// bf16 output.  No fp32 partials reach HBM and there is no second launch.
// Every reduction order is a function of absolute key positions only, so a
// row's output is the same whatever else shares the launch (batch
// invariance), as with the split path.
// ===========================================================================
constexpr int CL = 8;
constexpr int CL_MAX_PAGES = 1024;   // page ids of one CTA's chunks

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Remote shared-memory loads.  No "memory" clobber: they read state published
// before the cluster barrier, and without it the compiler issues all of them
// before the first use, so a thread waits for one round trip, not one per load.
__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ float2 ld_dsmem2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int D, int NT>
__global__ void __launch_bounds__(128, 1) attn_cluster_kernel(const AttnArgs a) {
  griddep_launch();
  constexpr int LD = D + 8;
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* ring = Qs + AT_ROWS * LD;  // NT x {K [64][LD], V [64][LD]}
  // after the key loop the ring holds this CTA's state: O [64][D], m [64], l [64] (fp32)
  float* red_o = reinterpret_cast<float*>(ring);
  float* red_m = red_o + AT_ROWS * D;
  float* red_l = red_m + AT_ROWS;
  __shared__ int s_rows[AT_ROWS][3];
  __shared__ int s_range[3];
  __shared__ int s_pages[CL_MAX_PAGES];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = a.Hq / a.Hkv;
  const int b = blockIdx.y / a.Hkv, h = blockIdx.y % a.Hkv;
  const int rank = static_cast<int>(cluster_rank());
  const int R0 = blockIdx.x * AT_ROWS;
  const int kv_end = a.kv_end[b];

  // ---- rows: descriptors and the union of their key ranges
  if (tid < AT_ROWS) {
    const int R = R0 + tid;
    const int t = R / g;
    int lim = 0, lo = 0, hi = 0;
    if (t < a.q_len) {
      const int* rr = a.rows + static_cast<size_t>(b * a.q_len + t) * 3;
      lim = min(rr[0], kv_end);
      lo = rr[1];
      hi = min(rr[2], kv_end);
      if (hi <= lo) lo = hi = 0;
    }
    s_rows[tid][0] = lim;
    s_rows[tid][1] = lo;
    s_rows[tid][2] = hi;
  }
  if (tid == 0) {
    s_range[0] = 0;
    s_range[1] = 0x7fffffff;
    s_range[2] = 0;
  }
  __syncthreads();
  if (tid < AT_ROWS) {
    atomicMax(&s_range[0], s_rows[tid][0]);
    if (s_rows[tid][2] > s_rows[tid][1]) {
      atomicMin(&s_range[1], s_rows[tid][1]);
      atomicMax(&s_range[2], s_rows[tid][2]);
    }
  }
  // ---- page ids of this CTA's chunks (chunk c = rank + CL * i, 64 / page_size pages each)
  const int ppc = AT_KEYS / a.page_size;
  const int nch = (kv_end + AT_KEYS - 1) / AT_KEYS;
  int nmy = nch > rank ? (nch - rank + CL - 1) / CL : 0;
  if (nmy * ppc > CL_MAX_PAGES) nmy = CL_MAX_PAGES / ppc;  // host rejects contexts this long
  const int* bt = a.block_table + static_cast<size_t>(b) * a.bt_stride;
  for (int idx = tid; idx < nmy * ppc; idx += 128) {
    const int pg = (rank + CL * (idx / ppc)) * ppc + idx % ppc;
    s_pages[idx] = pg < a.bt_stride ? bt[pg] : 0;
  }
  __syncthreads();
  const int max_lim = s_range[0], min_lo = s_range[1], max_hi = s_range[2];
  griddep_wait();

  // ---- Q tile (its own cp.async group, ahead of the K/V tiles)
  for (int c = tid; c < AT_ROWS * (D / 8); c += 128) {
    const int r = c / (D / 8), dc = (c % (D / 8)) * 8;
    const int R = R0 + r;
    const int t = R / g;
    if (t < a.q_len) {
      const int qh = h * g + R % g;
      cp_async16(smem_u32(Qs + r * LD + dc), a.q + (static_cast<size_t>(b * a.q_len + t) * a.Hq + qh) * D + dc);
    } else {
      *reinterpret_cast<uint4*>(Qs + r * LD + dc) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_commit();

  const int ra = warp * 16 + (lane >> 2), rb = ra + 8;
  const int limA = s_rows[ra][0], loA = s_rows[ra][1], hiA = s_rows[ra][2];
  const int limB = s_rows[rb][0], loB = s_rows[rb][1], hiB = s_rows[rb][2];
  const uint32_t q_base = smem_u32(Qs + (warp * 16 + (lane & 15)) * LD + (lane >> 4) * 8);

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  const float sl2 = a.scale * 1.4426950408889634f;  // scale * log2(e)

  auto k0_of = [&](int i) { return (rank + CL * i) * AT_KEYS; };
  auto needed = [&](int k0) { return k0 < max_lim || (k0 + AT_KEYS > min_lo && k0 < max_hi); };
  auto next_needed = [&](int i) {
    while (i < nmy && !needed(k0_of(i))) ++i;
    return i;
  };
  auto load_tile = [&](int i, int buf) {
    __nv_bfloat16* Ks = ring + buf * 2 * AT_KEYS * LD;
    __nv_bfloat16* Vs = Ks + AT_KEYS * LD;
    const int k0 = k0_of(i);
    for (int c = tid; c < AT_KEYS * (D / 8); c += 128) {
      const int kr = c / (D / 8), dc = (c % (D / 8)) * 8;
      const int s = k0 + kr;
      const int64_t page = s < kv_end ? s_pages[i * ppc + kr / a.page_size] : 0;
      const int64_t krow = page * a.page_size + s % a.page_size;
      if (s < kv_end && D3D_IN_BOUNDS(krow, a.num_slots, a.status)) {
        const size_t off = (krow * a.Hkv + h) * static_cast<size_t>(D) + dc;
        cp_async16(smem_u32(Ks + kr * LD + dc), a.k_cache + off);
        cp_async16(smem_u32(Vs + kr * LD + dc), a.v_cache + off);
      } else {
        *reinterpret_cast<uint4*>(Ks + kr * LD + dc) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(Vs + kr * LD + dc) = make_uint4(0, 0, 0, 0);
      }
    }
  };

  int cons = next_needed(0), iss = cons;
#pragma unroll
  for (int p = 0; p < NT; ++p) {
    if (iss < nmy) {
      load_tile(iss, p);
      iss = next_needed(iss + 1);
    }
    cp_async_commit();
  }
  for (int j = 0; cons < nmy; ++j) {
    cp_async_wait<NT - 1>();  // Q and tile j have landed
    __syncthreads();
    const __nv_bfloat16* Ks = ring + (j % NT) * 2 * AT_KEYS * LD;
    const __nv_bfloat16* Vs = Ks + AT_KEYS * LD;
    const int k0 = k0_of(cons);
    const int kend = min(k0 + AT_KEYS, kv_end);

    // ---- S = Q K^T (16 rows x 64 keys per warp)
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t qf[4];
      ldsm_x4(q_base + kk * 32, qf[0], qf[1], qf[2], qf[3]);
#pragma unroll
      for (int nb = 0; nb < 8; nb += 2) {
        const int key = nb * 8 + (lane & 7) + (lane >> 4) * 8;
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(Ks + key * LD + col), b0, b1, b2, b3);
        mma16816(s[nb], qf, b0, b1);
        mma16816(s[nb + 1], qf, b2, b3);
      }
    }
    // ---- mask + online softmax
    float tmA = -INFINITY, tmB = -INFINITY;
    const int k1e = k0 + AT_KEYS;
    const bool fullA = k1e <= kend && (k1e <= limA || (k0 >= loA && k1e <= hiA));
    const bool fullB = k1e <= kend && (k1e <= limB || (k0 >= loB && k1e <= hiB));
    if (__all_sync(0xffffffffu, fullA && fullB)) {
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          s[nb][e] *= sl2;
          s[nb][2 + e] *= sl2;
          tmA = fmaxf(tmA, s[nb][e]);
          tmB = fmaxf(tmB, s[nb][2 + e]);
        }
      }
    } else {
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = k0 + nb * 8 + (lane & 3) * 2 + e;
          const bool inb = key < kend;
          s[nb][e] = (inb && visible(key, limA, loA, hiA)) ? s[nb][e] * sl2 : -INFINITY;
          s[nb][2 + e] = (inb && visible(key, limB, loB, hiB)) ? s[nb][2 + e] * sl2 : -INFINITY;
          tmA = fmaxf(tmA, s[nb][e]);
          tmB = fmaxf(tmB, s[nb][2 + e]);
        }
      }
    }
    tmA = fmaxf(tmA, __shfl_xor_sync(0xffffffffu, tmA, 1));
    tmA = fmaxf(tmA, __shfl_xor_sync(0xffffffffu, tmA, 2));
    tmB = fmaxf(tmB, __shfl_xor_sync(0xffffffffu, tmB, 1));
    tmB = fmaxf(tmB, __shfl_xor_sync(0xffffffffu, tmB, 2));
    const float nmA = fmaxf(mA, tmA), nmB = fmaxf(mB, tmB);
    const float alA = (nmA == -INFINITY) ? 1.f : exp2f(mA - nmA);
    const float alB = (nmB == -INFINITY) ? 1.f : exp2f(mB - nmB);
    float sumA = 0.f, sumB = 0.f;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float pa = s[nb][e] == -INFINITY ? 0.f : exp2f(s[nb][e] - nmA);
        const float pb = s[nb][2 + e] == -INFINITY ? 0.f : exp2f(s[nb][2 + e] - nmB);
        s[nb][e] = pa;
        s[nb][2 + e] = pb;
        sumA += pa;
        sumB += pb;
      }
    }
    sumA += __shfl_xor_sync(0xffffffffu, sumA, 1);
    sumA += __shfl_xor_sync(0xffffffffu, sumA, 2);
    sumB += __shfl_xor_sync(0xffffffffu, sumB, 1);
    sumB += __shfl_xor_sync(0xffffffffu, sumB, 2);
    lA = lA * alA + sumA;
    lB = lB * alB + sumB;
    mA = nmA;
    mB = nmB;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alA;
      o[i][1] *= alA;
      o[i][2] *= alB;
      o[i][3] *= alB;
    }
    // ---- O += P V
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kb][0], s[2 * kb][1]);
      pa[1] = pack_bf16(s[2 * kb][2], s[2 * kb][3]);
      pa[2] = pack_bf16(s[2 * kb + 1][0], s[2 * kb + 1][1]);
      pa[3] = pack_bf16(s[2 * kb + 1][2], s[2 * kb + 1][3]);
#pragma unroll
      for (int nd = 0; nd < D / 8; nd += 2) {
        const int key = kb * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = nd * 8 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(Vs + key * LD + col), b0, b1, b2, b3);
        mma16816(o[nd], pa, b0, b1);
        mma16816(o[nd + 1], pa, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with buffer j % NT
    if (iss < nmy) {
      load_tile(iss, j % NT);
      iss = next_needed(iss + 1);
    }
    cp_async_commit();
    cons = next_needed(cons + 1);
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- this CTA's state -> shared memory (overwrites the ring)
#pragma unroll
  for (int nd = 0; nd < D / 8; ++nd) {
    const int d = nd * 8 + (lane & 3) * 2;
    *reinterpret_cast<float2*>(red_o + ra * D + d) = make_float2(o[nd][0], o[nd][1]);
    *reinterpret_cast<float2*>(red_o + rb * D + d) = make_float2(o[nd][2], o[nd][3]);
  }
  if ((lane & 3) == 0) {
    red_m[ra] = mA;
    red_l[ra] = lA;
    red_m[rb] = mB;
    red_l[rb] = lB;
  }
  cluster_sync_all();

  // ---- merge: rank r finalises rows 8r .. 8r+7 over ranks 0..CL-1, in rank order
  {
    constexpr int RPR = AT_ROWS / CL;   // rows per rank
    constexpr int TPR = 128 / RPR;      // threads per row
    constexpr int DPT = D / TPR;        // dims per thread (even)
    const int row = rank * RPR + tid / TPR;
    const int d0 = (tid % TPR) * DPT;
    // every remote load of this thread is issued before any of them is used
    float mj[CL], lj[CL];
    float2 ov[CL][DPT / 2];
#pragma unroll
    for (int j = 0; j < CL; ++j) {
      mj[j] = ld_dsmem(dsmem_addr(red_m + row, j));
      lj[j] = ld_dsmem(dsmem_addr(red_l + row, j));
      const uint32_t base = dsmem_addr(red_o + row * D + d0, j);
#pragma unroll
      for (int e = 0; e < DPT / 2; ++e) ov[j][e] = ld_dsmem2(base + e * 8);
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < CL; ++j) M = fmaxf(M, mj[j]);
    float L = 0.f;
    float wj[CL];
#pragma unroll
    for (int j = 0; j < CL; ++j) {
      wj[j] = (mj[j] == -INFINITY) ? 0.f : exp2f(mj[j] - M);
      L += wj[j] * lj[j];
    }
    float acc[DPT];
#pragma unroll
    for (int e = 0; e < DPT; ++e) acc[e] = 0.f;
#pragma unroll
    for (int j = 0; j < CL; ++j) {
#pragma unroll
      for (int e = 0; e < DPT / 2; ++e) {
        acc[2 * e] += wj[j] * ov[j][e].x;
        acc[2 * e + 1] += wj[j] * ov[j][e].y;
      }
    }
    const int R = R0 + row;
    const int t = R / g;
    if (t < a.q_len) {
      const int qh = h * g + R % g;
      const float inv = L > 0.f ? 1.f / L : 0.f;
      __nv_bfloat16* dst = a.out + (static_cast<size_t>(b * a.q_len + t) * a.Hq + qh) * D + d0;
#pragma unroll
      for (int e = 0; e < DPT; e += 2)
        *reinterpret_cast<__nv_bfloat162*>(dst + e) = __floats2bfloat162_rn(acc[e] * inv, acc[e + 1] * inv);
    }
  }
  cluster_sync_all();  // no CTA leaves while another still reads its shared memory
}

template <int D, int NT>
static void launch_attn_cluster(const AttnArgs& a, cudaStream_t st) {
  constexpr int LD = D + 8;
  const size_t smem = static_cast<size_t>(AT_ROWS + NT * 2 * AT_KEYS) * LD * 2;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attn_cluster_kernel<D, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    attr = true;
  }
  const int g = a.Hq / a.Hkv;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.q_len * g + AT_ROWS - 1) / AT_ROWS, a.B * a.Hkv, CL);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr2[2];
  attr2[0].id = cudaLaunchAttributeClusterDimension;
  attr2[0].val.clusterDim.x = 1;
  attr2[0].val.clusterDim.y = 1;
  attr2[0].val.clusterDim.z = CL;
  attr2[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr2[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr2;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, attn_cluster_kernel<D, NT>, a);
}

template <int D>
static void launch_attn_cluster_nt(const AttnArgs& a, cudaStream_t st) {
  // few clusters: one 160 KB CTA per SM with four tiles in flight; many
  // clusters: two CTAs per SM with two tiles each
  // D3D_ATTN_NT=2|4 overrides (the 87 KB two-tile CTA leaves room for a
  // GEMM CTA on the same SM to prefetch weights under programmatic launch)
  static const int nt_env = [] {
    const char* e = std::getenv("D3D_ATTN_NT");
    return e ? std::atoi(e) : 0;
  }();
  const long clusters = static_cast<long>((a.q_len * (a.Hq / a.Hkv) + AT_ROWS - 1) / AT_ROWS) * a.B * a.Hkv;
  const int nt = nt_env == 2 || nt_env == 4 ? nt_env : (clusters <= 16 ? 4 : 2);
  if (nt == 4) launch_attn_cluster<D, 4>(a, st);
  else launch_attn_cluster<D, 2>(a, st);
}

// Dispatch: batch-invariant callers (``invariant``: the target, whose verify
// and AR forwards must agree bit for bit) and decode-shaped launches (one
// 64-row tile per sequence and kv head) take the cluster kernel; larger
// query counts of other callers (the drafter's packed forward) take the
// split-KV kernels, whose CTAs run independently (no cluster barrier to wait
// at when the rows of a tile need uneven numbers of key tiles) when partial
// buffers are given.
void attention(const AttnArgs& a, cudaStream_t st) {
  if (a.B == 0 || a.q_len == 0) return;
  // the tcgen05/TMEM kernel serves every shape it supports (head_dim 64/128,
  // GQA group dividing 128, whole-tile pages); the mma.sync kernels below
  // remain for the others (e.g. head_dim 32 test models)
  if (attention_tc_supported(a)) {
    attention_tc(a, st);
    return;
  }
  static const bool force_split = [] {
    const char* e = std::getenv("D3D_ATTN_PATH");
    return e && std::string(e) == "split";
  }();
  const bool one_tile = a.q_len * (a.Hq / a.Hkv) <= AT_ROWS;
  if ((force_split || (!one_tile && !a.invariant)) && (a.n_chunks == 1 || (a.part_o && a.part_ml))) {
    const cudaError_t e = attention_split(a, st);
    if (e != cudaSuccess) throw std::runtime_error(std::string("attention (split-KV): ") + cudaGetErrorString(e));
    return;
  }
  if (AT_KEYS % a.page_size != 0) throw std::runtime_error("attention: page size must divide 64");
  // the CTA of rank 0 holds every 8th chunk: its page ids must fit CL_MAX_PAGES
  const long max_chunks = (static_cast<long>(a.bt_stride) * a.page_size + AT_KEYS - 1) / AT_KEYS;
  if ((max_chunks + CL - 1) / CL * (AT_KEYS / a.page_size) > CL_MAX_PAGES)
    throw std::runtime_error("attention: context too long for the cluster path");
  switch (a.head_dim) {
    case 32: launch_attn_cluster_nt<32>(a, st); break;
    case 64: launch_attn_cluster_nt<64>(a, st); break;
    case 128: launch_attn_cluster_nt<128>(a, st); break;
    default: throw std::runtime_error("attention: head_dim must be 32, 64 or 128");
  }
}
}  // namespace d3d

// ---------------------------------------------------------------------------
// Allocation-free C entry point (declared and documented in
// attention_noalloc.h; no counterpart in the reference).  It launches the
// split-KV kernels (attention_split) with their fp32 partials placed in a
// file-scope device array instead of caller- or allocator-provided memory.
// ---------------------------------------------------------------------------
#include <mutex>

#include "attention_noalloc.h"

static_assert(D3D_ATTN_NOALLOC_MAX_CHUNKS == d3d::MAX_CHUNKS, "combine kernel chunk limit");

namespace {

static __device__ __align__(256) unsigned char g_attn_scratch[D3D_ATTN_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_attn_scratch on the current device, looked up once per
// device (host code only sees a host-side stand-in for the symbol).  The
// kernels' shared-memory limit is raised per device by the launch path.
cudaError_t scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || p == nullptr) return e != cudaSuccess ? e : cudaErrorInvalidSymbol;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int d3d_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, long long num_slots,
                                     const int* block_table, int bt_stride, const int* rows, const int* kv_end, int B,
                                     int q_len, int Hq, int Hkv, int head_dim, int page_size, float scale, int chunk,
                                     int n_chunks, void* out, cudaStream_t stream) {
  if (!q || !k_cache || !v_cache || !block_table || !rows || !kv_end || !out) return D3D_NOALLOC_ERR_BAD_ARG;
  if (B <= 0 || q_len <= 0 || Hkv <= 0 || Hq % Hkv != 0 || bt_stride <= 0 || num_slots <= 0)
    return D3D_NOALLOC_ERR_BAD_ARG;
  if (head_dim != 32 && head_dim != 64 && head_dim != 128) return D3D_NOALLOC_ERR_BAD_ARG;
  // a 64-key tile spans whole pages, and a chunk spans whole tiles
  if (page_size <= 0 || d3d::AT_KEYS % page_size != 0) return D3D_NOALLOC_ERR_BAD_ARG;
  if (chunk <= 0 || chunk % d3d::AT_KEYS != 0 || chunk % page_size != 0 ||
      chunk / page_size + 1 > d3d::AT_MAX_PAGES)
    return D3D_NOALLOC_ERR_BAD_ARG;
  // the combine kernel merges at most D3D_ATTN_NOALLOC_MAX_CHUNKS chunks
  if (n_chunks < 1 || n_chunks > D3D_ATTN_NOALLOC_MAX_CHUNKS) return D3D_NOALLOC_ERR_BAD_ARG;
  const size_t T = static_cast<size_t>(B) * q_len;
  const size_t part_o = n_chunks > 1 ? static_cast<size_t>(n_chunks) * T * Hq * head_dim : 0;
  const size_t part_ml = n_chunks > 1 ? static_cast<size_t>(n_chunks) * T * Hq * 2 : 0;
  if ((part_o + part_ml) * sizeof(float) > D3D_ATTN_NOALLOC_SCRATCH_BYTES) return D3D_NOALLOC_ERR_TOO_LARGE;
  void* base = nullptr;
  const cudaError_t e = scratch_for_current_device(&base);
  if (e != cudaSuccess) return e == cudaErrorInvalidSymbol ? D3D_NOALLOC_ERR_SYMBOL : static_cast<int>(e);
  d3d::AttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k_cache = static_cast<const __nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<const __nv_bfloat16*>(v_cache);
  a.block_table = block_table;
  a.bt_stride = bt_stride;
  a.rows = rows;
  a.kv_end = kv_end;
  a.B = B;
  a.q_len = q_len;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.head_dim = head_dim;
  a.page_size = page_size;
  a.scale = scale;
  a.chunk = chunk;
  a.n_chunks = n_chunks;
  a.part_o = n_chunks > 1 ? static_cast<float*>(base) : nullptr;
  a.part_ml = n_chunks > 1 ? static_cast<float*>(base) + part_o : nullptr;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.num_slots = num_slots;
  a.status = nullptr;
  return static_cast<int>(d3d::attention_split(a, stream));
}
