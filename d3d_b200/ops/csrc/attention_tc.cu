// Paged-KV attention with structured row masks on the 5th-generation tensor
// cores (tcgen05 + TMEM, TMA-fed), sm_100a.  Reference counterparts: the
// FlashAttention-2 / dense-mask SDPA calls of serving/vendor/ssd/layers/
// attention.py:8-53 (prefill, paged verify, packed draft) and the mask
// builders of single/eval_sync.py:194-275, whose masks arrive here as one
// (lim, lo, hi) triple per query row: the row sees key slots
// ``k < lim  or  lo <= k < hi`` (structured; no dense mask exists).
//
// CTA = 128 packed query rows of one (sequence, kv head) and one key chunk.
// Packed row r is query token r / g and query head h*g + r % g (g = GQA
// group), so every K/V tile serves the whole group.  Roles (320 threads):
//   warp 0, lane 0   TMA: the Q tile once (3-D box {64 d, g heads, 128/g
//                    tokens}, two boxes for d = 128), then per 64-key tile
//                    one K and one V box per page ({64 d, 1 head, page keys})
//                    into a 3-stage ring, 128-byte swizzle, mbarrier tx;
//                    key tiles no row of the CTA can see are never loaded;
//   warp 1, lane 0   MMA issuer: S_j = Q K_j^T (M=128, N=64, K=d: K-major
//                    A and B) into one of two TMEM S buffers; then, once the
//                    softmax warps have written P_j, O += P_j V_j (M=128,
//                    N=d, K=64; V is read N-major straight from the ring)
//                    into one TMEM O accumulator that lives across tiles.
//                    S_{j+1} is issued before PV_j, so the softmax of tile
//                    j+1 overlaps PV_j;
//   warps 2..9       softmax: warp w reads TMEM lane quadrant w % 4 (its 32
//                    rows); warps 2-5 own key columns 0-31 and d columns
//                    0..d/2-1, warps 6-9 the other halves.  Each thread
//                    loads its row's 64 scores, takes the row max over all
//                    64 (both halves agree on it), masks with (lim, lo, hi)
//                    and writes bf16 P = 2^(s - m) for its 32 keys into a
//                    swizzled shared tile (the A operand of PV).  The
//                    reference max m of a row only moves when the row's
//                    running max exceeds it by more than 2^8; then the row's
//                    O columns are rescaled in TMEM (after PV_{j-1} has
//                    retired) before P_j is published.  Every decision
//                    depends on the row's own scores only.
// Keys are cut into chunks at fixed absolute boundaries (grid z); a chunk's
// tiles run in increasing key order; chunk results are merged by the
// fixed-order combine kernel.  A row's result therefore depends only on its
// own query, keys and mask -- never on which rows share its CTA -- so a
// token's attention is bit-identical whether it is verified in a block or
// decoded alone (greedy token identity with AR decoding).
//
// Every mbarrier wait is bounded (timeout -> status code, CTA-wide abort,
// every role leaves its loop); teardown waits, bounded, for issued TMA loads
// and MMAs before TMEM is released.  No cluster multicast is used.
#include <atomic>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace d3d {

constexpr int TA_ROWS = 128;
constexpr int TA_KEYS = 64;
constexpr int TA_STAGES = 3;
constexpr int TA_THREADS = 320;
constexpr int TA_MAX_PAGES = 1024;

template <int D>
struct TaCfg {
  static constexpr int NH = D / 64;                        // 64-wide d halves (one swizzle row each)
  static constexpr int Q_HALF = TA_ROWS * 64 * 2;          // 16 KB
  static constexpr int KV_HALF = TA_KEYS * 64 * 2;         // 8 KB
  static constexpr int STAGE = 2 * NH * KV_HALF;           // K halves then V halves
  static constexpr int P_BYTES = TA_ROWS * TA_KEYS * 2;    // 16 KB
  static constexpr int OFF_KV = NH * Q_HALF;
  static constexpr int OFF_P = OFF_KV + TA_STAGES * STAGE;
  static constexpr int SMEM = OFF_P + 2 * P_BYTES + 1024;  // + 1024-byte alignment slack
  static constexpr int COL_S = 0;                          // TMEM: S buffers, 2 x 64 columns
  static constexpr int COL_O = 128;                        // TMEM: O accumulator, D columns
  static constexpr uint32_t TMEM_COLS = (128 + D) <= 256 ? 256u : 512u;
};

// 2^x on the MUFU unit (PTX ex2.approx, subnormal results flushed to zero;
// 2^-inf = +0).  Softmax weights are rounded to bf16 right after, so the
// instruction's approximation error is below that rounding.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
__global__ void __launch_bounds__(TA_THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnArgs a, const int kb,
                   const unsigned long long lim_ns) {
  using C = TaCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ int s_rows[TA_ROWS][3];
  __shared__ int s_range[3];
  __shared__ int s_pages[TA_MAX_PAGES];
  __shared__ float s_lpart[2][TA_ROWS];
  __shared__ uint64_t q_full, kv_full[TA_STAGES], kv_empty[TA_STAGES];
  __shared__ uint64_t s_full[2], s_free[2], p_full[2], o_done, done;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int flags[4];  // [0] abort  [1] tiles issued (TMA)  [2] tiles consumed (MMA)  [3] Q issued

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = a.Hq / a.Hkv;
  const int b = blockIdx.y / a.Hkv, h = blockIdx.y % a.Hkv;
  const int chunk_id = blockIdx.z;
  const int R0 = blockIdx.x * TA_ROWS;
  const int kv_end = a.kv_end[b];
  const int ps = a.page_size;
  const int kbeg = chunk_id * a.chunk;
  const int kend = min(kbeg + a.chunk, kv_end);
  const int pg0 = kbeg / ps;

  // ---------------------------------------------------------------- prologue
  // Row descriptors, kv_end and the block table are step inputs written
  // before the forward starts; they are read before the grid dependency.
  if (tid < TA_ROWS) {
    const int t = (R0 + tid) / g;
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
    mbar_init(&q_full, 1);
    for (int s = 0; s < TA_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 8);
      mbar_init(&p_full[i], 8);
    }
    mbar_init(&o_done, 1);       // one phase per PV product, waited in order
    mbar_init(&done, 1);
    flags[0] = flags[1] = flags[2] = flags[3] = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    griddep_launch();
  }
  {
    // pages of this chunk (clamped to the block-table row)
    const int* bt = a.block_table + static_cast<size_t>(b) * a.bt_stride;
    const int npg = kend > kbeg ? min((kend - 1) / ps - pg0 + 1, a.bt_stride - pg0) : 0;
    for (int i = tid; i < npg && i < TA_MAX_PAGES; i += TA_THREADS) s_pages[i] = bt[pg0 + i];
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  if (tid < TA_ROWS) {
    atomicMax(&s_range[0], s_rows[tid][0]);
    if (s_rows[tid][2] > s_rows[tid][1]) {
      atomicMin(&s_range[1], s_rows[tid][1]);
      atomicMax(&s_range[2], s_rows[tid][2]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int max_lim = s_range[0], min_lo = s_range[1], max_hi = s_range[2];
  auto needed = [&](int k0) { return k0 < max_lim || (k0 + TA_KEYS > min_lo && k0 < max_hi); };
  auto next_tile = [&](int k0) {
    while (k0 < kend && !needed(k0)) k0 += TA_KEYS;
    return k0;
  };
  auto fail = [&](int code) {
    set_error(a.status, code);
    flags[0] = 1;
  };
  const uint64_t lim = lim_ns;

  if (warp == 0) {
    // --------------------------------------------------------------- TMA
    // lane 0 issues the copies; the whole warp zeroes the V rows of boxes
    // past kv_end (never loaded: a masked key contributes P = 0, and
    // 0 * finite = 0 in the PV product, so those rows must hold finite values)
    griddep_wait();
    if (lane == 0 && kend > kbeg) {
      mbar_arrive_expect_tx(&q_full, C::NH * C::Q_HALF);
      for (int hf = 0; hf < C::NH; ++hf)
        tma_load_3d(smem + hf * C::Q_HALF, &tmQ, &q_full, hf * 64, h * g, b * a.q_len + R0 / g);
      flags[3] = 1;
    }
    int j = 0;
    for (int k0 = next_tile(kbeg); k0 < kend && !flags[0]; k0 = next_tile(k0 + TA_KEYS), ++j) {
      const int s = j % TA_STAGES;
      bool ok = mbar_wait(&kv_empty[s], ((j / TA_STAGES) & 1) ^ 1, lim);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) fail(ERR_TIMEOUT_PRODUCER);
        break;
      }
      uint8_t* st = smem + C::OFF_KV + s * C::STAGE;
      int boxes = 0;
      for (int i = 0; i < TA_KEYS / kb; ++i) {
        if (k0 + i * kb < kv_end) {
          ++boxes;
          continue;
        }
        for (int hf = 0; hf < C::NH; ++hf) {
          uint4* z = reinterpret_cast<uint4*>(st + (C::NH + hf) * C::KV_HALF + i * kb * 128);
          for (int e = lane; e < kb * 8; e += 32) z[e] = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&kv_full[s], static_cast<uint32_t>(boxes * 2 * C::NH * kb * 128));
        for (int i = 0; i < boxes; ++i) {
          const int key = k0 + i * kb;
          const int slot = s_pages[key / ps - pg0] * ps + key % ps;
          for (int hf = 0; hf < C::NH; ++hf) {
            tma_load_3d(st + hf * C::KV_HALF + i * kb * 128, &tmK, &kv_full[s], hf * 64, h, slot);
            tma_load_3d(st + (C::NH + hf) * C::KV_HALF + i * kb * 128, &tmV, &kv_full[s], hf * 64, h, slot);
          }
        }
        flags[1] = j + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------- MMA
      constexpr uint32_t idesc_s = idesc_bf16_f32(TA_ROWS, TA_KEYS);
      constexpr uint32_t idesc_o = idesc_bf16_f32(TA_ROWS, D) | (1u << 16);  // B (V) N-major
      const uint32_t q_addr = smem_u32(smem);
      bool ok = true;
      int n = 0;
      for (int k0 = next_tile(kbeg); k0 < kend; k0 = next_tile(k0 + TA_KEYS)) ++n;
      if (n > 0 && !mbar_wait(&q_full, 0, lim)) {
        fail(ERR_TIMEOUT_MMA);
        ok = false;
      }
      auto issue_s = [&](int j) -> bool {
        const int s = j % TA_STAGES, buf = j & 1;
        if (!mbar_wait(&kv_full[s], (j / TA_STAGES) & 1, lim) || !mbar_wait(&s_free[buf], ((j >> 1) & 1) ^ 1, lim)) {
          fail(ERR_TIMEOUT_MMA);
          return false;
        }
        flags[2] = j + 1;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + C::OFF_KV + s * C::STAGE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int hf = kk >> 2, off = (kk & 3) * 32;
          umma_bf16(tmem + C::COL_S + buf * TA_KEYS, sdesc_kmajor_sw128(q_addr + hf * C::Q_HALF + off),
                    sdesc_kmajor_sw128(k_addr + hf * C::KV_HALF + off), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[buf]);
        return true;
      };
      auto issue_o = [&](int j) -> bool {
        const int s = j % TA_STAGES, buf = j & 1;
        if (!mbar_wait(&p_full[buf], (j >> 1) & 1, lim)) {
          fail(ERR_TIMEOUT_MMA);
          return false;
        }
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + C::OFF_P + buf * C::P_BYTES);
        const uint32_t v_addr = smem_u32(smem + C::OFF_KV + s * C::STAGE + C::NH * C::KV_HALF);
#pragma unroll
        for (int kk = 0; kk < TA_KEYS / 16; ++kk)
          umma_bf16(tmem + C::COL_O, sdesc_kmajor_sw128(p_addr + kk * 32),
                    sdesc_mnmajor_sw128(v_addr + kk * 16 * 128, C::KV_HALF), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&o_done);
        umma_commit(&kv_empty[s]);
        return true;
      };
      if (ok && n > 0) ok = issue_s(0);
      for (int j = 0; ok && j < n && !flags[0]; ++j) {
        if (j + 1 < n && !(ok = issue_s(j + 1))) break;
        ok = issue_o(j);
      }
    }
  } else {
    // ------------------------------------------------------------- softmax
    const int qd = warp & 3;                 // TMEM lane quadrant
    const int ch = (warp - 2) >> 2;          // column half
    const int row = qd * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    const uint32_t t_o = t_lane + C::COL_O + ch * (D / 2);
    const int lim_r = s_rows[row][0], lo_r = s_rows[row][1], hi_r = s_rows[row][2];
    const float sl2 = a.scale * 1.4426950408889634f;  // scale * log2(e)
    constexpr int DH = D / 2;
    constexpr float RESCALE = 8.f;           // move the reference max when it is exceeded by 2^8
    float m = -INFINITY, l = 0.f;
    uint8_t* prow_base = smem + C::OFF_P + row * 128;
    bool ok = true;

    // every lane waits; the warp follows lane 0's verdict so warp-collective
    // TMEM accesses stay converged
    auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
      bool w = mbar_wait(bar, parity, lim);
      w = __shfl_sync(0xffffffffu, w && !flags[0], 0);
      if (!w && lane == 0 && !flags[0]) fail(ERR_TIMEOUT_EPILOGUE);
      return w;
    };

    int j = 0;
    for (int k0 = next_tile(kbeg); k0 < kend; k0 = next_tile(k0 + TA_KEYS), ++j) {
      const int buf = j & 1;
      if (!(ok = warp_wait(&s_full[buf], (j >> 1) & 1))) break;
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld32_nowait(t_lane + C::COL_S + buf * TA_KEYS, sr);
      tmem_ld32_nowait(t_lane + C::COL_S + buf * TA_KEYS + 32, sr + 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[buf]);
      // Visible keys of this row inside the tile, as tile columns:
      // [0, va) U [vb, ve)  (from k < lim  or  lo <= k < hi, clipped to kend).
      const int kc = kend - k0;
      const int va = max(0, min(min(lim_r, kend) - k0, TA_KEYS));
      const int vb = max(0, min(lo_r - k0, TA_KEYS));
      const int ve = max(vb, min(min(hi_r, kend) - k0, TA_KEYS));
      const bool full = kc >= TA_KEYS && (va == TA_KEYS || (vb == 0 && ve == TA_KEYS));
      // row max over the raw scores (scale > 0 commutes with max)
      float tr = -INFINITY;
      if (full) {
#pragma unroll
        for (int c = 0; c < 64; ++c) tr = fmaxf(tr, __uint_as_float(sr[c]));
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const bool vis = c < va || static_cast<unsigned>(c - vb) < static_cast<unsigned>(ve - vb);
          sr[c] = vis ? sr[c] : 0xff800000u;          // -inf
          tr = fmaxf(tr, __uint_as_float(sr[c]));
        }
      }
      const float tm = tr * sl2;
      // reference max: set on the first visible scores, moved only by > 2^8
      float alpha = 1.f;
      if (m == -INFINITY) {
        m = tm;
      } else if (tm > m + RESCALE) {
        alpha = ex2_ftz(m - tm);
        m = tm;
      }
      float sum = 0.f;
      uint32_t pk[16];
      if (m == -INFINITY) {        // nothing visible yet: P = 0
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = 0u;
      } else {
        // p = 2^(raw * scale*log2e - m); a masked key (raw = -inf) gives 0
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float x0 = __uint_as_float(ch ? sr[32 + e] : sr[e]);    // static indices
          const float x1 = __uint_as_float(ch ? sr[33 + e] : sr[e + 1]);
          const float p0 = ex2_ftz(fmaf(x0, sl2, -m));
          const float p1 = ex2_ftz(fmaf(x1, sl2, -m));
          sum += p0 + p1;
          __nv_bfloat162 v = __floats2bfloat162_rn(p0, p1);
          pk[e >> 1] = *reinterpret_cast<uint32_t*>(&v);
        }
      }
      l = l * alpha + sum;
      // PV_{j-1} has retired before P_j is published (the O rescale below and
      // the reuse of P buffer (j & 1), last read by PV_{j-2}, rely on it)
      if (j > 0 && !(ok = warp_wait(&o_done, (j - 1) & 1))) break;
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < DH; c += 32) {
          uint32_t r[32];
          tmem_ld32_nowait(t_o + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
          tmem_st32(t_o + c, r);
        }
        tmem_wait_st();
      }
      // P row: keys 32ch..32ch+31 = 16-byte chunks 4ch..4ch+3, 128-byte swizzle
      uint8_t* prow = prow_base + buf * C::P_BYTES;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int chunk = (ch * 4 + i) ^ (row & 7);
        *reinterpret_cast<uint4*>(prow + chunk * 16) = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[buf]);
    }
    // the last PV product, then this thread's O columns
    float o[DH];
    if (ok && j > 0) ok = warp_wait(&o_done, (j - 1) & 1);
    if (ok && j > 0) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < DH; c += 32) {
        uint32_t r[32];
        tmem_ld32_nowait(t_o + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[c + e] = __uint_as_float(r[e]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < DH; ++e) o[e] = 0.f;
    }

    // ---- combine the two column halves' row sums (fixed order: half 0 + half 1)
    s_lpart[ch][row] = l;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float ltot = s_lpart[0][row] + s_lpart[1][row];
    griddep_wait();   // outputs may still be read by the previous kernel until it completes
    const int R = R0 + row;
    const int t = R / g;
    if (ok && !flags[0] && t < a.q_len) {
      const size_t tok = static_cast<size_t>(b) * a.q_len + t;
      const int qh = h * g + R % g;
      if (a.n_chunks == 1) {
        const float inv = ltot > 0.f ? 1.f / ltot : 0.f;
        __nv_bfloat16* dst = a.out + (tok * a.Hq + qh) * D + ch * DH;
#pragma unroll
        for (int c = 0; c < DH; c += 8) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 v = __floats2bfloat162_rn(o[c + 2 * e] * inv, o[c + 2 * e + 1] * inv);
            w[e] = *reinterpret_cast<uint32_t*>(&v);
          }
          *reinterpret_cast<uint4*>(dst + c) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
        const size_t T = static_cast<size_t>(a.B) * a.q_len;
        const size_t cb = static_cast<size_t>(chunk_id) * T * a.Hq;
        float* dst = a.part_o + (cb + tok * a.Hq + qh) * D + ch * DH;
#pragma unroll
        for (int c = 0; c < DH; c += 4)
          *reinterpret_cast<float4*>(dst + c) = make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
        if (ch == 0) *reinterpret_cast<float2*>(a.part_ml + (cb + tok * a.Hq + qh) * 2) = make_float2(m, ltot);
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  __syncthreads();
  if (tid == 32) {
    // every MMA this thread issued has retired before TMEM is released
    umma_commit(&done);
    if (!mbar_wait(&done, 0, lim)) set_error(a.status, ERR_TIMEOUT_MMA);
  }
  if (tid == 0 && flags[0]) {
    // drain TMA loads that were issued but never consumed, so no copy lands
    // in shared memory after the CTA has exited
    if (flags[3] && flags[2] == 0) mbar_wait(&q_full, 0, lim);
    for (int i = flags[2]; i < flags[1]; ++i) mbar_wait(&kv_full[i % TA_STAGES], (i / TA_STAGES) & 1, lim);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ------------------------------------------------------------------ host side
// The tensor-core path serves head_dim 64 / 128, GQA groups dividing 128 and
// pages of 8..64 keys dividing 64 or multiples of 64 (whole 64-key tiles).
// D3D_ATTN_TC=0 sends every shape to the mma.sync kernels instead.
bool attention_tc_supported(const AttnArgs& a) {
  static const int mode = [] {
    const char* e = std::getenv("D3D_ATTN_TC");
    return e ? std::atoi(e) : 1;
  }();
  if (!mode) return false;
  const int g = a.Hkv > 0 ? a.Hq / a.Hkv : 0;
  if (a.head_dim != 64 && a.head_dim != 128) return false;
  if (g <= 0 || a.Hq % a.Hkv || TA_ROWS % g) return false;
  const int ps = a.page_size;
  if (ps < 8 || ps % 8 || !(TA_KEYS % ps == 0 || ps % TA_KEYS == 0)) return false;
  if (a.chunk <= 0 || a.chunk % TA_KEYS || a.chunk / ps + 1 > TA_MAX_PAGES) return false;
  if (a.n_chunks > 1 && (!a.part_o || !a.part_ml)) return false;
  if (a.n_chunks < 1 || a.n_chunks > 512) return false;
  return a.num_slots > 0;
}

template <int D>
static cudaError_t ensure_tc_attr() {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(attn_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, TaCfg<D>::SMEM);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

template <int D>
static void launch_tc(const AttnArgs& a, cudaStream_t st) {
  const int g = a.Hq / a.Hkv;
  const int kb = a.page_size < TA_KEYS ? a.page_size : TA_KEYS;
  const uint64_t T = static_cast<uint64_t>(a.B) * a.q_len;
  CUtensorMap tq, tk, tv;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(a.Hq), T};
    const uint64_t str[2] = {static_cast<uint64_t>(D), static_cast<uint64_t>(a.Hq) * D};
    const uint32_t box[3] = {64u, static_cast<uint32_t>(g), static_cast<uint32_t>(TA_ROWS / g)};
    make_tmap_bf16_3d(&tq, a.q, dims, str, box);
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(a.Hkv),
                              static_cast<uint64_t>(a.num_slots)};
    const uint64_t str[2] = {static_cast<uint64_t>(D), static_cast<uint64_t>(a.Hkv) * D};
    const uint32_t box[3] = {64u, 1u, static_cast<uint32_t>(kb)};
    make_tmap_bf16_3d(&tk, a.k_cache, dims, str, box);
    make_tmap_bf16_3d(&tv, a.v_cache, dims, str, box);
  }
  cudaError_t e = ensure_tc_attr<D>();
  if (e != cudaSuccess) throw std::runtime_error(std::string("attention_tc attribute: ") + cudaGetErrorString(e));
  dim3 grid((a.q_len * g + TA_ROWS - 1) / TA_ROWS, a.B * a.Hkv, a.n_chunks);
  const unsigned long long lim = 2000000000ull;  // 2 s per wait
  e = launch_pdl(attn_tc_kernel<D>, grid, dim3(TA_THREADS), static_cast<size_t>(TaCfg<D>::SMEM), st, tq, tk, tv,
                 a, kb, lim);
  if (e != cudaSuccess) throw std::runtime_error(std::string("attention_tc launch: ") + cudaGetErrorString(e));
  if (a.n_chunks > 1) {
    e = attention_combine(a, st);
    if (e != cudaSuccess) throw std::runtime_error(std::string("attention combine: ") + cudaGetErrorString(e));
  }
}

void attention_tc(const AttnArgs& a, cudaStream_t st) {
  if (a.B == 0 || a.q_len == 0) return;
  if (!attention_tc_supported(a)) throw std::runtime_error("attention_tc: unsupported shape");
  if (a.head_dim == 128) launch_tc<128>(a, st);
  else launch_tc<64>(a, st);
}

}  // namespace d3d
