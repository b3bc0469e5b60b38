// Weight-stationary tcgen05 GEMM for sm_100a:  Y[M, N] = X[M, K] · W[N, K]^T.
// It stands in for the reference's linear layers (serving/vendor/ssd/layers/
// linear.py:42-199) and its chunked LM-head greedy / top-k selection
// (serving/backend.py:78-95), with the top-k fused into the epilogue.
//
// Decode-time matmuls have few tokens (M = 1..1088) against large weights, so
// the tile is laid out "swap-AB": the 128-row MMA M dimension runs over weight
// rows (output features) and the MMA N dimension over tokens: ``bt`` = 16..256
// (a multiple of 16) in one MMA, or up to 512 (a multiple of 32) as two MMAs
// of bt/2 columns each.  A work unit is a 128 x bt output tile and a
// contiguous range of K blocks (split-K chosen by the host from the weight
// shape alone, so the fp32 reduction order of every output element is
// independent of M -- the property greedy token identity between AR and
// speculative decoding rests on).
//
// The kernel is persistent: min(units, SMs x CTAs-per-SM) CTAs walk the units
// round-robin (unit order: weight tile, then token tile, then split, so CTAs
// running side by side share weight tiles in L2).  Per CTA (192 threads):
//   warp 0 lane 0  TMA producer: W tile [128 x 64] and X tile [bt x 64] per
//                  stage, 128-byte swizzle, mbarrier complete_tx, one
//                  continuous pipeline across units;
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma (K = 16 each) per stage into
//                  one of two TMEM accumulators (128 lanes x bt fp32 columns),
//                  tcgen05.commit frees the stage; after a unit's last stage
//                  it commits the accumulator to the epilogue;
//   warps 2..5     epilogue: tcgen05.ld 32x32b (warp w reads TMEM lanes
//                  32(w%4)..+31 = output rows), hands the accumulator back,
//                  then stores -- overlapping the next unit's main loop:
//                  MODE 0  fp32 split-K partials  P[split][M][N]
//                  MODE 1  bf16 Y (+ bf16 residual, rounded like two bf16 ops)
//                  MODE 2  per-tile top-KT (value, index) over the 128 rows,
//                          for LM-head argmax / top-k without storing logits
//                  MODE 3  SwiGLU of an interleaved gate|up weight: tile row
//                          32w+i holds gate row 64t+16w+i (i < 16) or the
//                          matching up row (i >= 16), so lane i pairs with
//                          lane i+16 of the same warp: h = silu(g) * u, bf16.
// Every mbarrier wait is bounded; a timeout records an error code in
// ``status``, raises a CTA-wide abort flag and every role leaves its loop;
// teardown waits (bounded) for issued TMA loads and MMAs before TMEM is
// freed.  Launched with programmatic dependent launch: the producer streams
// the first stages of weights before griddepcontrol.wait.
#include "common.cuh"
#include "gemm.h"

#include <cudaTypedefs.h>
#include <mutex>
#include <stdexcept>
#include <string>

namespace d3d {

constexpr int GBN = 128;  // weight rows per tile (MMA M)
constexpr int GBK = 64;   // K per stage (one 128-byte swizzle atom of bf16)
constexpr int A_TILE_BYTES = GBN * GBK * 2;
constexpr int GEMM_THREADS = 192;
constexpr int TSCR_WORDS = 32 * 33;   // MODE 2 transpose scratch per epilogue warp

__host__ __device__ inline int acc_cols_for(int bt) {
  if (bt > 256) return 512;
  int c = 32;
  while (c < bt) c <<= 1;
  return c;
}
__host__ __device__ inline int num_acc_for(int bt) { return (bt <= 256 && 2 * acc_cols_for(bt) <= 512) ? 2 : 1; }

struct UnitCoord {
  int n_t, m_t, split, kb0, kb1;
};

__device__ __forceinline__ UnitCoord unit_coord(int t, int ntm, int nsplit, int nkb) {
  UnitCoord u;
  u.split = t % nsplit;
  const int r = t / nsplit;
  u.m_t = r % ntm;
  u.n_t = r / ntm;
  u.kb0 = (nkb * u.split) / nsplit;
  u.kb1 = (nkb * (u.split + 1)) / nsplit;
  return u;
}

template <int MODE, int KT>
__global__ void __launch_bounds__(GEMM_THREADS, 2)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bt = p.bt;
  const int stages = p.stages;
  const int stage_bytes = A_TILE_BYTES + bt * GBK * 2;
  // MODE 2 cross-warp merge areas, double-buffered: [2][4 warps][bt][KT] (value, index)
  const int marea = MODE == 2 ? 4 * bt * KT : 0;
  float* mval = reinterpret_cast<float*>(smem + stages * stage_bytes);
  int* midx = reinterpret_cast<int*>(mval + 2 * marea);
  // MODE 2: per-epilogue-warp transpose scratch, 32 rows x 33 words (padded: conflict-free both ways)
  uint32_t* tscr = reinterpret_cast<uint32_t*>(midx + 2 * marea);
  uint64_t* full = reinterpret_cast<uint64_t*>(tscr + (MODE == 2 && bt > 32 ? 4 * TSCR_WORDS : 0));
  uint64_t* empty = full + stages;
  uint64_t* accf = empty + stages;  // [2] accumulator ready for the epilogue
  uint64_t* acce = accf + 2;        // [2] accumulator drained by the epilogue
  uint64_t* mfull = acce + 2;       // [2] MODE 2: the four warps' candidates are in
  uint64_t* mempty = mfull + 2;     // [2] MODE 2: merge area read, may be rewritten
  uint64_t* done = mempty + 2;
  uint64_t* finb = done + 1;        // MODE 4: the four epilogue warps meet here (bounded waits)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(finb + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort [1] issued [2] consumed
                                                                         // [3] MODE 4: this CTA finalizes

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (p.K + GBK - 1) / GBK;
  const int ntn = (p.N + GBN - 1) / GBN, ntm = (p.M + bt - 1) / bt, nsplit = p.splits;
  const int units = ntn * ntm * nsplit;
  const int nsub = bt > 256 ? 2 : 1;  // MMAs per K step
  const int sub = bt / nsub;          // tokens per MMA (multiple of 16)
  const int acc_cols = acc_cols_for(bt);
  const int nacc = num_acc_for(bt);
  const uint32_t tmem_cols = static_cast<uint32_t>(acc_cols * nacc);
  const uint64_t lim = p.timeout_ns;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 4);
      mbar_init(&mfull[a], 4);
      mbar_init(&mempty[a], 1);
    }
    mbar_init(done, 1);
    mbar_init(finb, 4);
    flags[0] = flags[1] = flags[2] = flags[3] = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmW);
    prefetch_tensormap(&tmX);
    griddep_launch();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto fail = [&](int code) {
    set_error(p.status, code);
    flags[0] = 1;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol_w = policy_evict_first();  // weights stream through L2 once
      auto load_w = [&](const UnitCoord& u, int kb, int s) {
        uint8_t* sa = smem + s * stage_bytes;
        if (p.w_packed)  // contiguous 16 KB tiles: [N/128][K/64][128][64]
          tma_load_2d_hint(sa, &tmW, &full[s], 0, (u.n_t * nkb + kb) * GBN, pol_w);
        else
          tma_load_2d_hint(sa, &tmW, &full[s], kb * GBK, u.n_t * GBN, pol_w);
      };
      auto load_x = [&](const UnitCoord& u, int kb, int s) {
        uint8_t* sb = smem + s * stage_bytes + A_TILE_BYTES;
        for (int v = 0; v < nsub; ++v)
          tma_load_2d(sb + v * sub * GBK * 2, &tmX, &full[s], kb * GBK, u.m_t * bt + v * sub);
      };
      uint32_t it = 0;
      int pre = 0;
      if (static_cast<int>(blockIdx.x) < units) {
        // weights do not depend on earlier kernels: fill the pipeline before
        // the grid dependency resolves, then add the activation tiles
        const UnitCoord u0 = unit_coord(blockIdx.x, ntm, nsplit, nkb);
        pre = min(u0.kb1 - u0.kb0, stages);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], stage_bytes);
          load_w(u0, u0.kb0 + i, i);
        }
        griddep_wait();
        for (int i = 0; i < pre; ++i) load_x(u0, u0.kb0 + i, i);
        it = pre;
      } else {
        griddep_wait();
      }
      bool first = true;
      for (int t = blockIdx.x; t < units && !flags[0]; t += gridDim.x, first = false) {
        const UnitCoord u = unit_coord(t, ntm, nsplit, nkb);
        for (int kb = u.kb0 + (first ? pre : 0); kb < u.kb1; ++kb, ++it) {
          const int s = it % stages;
          if (!mbar_wait(&empty[s], ((it / stages) & 1) ^ 1, lim)) {
            fail(ERR_TIMEOUT_PRODUCER);
            break;
          }
          mbar_arrive_expect_tx(&full[s], stage_bytes);
          load_w(u, kb, s);
          load_x(u, kb, s);
        }
      }
      flags[1] = static_cast<int>(it);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // -------------------------------------------------------- MMA issuer
      const uint32_t idesc = idesc_bf16_f32(GBN, sub);
      uint32_t it = 0;
      int ti = 0;
      for (int t = blockIdx.x; t < units && !flags[0]; t += gridDim.x, ++ti) {
        const UnitCoord u = unit_coord(t, ntm, nsplit, nkb);
        const int a = ti % nacc, use = ti / nacc;
        if (!mbar_wait(&acce[a], (use & 1) ^ 1, lim)) {
          fail(ERR_TIMEOUT_MMA);
          break;
        }
        tc_fence_after();
        const uint32_t td = tmem + static_cast<uint32_t>(a * acc_cols);
        bool ok = true;
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++it) {
          const int s = it % stages;
          if (!mbar_wait(&full[s], (it / stages) & 1, lim)) {
            fail(ERR_TIMEOUT_MMA);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * stage_bytes);
          const uint64_t ad = sdesc_kmajor_sw128(sa);
          const uint64_t bd = sdesc_kmajor_sw128(sa + A_TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < GBK / 16; ++kk) {
            // +32 bytes along K inside the swizzle atom = +2 in the >>4 address field
            const uint32_t acc = (kb > u.kb0 || kk > 0) ? 1u : 0u;
            umma_bf16(td, ad + 2 * kk, bd + 2 * kk, idesc, acc);
            if (nsub == 2) {
              const uint64_t bd2 = sdesc_kmajor_sw128(sa + A_TILE_BYTES + sub * GBK * 2);
              umma_bf16(td + sub, ad + 2 * kk, bd2 + 2 * kk, idesc, acc);
            }
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&accf[a]);
      }
      flags[2] = static_cast<int>(it);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    griddep_wait();  // outputs may still be read by the previous kernel until it completes
    const int q = warp & 3;           // TMEM lane quadrant of this warp
    const int row = q * 32 + lane;    // weight row within the tile
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t fph = 0;   // MODE 4: completed phases of finb
    // the four epilogue warps meet (lane 0 of each arrives; every lane waits,
    // bounded); false when the wait ran out or the CTA aborted
    auto fsync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(finb);
      bool w = mbar_wait(finb, fph & 1, lim);
      ++fph;
      w = __shfl_sync(0xffffffffu, w && !flags[0], 0);
      if (!w && lane == 0 && !flags[0]) fail(ERR_TIMEOUT_EPILOGUE);
      return w;
    };
    int ti = 0;
    for (int t = blockIdx.x; t < units; t += gridDim.x, ++ti) {
      const UnitCoord u = unit_coord(t, ntm, nsplit, nkb);
      const int a = ti % nacc, use = ti / nacc;
      bool ok = !flags[0] && mbar_wait(&accf[a], use & 1, lim);
      if (!ok) {
        if (!flags[0]) fail(ERR_TIMEOUT_EPILOGUE);
        break;
      }
      tc_fence_after();
      const uint32_t tacc = t_lane + static_cast<uint32_t>(a * acc_cols);
      const int n0 = u.n_t * GBN, m0 = u.m_t * bt;
      const int n = n0 + row;
      const bool n_ok = n < p.N;
      if constexpr (MODE == 0 || MODE == 1 || MODE == 3 || MODE == 4) {
        // MODE 3 output column of this lane (lanes 0..15 of each warp write)
        const int hcol = u.n_t * (GBN / 2) + q * 16 + (lane & 15);
        const int cols = min(bt, p.M - m0);
        for (int c = 0; c < cols; c += 16) {
          float v[16];
          tmem_ld16(tacc + c, v);
          if constexpr (MODE == 0 || MODE == 4) {
            if (n_ok && p.tp == 0) {
              float* base = p.out_f32 + static_cast<size_t>(u.split) * p.M * p.N;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int m = m0 + c + j;
                if (c + j < cols) base[static_cast<size_t>(m) * p.N + n] = v[j];
              }
            } else if (n_ok) {
              // tensor parallel: the same partial into every rank's exchange
              // buffer (peer stores over NVLink), slot rank * splits + split
              const size_t slot = static_cast<size_t>(p.tp_rank * p.splits + u.split) * p.M * p.N;
              for (int r = p.tp_pull ? p.tp_rank : 0; r < (p.tp_pull ? p.tp_rank + 1 : p.tp); ++r) {
                float* base = p.tp_out[r] + slot;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const int m = m0 + c + j;
                  if (c + j < cols) base[static_cast<size_t>(m) * p.N + n] = v[j];
                }
              }
            }
          } else if constexpr (MODE == 1) {
            if (n_ok) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int m = m0 + c + j;
                if (c + j < cols) {
                  float y = v[j];
                  if (p.residual) y = bf16r(y) + __bfloat162float(p.residual[static_cast<size_t>(m) * p.ldr + n]);
                  p.out_bf16[static_cast<size_t>(m) * p.ldc + n] = __float2bfloat16(y);
                }
              }
            }
          } else {
            float uu[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) uu[j] = __shfl_down_sync(0xffffffffu, v[j], 16);
            if (lane < 16 && 2 * hcol < p.N) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int m = m0 + c + j;
                if (c + j < cols) {
                  const float g = bf16r(v[j]);
                  const float sl = bf16r(g / (1.f + expf(-g)));
                  p.out_bf16[static_cast<size_t>(m) * p.ldc + hcol] = __float2bfloat16(sl * bf16r(uu[j]));
                }
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[a]);
        if constexpr (MODE == 4) {
          // ---- in-kernel split-K reduction: the last unit of this output
          // tile to store its partials sums all splits (split order), adds
          // them to the residual (rounded like two bf16 ops) and writes the
          // tile's per-row sum of squares of the new residual.
          __threadfence();
          if (!fsync()) break;
          const int tile = u.n_t * ntm + u.m_t;
          if (threadIdx.x == 64) {
            const unsigned int tk = atomicAdd(p.fin_ticket + tile, 1u);
            flags[3] = (tk == static_cast<unsigned int>(nsplit - 1)) ? 1 : 0;
          }
          if (!fsync()) break;
          if (flags[3]) {
            __threadfence();
            // warp q takes token columns q, q+4, ...; lane l the tile's rows
            // 4l..4l+3 (16-byte loads, every split's load in flight before the
            // adds), so one warp finishes a column and its sum of squares
            // (residual_split_reduce in fused.cu computes the same values)
            for (int c = q; c < cols; c += 4)
              split_reduce_row(p.out_f32, nsplit, static_cast<size_t>(p.M) * p.N, p.N, p.fin_x, p.fin_ldx,
                               p.fin_sumsq, p.M, m0 + c, u.n_t, lane);
            if (threadIdx.x == 64) p.fin_ticket[tile] = 0u;   // ready for the next launch
          }
        }
      } else {
        // ------------------------------------------ MODE 2: per-tile top-KT
        // More than 32 token columns: per 32-column chunk, each epilogue warp stores its 32 rows x 32
        // columns of order-preserving keys (0 = row past N) into its padded
        // shared-memory scratch and reads them back transposed: lane j then
        // scans column j's 32 rows in row order, keeping the top KT with the
        // lowest row winning ties (strict >) -- independent per lane, no
        // cross-lane chains.  The four warps' candidates go to a merge area
        // (double-buffered by unit); warp 2 merges them, one column per lane,
        // and writes the tile's top-KT.  The hand-offs are mbarriers with
        // bounded waits, never an unbounded named barrier.
        const int cols = min(bt, p.M - m0);
        const int b2 = ti & 1, use2 = ti >> 1;
        float* mv = mval + b2 * marea;
        int* mi = midx + b2 * marea;
        uint32_t* ts = tscr + q * TSCR_WORDS;
        if (!mbar_wait(&mempty[b2], (use2 & 1) ^ 1, lim)) {
          fail(ERR_TIMEOUT_EPILOGUE);
          break;
        }
        if (bt <= 32) {
          // few token columns (verify / AR): KT rounds of a warp max (redux.sync
          // on the keys) per column, lowest row winning ties -- same result
          for (int c = 0; c < cols; c += 16) {
            float v[16];
            tmem_ld16(tacc + c, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              uint32_t key = n_ok ? float_key(v[j]) : 0u;
#pragma unroll
              for (int r = 0; r < KT; ++r) {
                const uint32_t mx = __reduce_max_sync(0xffffffffu, key);
                const uint32_t win = __ballot_sync(0xffffffffu, key == mx && mx != 0u);
                const int wl = win ? __ffs(win) - 1 : 0;
                if (lane == 0) {
                  const int o = (q * bt + c + j) * KT + r;
                  mv[o] = mx ? key_float(mx) : -INFINITY;
                  mi[o] = mx ? n0 + q * 32 + wl : 0x7fffffff;
                }
                if (lane == wl && win) key = 0u;
              }
            }
          }
        }
        for (int c0 = 0; bt > 32 && c0 < cols; c0 += 32) {
          float v[32];
          tmem_ld16(tacc + c0, v);
          tmem_ld16(tacc + c0 + 16, v + 16);   // accumulators span >= 32 columns, a multiple of 32
#pragma unroll
          for (int j = 0; j < 32; ++j) ts[lane * 33 + j] = n_ok ? float_key(v[j]) : 0u;
          __syncwarp();
          uint32_t bk[KT];
          int br[KT];
#pragma unroll
          for (int z = 0; z < KT; ++z) {
            bk[z] = 0u;
            br[z] = 0;
          }
#pragma unroll 8
          for (int r = 0; r < 32; ++r) {
            uint32_t kk = ts[r * 33 + lane];
            int rr = r;
#pragma unroll
            for (int z = 0; z < KT; ++z) {
              if (kk > bk[z]) {
                const uint32_t tk = bk[z];
                const int tr = br[z];
                bk[z] = kk;
                br[z] = rr;
                kk = tk;
                rr = tr;
              }
            }
          }
          __syncwarp();   // the scratch is rewritten by the next chunk
          if (c0 + lane < cols) {
#pragma unroll
            for (int z = 0; z < KT; ++z) {
              const int o = (q * bt + c0 + lane) * KT + z;
              mv[o] = bk[z] ? key_float(bk[z]) : -INFINITY;
              mi[o] = bk[z] ? n0 + q * 32 + br[z] : 0x7fffffff;
            }
          }
        }
        // TMEM is free once every lane's loads are done
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&acce[a]);
          mbar_arrive(&mfull[b2]);   // release semantics publish the candidates
        }
        if (warp == 2) {
          if (!mbar_wait(&mfull[b2], use2 & 1, lim)) {
            fail(ERR_TIMEOUT_EPILOGUE);
            break;
          }
          for (int j = lane; j < cols; j += 32) {
            float bv[KT];
            int bi[KT];
#pragma unroll
            for (int r = 0; r < KT; ++r) {
              bv[r] = -INFINITY;
              bi[r] = 0x7fffffff;
            }
            for (int w = 0; w < 4; ++w) {
#pragma unroll
              for (int r = 0; r < KT; ++r) {
                float x = mv[(w * bt + j) * KT + r];
                int xi = mi[(w * bt + j) * KT + r];
#pragma unroll
                for (int z = 0; z < KT; ++z) {
                  if (x > bv[z] || (x == bv[z] && xi < bi[z])) {
                    const float t1 = bv[z];
                    const int t2 = bi[z];
                    bv[z] = x;
                    bi[z] = xi;
                    x = t1;
                    xi = t2;
                  }
                }
              }
            }
            const size_t o = (static_cast<size_t>(m0 + j) * p.ntiles + u.n_t) * KT;
#pragma unroll
            for (int r = 0; r < KT; ++r) {
              p.topv[o + r] = bv[r];
              p.topi[o + r] = bi[r] < p.N ? bi[r] : 0x7fffffff;
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&mempty[b2]);
        }
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  if (MODE == 0 && p.tp > 0) {
    // this thread's partial stores are visible (to peers' loads, or as peer
    // stores) before the flags go up
    if (p.tp_pull) __threadfence();
    else __threadfence_system();
  }
  __syncthreads();
  if (MODE == 0 && p.tp > 0 && threadIdx.x == 0) {
    // the last CTA to finish publishes the exchange on every rank
    const unsigned int t = atomicAdd(p.tp_ticket, 1u);
    if (t == gridDim.x - 1) {
      *p.tp_ticket = 0;
      __threadfence_system();
      const int64_t e = *p.tp_epoch;
      for (int r = 0; r < p.tp; ++r) {
        int64_t* f = p.tp_flags[r] + static_cast<size_t>(p.tp_x) * p.tp + p.tp_rank;
        asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(f), "l"(e) : "memory");
      }
    }
  }
  if (threadIdx.x == 32) {
    // every MMA this thread issued has retired before TMEM is released
    umma_commit(done);
    if (!mbar_wait(done, 0, lim)) set_error(p.status, ERR_TIMEOUT_MMA);
  }
  if (threadIdx.x == 0 && flags[0]) {
    // drain TMA loads that were issued but never consumed, so no copy lands
    // in shared memory after the CTA has exited
    for (int i = flags[2]; i < flags[1]; ++i) mbar_wait(&full[i % stages], (i / stages) & 1, lim);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, tmem_cols);
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static void init_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
}

void make_tmap_bf16_2d(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                       uint32_t box_inner, uint32_t box_outer) {
  init_encode();
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((row_stride_elems * 2) % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
}

void make_tmap_bf16_3d(CUtensorMap* tm, const void* base, const uint64_t dims[3], const uint64_t strides_elems[2],
                       const uint32_t box[3]) {
  init_encode();
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  for (int i = 0; i < 2; ++i)
    if ((strides_elems[i] * 2) % 16 != 0) throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  if (box[0] * 2 > 128) throw std::runtime_error("TMA box row exceeds the 128-byte swizzle span");
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {strides_elems[0] * 2, strides_elems[1] * 2};
  cuuint32_t bx[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), d, st, bx, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (3d) failed: " + std::to_string(int(r)));
}

// Pipeline depth.  Measured on B200: two co-resident CTAs per SM (~110 KB of
// shared memory each) stream weights at 85-92% of HBM bandwidth where one CTA
// with a 12-stage pipeline reaches ~50%, so small token tiles use the 110 KB
// budget whenever it still holds >= 4 stages; large tiles (compute-heavy) use
// one CTA with ~220 KB.  ``reserve`` bytes (the top-k merge areas) come off
// the budget.  D3D_GEMM_SMEM_KB / D3D_GEMM_MAX_STAGES override.
static int stages_for(int bt, int reserve) {
  static const int env_kb = [] {
    const char* e = std::getenv("D3D_GEMM_SMEM_KB");
    return e ? std::atoi(e) : 0;
  }();
  static const int max_stages = [] {
    const char* e = std::getenv("D3D_GEMM_MAX_STAGES");
    return e ? std::atoi(e) : 16;
  }();
  const int stage_bytes = A_TILE_BYTES + bt * GBK * 2;
  const int small = 110 * 1024 - reserve;
  const int budget = env_kb > 0 ? env_kb * 1024 - reserve : (small / stage_bytes >= 4 ? small : 220 * 1024 - reserve);
  int s = budget / stage_bytes;
  if (s > max_stages) s = max_stages;
  return s < 2 ? 2 : s;
}

int gemm_stages(int bt) { return stages_for(bt, 0); }

static size_t smem_bytes(int bt, int stages, int reserve) {
  const int stage_bytes = A_TILE_BYTES + bt * GBK * 2;
  return 1024 + static_cast<size_t>(stages) * stage_bytes + reserve + (2 * stages + 10) * 8 + 48;
}

size_t gemm_smem_bytes(int bt, int stages) { return smem_bytes(bt, stages, 0); }

int gemm_ctas_per_sm(int bt) { return gemm_smem_bytes(bt, gemm_stages(bt)) <= 114 * 1024 ? 2 : 1; }

static int num_sms() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

template <int MODE, int KT>
static void launch_mode(const CUtensorMap& tw, const CUtensorMap& tx, GemmParams p, int units, size_t smem,
                        cudaStream_t st) {
  static bool attr_set = false;  // per template instance
  if (!attr_set) {
    cudaFuncSetAttribute(gemm_tn_kernel<MODE, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    attr_set = true;
  }
  // persistent grid (one CTA per resident slot) unless D3D_GEMM_GRID=units
  // asks for one CTA per work unit
  static const bool per_unit = [] {
    const char* e = std::getenv("D3D_GEMM_GRID");
    return e && std::string(e) == "units";
  }();
  const int per_sm = smem <= 114 * 1024 ? 2 : 1;
  int grid = per_unit ? units : num_sms() * per_sm;
  if (grid > units) grid = units;
  launch_pdl(gemm_tn_kernel<MODE, KT>, dim3(grid), dim3(GEMM_THREADS), smem, st, tw, tx, p);
}

void gemm_launch(const GemmArgs& a, cudaStream_t stream) {
  if (a.bt < 16 || a.bt > 512 || a.bt % 16 || (a.bt > 256 && a.bt % 32))
    throw std::runtime_error("gemm: bt must be a multiple of 16 in [16,256] or of 32 in (256,512]");
  if (a.K % 8) throw std::runtime_error("gemm: K must be a multiple of 8");
  const int nkb = (a.K + GBK - 1) / GBK;
  if (a.splits < 1 || a.splits > nkb || a.splits > 16)
    throw std::runtime_error("gemm: splits must be in [1, min(16, K/64)]");
  if (a.mode != 0 && a.mode != 4 && a.splits != 1) throw std::runtime_error("gemm: split-K needs fp32 partial mode");
  if (a.mode == 4 && (!a.fin_x || !a.fin_sumsq || !a.fin_ticket || a.out_f32 == nullptr))
    throw std::runtime_error("gemm: mode 4 needs partials, residual, sums-of-squares and tickets");
  CUtensorMap tw, tx;
  if (a.w_packed) {
    const uint64_t rows = static_cast<uint64_t>((a.N + GBN - 1) / GBN) * nkb * GBN;
    make_tmap_bf16_2d(&tw, a.w, GBK, rows, GBK, GBK, GBN);
  } else {
    make_tmap_bf16_2d(&tw, a.w, a.K, a.N, a.ldw, GBK, GBN);
  }
  make_tmap_bf16_2d(&tx, a.x, a.K, a.M, a.ldx, GBK, a.bt > 256 ? a.bt / 2 : a.bt);
  const int kt = a.mode == 2 ? (a.topk <= 1 ? 1 : (a.topk <= 2 ? 2 : 4)) : 1;
  if (a.mode == 2 && a.topk > 4) throw std::runtime_error("gemm: fused top-k supports k <= 4");
  const int reserve = a.mode == 2 ? 2 * 4 * a.bt * kt * 8 + (a.bt > 32 ? 4 * TSCR_WORDS * 4 : 0) : 0;
  GemmParams p{};
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.out_f32 = a.out_f32;
  p.out_bf16 = a.out_bf16;
  p.ldc = a.ldc;
  p.residual = a.residual;
  p.ldr = a.ldr;
  p.topv = a.topv;
  p.topi = a.topi;
  p.bt = a.bt;
  p.splits = a.splits;
  p.w_packed = a.w_packed;
  p.stages = stages_for(a.bt, reserve);
  p.status = a.status;
  p.timeout_ns = a.timeout_ns;
  p.tp = a.tp;
  p.fin_x = a.fin_x;
  p.fin_ldx = a.fin_ldx;
  p.fin_sumsq = a.fin_sumsq;
  p.fin_ticket = a.fin_ticket;
  if (a.tp > 0 && a.mode == 4) throw std::runtime_error("gemm: mode 4 is not tensor-parallel");
  if (a.tp > 0) {
    if (a.mode != 0 || a.tp > 8 || !a.tp_epoch || !a.tp_ticket)
      throw std::runtime_error("gemm: tensor-parallel push needs mode 0, tp <= 8, epoch and ticket");
    p.tp_rank = a.tp_rank;
    p.tp_x = a.tp_x;
    p.tp_pull = a.tp_pull;
    for (int r = 0; r < a.tp; ++r) {
      p.tp_out[r] = a.tp_out[r];
      p.tp_flags[r] = a.tp_flags[r];
    }
    p.tp_epoch = a.tp_epoch;
    p.tp_ticket = a.tp_ticket;
  }
  const int ntn = (a.N + GBN - 1) / GBN;
  p.ntiles = ntn;
  const int units = ntn * ((a.M + a.bt - 1) / a.bt) * a.splits;
  const size_t smem = smem_bytes(a.bt, p.stages, reserve);
  if (smem > 232448) throw std::runtime_error("gemm: shared memory budget exceeded");
  switch (a.mode) {
    case 0: launch_mode<0, 1>(tw, tx, p, units, smem, stream); break;
    case 1: launch_mode<1, 1>(tw, tx, p, units, smem, stream); break;
    case 2:
      if (kt == 1) launch_mode<2, 1>(tw, tx, p, units, smem, stream);
      else if (kt == 2) launch_mode<2, 2>(tw, tx, p, units, smem, stream);
      else launch_mode<2, 4>(tw, tx, p, units, smem, stream);
      break;
    case 3:
      if (a.N % GBN) throw std::runtime_error("gemm: SwiGLU epilogue needs 2*I to be a multiple of 128");
      launch_mode<3, 1>(tw, tx, p, units, smem, stream);
      break;
    case 4: launch_mode<4, 1>(tw, tx, p, units, smem, stream); break;
    default: throw std::runtime_error("gemm: bad mode");
  }
}

}  // namespace d3d
