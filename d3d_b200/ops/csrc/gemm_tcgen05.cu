// Weight-stationary tcgen05 GEMM for sm_100a:  Y[M, N] = X[M, K] · W[N, K]^T.
//
// Decode-time matmuls have few tokens (M = 1..1088) against large weights, so
// the tile is laid out "swap-AB": the 128-row MMA M dimension runs over weight
// rows (output features) and the MMA N dimension over tokens: ``bt`` = 16..256
// (a multiple of 16) in one MMA, or up to 512 (a multiple of 32) as two MMAs
// of bt/2 columns each, so one CTA can reuse its weight tile for 512 tokens
// (TMEM holds 512 fp32 columns).  One CTA owns a 128 x bt output tile and a contiguous
// range of K blocks (split-K chosen by the host from the weight shape alone,
// so the fp32 reduction order of every output element is independent of M —
// the property greedy token identity between AR and speculative decoding
// rests on).
//
// Per CTA (128 threads):
//   warp 0 lane 0  TMA producer: W tile [128 x 64] and X tile [bt x 64] per
//                  stage, 128-byte swizzle, mbarrier complete_tx;
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma (K = 16 each) per stage into a
//                  TMEM accumulator (128 lanes x bt fp32 columns), then
//                  tcgen05.commit to free the stage;
//   all 4 warps    epilogue: tcgen05.ld 32x32b (warp w owns TMEM lanes
//                  32w..32w+31 = output rows) and one of three stores:
//                  MODE 0  fp32 split-K partials  P[split][M][N]
//                  MODE 1  bf16 Y (+ bf16 residual, rounded like two bf16 ops)
//                  MODE 2  per-tile top-KT (value, index) over the 128 rows,
//                          for LM-head argmax / top-k without storing logits.
// Every mbarrier wait is bounded; a timeout records an error code in
// ``status`` and the kernel leaves its loop.  Launched with programmatic
// dependent launch: the producer streams the first pipeline stages of weights
// before griddepcontrol.wait, overlapping the previous kernel's tail.
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

template <int MODE, int KT>
__global__ void __launch_bounds__(128, 2)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bt = p.bt;
  const int stages = p.stages;
  const int stage_bytes = A_TILE_BYTES + bt * GBK * 2;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * stage_bytes);
  uint64_t* empty = full + stages;
  uint64_t* accb = empty + stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] issued, [1] consumed, [2] failed

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * GBN, m0 = blockIdx.y * bt;
  const int nkb = (p.K + GBK - 1) / GBK;
  const int split = blockIdx.z, nsplit = gridDim.z;
  const int kb0 = (nkb * split) / nsplit, kb1 = (nkb * (split + 1)) / nsplit;
  const int nk = kb1 - kb0;
  const int nsub = bt > 256 ? 2 : 1;      // MMAs per K step
  const int sub = bt / nsub;              // tokens per MMA (multiple of 16)
  const uint32_t tmem_cols = bt <= 32 ? 32 : (bt <= 64 ? 64 : (bt <= 128 ? 128 : (bt <= 256 ? 256 : 512)));
  const uint64_t lim = p.timeout_ns;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    flags[0] = flags[1] = flags[2] = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmW);
    prefetch_tensormap(&tmX);
    griddep_launch();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_w = policy_evict_first();  // weights stream through L2 once
    auto load_w = [&](int i, int s) {
      uint8_t* sa = smem + s * stage_bytes;
      if (p.w_packed)  // contiguous 16 KB tiles: [N/128][K/64][128][64]
        tma_load_2d_hint(sa, &tmW, &full[s], 0, (blockIdx.x * nkb + kb0 + i) * GBN, pol_w);
      else
        tma_load_2d_hint(sa, &tmW, &full[s], (kb0 + i) * GBK, n0, pol_w);
    };
    auto load_x = [&](int i, int s) {
      uint8_t* sb = smem + s * stage_bytes + A_TILE_BYTES;
      for (int u = 0; u < nsub; ++u)
        tma_load_2d(sb + u * sub * GBK * 2, &tmX, &full[s], (kb0 + i) * GBK, m0 + u * sub);
    };
    // weights do not depend on earlier kernels: fill the pipeline before the
    // grid dependency resolves, then add the activation tiles
    const int pre = nk < stages ? nk : stages;
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], stage_bytes);
      load_w(i, i);
    }
    griddep_wait();
    for (int i = 0; i < pre; ++i) load_x(i, i);
    int i = pre;
    for (; i < nk; ++i) {
      const int s = i % stages;
      const uint32_t ph = (i / stages) & 1;
      if (!mbar_wait(&empty[s], ph ^ 1, lim)) {
        set_error(p.status, ERR_TIMEOUT_PRODUCER);
        break;
      }
      mbar_arrive_expect_tx(&full[s], stage_bytes);
      load_w(i, s);
      load_x(i, s);
    }
    flags[0] = i;
  } else if (warp == 1 && lane == 0) {
    // ----------------------------------------------------------- MMA issuer
    const uint32_t idesc = idesc_bf16_f32(GBN, sub);
    int i = 0;
    for (; i < nk; ++i) {
      const int s = i % stages;
      const uint32_t ph = (i / stages) & 1;
      if (!mbar_wait(&full[s], ph, lim)) {
        set_error(p.status, ERR_TIMEOUT_MMA);
        flags[2] = 1;
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + s * stage_bytes);
      const uint64_t ad = sdesc_kmajor_sw128(sa);
      const uint64_t bd = sdesc_kmajor_sw128(sa + A_TILE_BYTES);
#pragma unroll
      for (int kk = 0; kk < GBK / 16; ++kk) {
        // +32 bytes along K inside the swizzle atom = +2 in the >>4 address field
        umma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
        if (nsub == 2) {
          const uint64_t bd2 = sdesc_kmajor_sw128(sa + A_TILE_BYTES + sub * GBK * 2);
          umma_bf16(tmem + sub, ad + 2 * kk, bd2 + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
        }
      }
      umma_commit(&empty[s]);
    }
    flags[1] = i;
    umma_commit(accb);
  }
  __syncwarp();
  griddep_wait();  // outputs may still be read by the previous kernel until it completes

  // -------------------------------------------------------------- epilogue
  bool ok = mbar_wait(accb, 0, lim);
  if (!ok) set_error(p.status, ERR_TIMEOUT_EPILOGUE);
  __syncwarp();
  tc_fence_after();
  const int row = warp * 32 + lane;
  const int n = n0 + row;
  const uint32_t t_row = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const bool n_ok = n < p.N;
  const bool live = ok && nk > 0;

  for (int c = 0; c < (MODE == 2 ? 0 : bt); c += 16) {
    float v[16];
    tmem_ld16(t_row + c, v);
    if (!live) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = 0.f;
    }
    if constexpr (MODE == 0) {
      if (n_ok) {
        float* base = p.out_f32 + static_cast<size_t>(split) * p.M * p.N;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c + j;
          if (m < p.M) base[static_cast<size_t>(m) * p.N + n] = v[j];
        }
      }
    } else if constexpr (MODE == 1) {
      if (n_ok) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c + j;
          if (m < p.M) {
            float y = v[j];
            if (p.residual) y = bf16r(y) + __bfloat162float(p.residual[static_cast<size_t>(m) * p.ldr + n]);
            p.out_bf16[static_cast<size_t>(m) * p.ldc + n] = __float2bfloat16(y);
          }
        }
      }
    }
  }
  if constexpr (MODE == 2) {
    // ------------------------------------------------- MODE 2: per-tile top-KT
    // The accumulator is copied, transposed, into the idle pipeline stages
    // ([column][129] floats: the padding keeps both the row-wise writes and
    // the column-wise scans bank-conflict free); then every thread scans
    // whole token columns on its own, so there is no cross-lane dependency
    // chain.  Columns are processed in groups that fit the stage area.
    float* tile = reinterpret_cast<float*>(smem);
    constexpr int LDT = GBN + 1;
    const int avail = stages * stage_bytes / (LDT * 4);
    const int group = avail >= bt ? bt : (avail / 16) * 16;
    for (int g0 = 0; g0 < bt; g0 += group) {
      const int g1 = min(bt, g0 + group);
      for (int c = g0; c < g1; c += 16) {
        float v[16];
        tmem_ld16(t_row + c, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) tile[(c - g0 + j) * LDT + row] = (live && n_ok) ? v[j] : -INFINITY;
      }
      __syncthreads();
      for (int j = g0 + threadIdx.x; j < g1; j += blockDim.x) {
        const int m = m0 + j;
        if (m >= p.M) continue;
        const float* col = tile + (j - g0) * LDT;
        float bv[KT];
        int bi[KT];
#pragma unroll
        for (int r = 0; r < KT; ++r) {
          bv[r] = -INFINITY;
          bi[r] = 0x7fffffff;
        }
#pragma unroll 8
        for (int rr = 0; rr < GBN; ++rr) {
          float x = col[rr];
          if (x > bv[KT - 1]) {   // strict: equal values keep the lower row
            int xi = n0 + rr;
#pragma unroll
            for (int q = 0; q < KT; ++q) {
              if (x > bv[q]) {
                const float t1 = bv[q];
                const int t2 = bi[q];
                bv[q] = x;
                bi[q] = xi;
                x = t1;
                xi = t2;
              }
            }
          }
        }
        const size_t o = (static_cast<size_t>(m) * p.ntiles + blockIdx.x) * KT;
#pragma unroll
        for (int r = 0; r < KT; ++r) {
          p.topv[o + r] = bv[r];
          p.topi[o + r] = bi[r] < p.N ? bi[r] : 0x7fffffff;
        }
      }
      __syncthreads();
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && flags[2]) {
    // drain TMA loads that were issued but never consumed, so no copy lands
    // in shared memory after the CTA has exited
    for (int i = flags[1]; i < flags[0]; ++i) mbar_wait(&full[i % stages], (i / stages) & 1, lim);
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, tmem_cols);
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

// Pipeline depth.  Measured on B200: two co-resident CTAs per SM (~110 KB of
// shared memory each) stream weights at 85-92% of HBM bandwidth where one CTA
// with a 12-stage pipeline reaches ~50%, so small token tiles use the 110 KB
// budget whenever it still holds >= 4 stages; large tiles (compute-heavy) use
// one CTA with ~220 KB.  D3D_GEMM_SMEM_KB / D3D_GEMM_MAX_STAGES override.
int gemm_stages(int bt) {
  static const int env_kb = [] {
    const char* e = std::getenv("D3D_GEMM_SMEM_KB");
    return e ? std::atoi(e) : 0;
  }();
  static const int max_stages = [] {
    const char* e = std::getenv("D3D_GEMM_MAX_STAGES");
    return e ? std::atoi(e) : 16;
  }();
  const int stage_bytes = A_TILE_BYTES + bt * GBK * 2;
  const int budget_kb = env_kb > 0 ? env_kb : ((110 * 1024) / stage_bytes >= 4 ? 110 : 220);
  int s = (budget_kb * 1024) / stage_bytes;
  if (s > max_stages) s = max_stages;
  return s < 2 ? 2 : s;
}

int gemm_ctas_per_sm(int bt) { return gemm_smem_bytes(bt, gemm_stages(bt)) <= 114 * 1024 ? 2 : 1; }

size_t gemm_smem_bytes(int bt, int stages) {
  const int stage_bytes = A_TILE_BYTES + bt * GBK * 2;
  return 1024 + static_cast<size_t>(stages) * stage_bytes + (2 * stages + 1) * 8 + 32;
}

template <int MODE, int KT>
static void launch_mode(const CUtensorMap& tw, const CUtensorMap& tx, GemmParams p, dim3 grid, size_t smem,
                        cudaStream_t st) {
  static bool attr_set = false;  // per template instance
  if (!attr_set) {
    cudaFuncSetAttribute(gemm_tn_kernel<MODE, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    attr_set = true;
  }
  launch_pdl(gemm_tn_kernel<MODE, KT>, grid, dim3(128), smem, st, tw, tx, p);
}

void gemm_launch(const GemmArgs& a, cudaStream_t stream) {
  if (a.bt < 16 || a.bt > 512 || a.bt % 16 || (a.bt > 256 && a.bt % 32))
    throw std::runtime_error("gemm: bt must be a multiple of 16 in [16,256] or of 32 in (256,512]");
  if (a.K % 8) throw std::runtime_error("gemm: K must be a multiple of 8");
  const int nkb = (a.K + GBK - 1) / GBK;
  if (a.splits < 1 || a.splits > nkb || a.splits > 16)
    throw std::runtime_error("gemm: splits must be in [1, min(16, K/64)]");
  if (a.mode != 0 && a.splits != 1) throw std::runtime_error("gemm: split-K needs fp32 partial mode");
  CUtensorMap tw, tx;
  if (a.w_packed) {
    const uint64_t rows = static_cast<uint64_t>((a.N + GBN - 1) / GBN) * nkb * GBN;
    make_tmap_bf16_2d(&tw, a.w, GBK, rows, GBK, GBK, GBN);
  } else {
    make_tmap_bf16_2d(&tw, a.w, a.K, a.N, a.ldw, GBK, GBN);
  }
  make_tmap_bf16_2d(&tx, a.x, a.K, a.M, a.ldx, GBK, a.bt > 256 ? a.bt / 2 : a.bt);
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
  p.w_packed = a.w_packed;
  p.stages = gemm_stages(a.bt);
  p.status = a.status;
  p.timeout_ns = a.timeout_ns;
  const int ntn = (a.N + GBN - 1) / GBN;
  p.ntiles = ntn;
  dim3 grid(ntn, (a.M + a.bt - 1) / a.bt, a.splits);
  const size_t smem = gemm_smem_bytes(a.bt, p.stages);
  switch (a.mode) {
    case 0: launch_mode<0, 1>(tw, tx, p, grid, smem, stream); break;
    case 1: launch_mode<1, 1>(tw, tx, p, grid, smem, stream); break;
    case 2:
      if (a.topk == 1) launch_mode<2, 1>(tw, tx, p, grid, smem, stream);
      else if (a.topk == 2) launch_mode<2, 2>(tw, tx, p, grid, smem, stream);
      else if (a.topk <= 4) launch_mode<2, 4>(tw, tx, p, grid, smem, stream);
      else throw std::runtime_error("gemm: fused top-k supports k <= 4");
      break;
    default: throw std::runtime_error("gemm: bad mode");
  }
}

}  // namespace d3d
