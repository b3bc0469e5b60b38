// Host-side interface of the tcgen05 GEMM (raw pointers; no torch headers so
// the .cu files compile quickly and can be linked into any host program).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace d3d {

struct GemmParams {
  int M, N, K;
  float* out_f32;
  __nv_bfloat16* out_bf16;
  int ldc;
  const __nv_bfloat16* residual;
  int ldr;
  float* topv;
  int* topi;
  int ntiles;
  int bt;
  int splits;
  int stages;
  int w_packed;
  int* status;
  unsigned long long timeout_ns;
  // tensor-parallel push (MODE 0): partials of split s go to slot (tp_rank * splits + s)
  // of every rank's exchange buffer; the last CTA raises flags[j][x * tp + tp_rank] = *epoch
  int tp, tp_rank, tp_x, tp_pull;
  float* tp_out[8];
  int64_t* tp_flags[8];
  int64_t* tp_epoch;
  unsigned int* tp_ticket;
  // MODE 4 (split-K partials + in-kernel finalize): the last unit of an output
  // tile to finish reduces the splits in split order, adds them to the bf16
  // residual fin_x (in place) and writes the tile's per-row sum of squares
  __nv_bfloat16* fin_x;
  int fin_ldx;
  float* fin_sumsq;          // [ceil(N/128)][M]
  unsigned int* fin_ticket;  // [ceil(N/128) * ceil(M/bt)], zero, reset after use
};

struct GemmArgs {
  const __nv_bfloat16* x;  // [M, K] activations (row stride ldx elements)
  const __nv_bfloat16* w;  // [N, K] weights (row stride ldw elements)
  int M, N, K, ldx, ldw;
  int mode;      // 0 fp32 split-K partials, 1 bf16 (+residual), 2 fused top-k, 3 SwiGLU (interleaved gate|up),
                 // 4 fp32 partials + in-kernel split reduce into a residual (+ row sums of squares)
  int splits;    // split-K factor (mode 0 only)
  int bt;        // token tile (MMA N), multiple of 16 in [16, 256]
  int topk;      // mode 2: k <= 4
  float* out_f32;              // mode 0: [splits, M, N]
  __nv_bfloat16* out_bf16;     // mode 1: [M, ldc]; mode 3: [M, ldc] with N/2 columns
  int ldc;
  const __nv_bfloat16* residual;  // mode 1 optional [M, ldr]
  int ldr;
  float* topv;                 // mode 2: [M, ceil(N/128), kt]
  int* topi;
  int* status;                 // device error word (may be null)
  unsigned long long timeout_ns;
  int w_packed;                // w is in the packed tile layout (see pack_weight)
  // tensor-parallel exchange (mode 0 only; tp = 0 disables): see GemmParams;
  // tp_pull = 1 stores only this rank's slot (peers read it) instead of pushing
  int tp, tp_rank, tp_x, tp_pull;
  float* tp_out[8];
  int64_t* tp_flags[8];
  int64_t* tp_epoch;
  unsigned int* tp_ticket;
  __nv_bfloat16* fin_x;        // mode 4: residual [M, fin_ldx] updated in place
  int fin_ldx;
  float* fin_sumsq;            // mode 4: [ceil(N/128)][M] per-tile row sums of squares
  unsigned int* fin_ticket;    // mode 4: [ceil(N/128) * ceil(M/bt)] zeroed counters
};

void gemm_launch(const GemmArgs& a, cudaStream_t stream);
int gemm_stages(int bt);
int gemm_ctas_per_sm(int bt);
size_t gemm_smem_bytes(int bt, int stages);
void make_tmap_bf16_2d(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                       uint32_t box_inner, uint32_t box_outer);
// 3-D bf16 tensor map with 128-byte swizzle: dims {d0, d1, d2} (d0 contiguous),
// strides of d1 and d2 in elements, box {b0, b1, b2} (b0 * 2 bytes <= 128).
void make_tmap_bf16_3d(CUtensorMap* tm, const void* base, const uint64_t dims[3], const uint64_t strides_elems[2],
                       const uint32_t box[3]);

}  // namespace d3d
