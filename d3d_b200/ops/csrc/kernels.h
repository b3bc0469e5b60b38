// Host-side prototypes of the non-GEMM kernels (raw pointers, no torch).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace d3d {

void add_rmsnorm(const float* part, int nsplit, __nv_bfloat16* residual, const __nv_bfloat16* w, __nv_bfloat16* out,
                 int M, int N, float eps, cudaStream_t st);

void swiglu(const float* part, int nsplit, __nv_bfloat16* h, int M, int I, bool interleaved, cudaStream_t st);

struct QkvRopeArgs {
  const float* part;        // [nsplit][M][(Hq+2Hkv)*D] fp32 partials, or null
  const __nv_bfloat16* y;   // bf16 qkv when part is null
  int nsplit, M, Hq, Hkv, head_dim;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const float* inv_freq;    // [D/2]
  const int64_t* positions;  // [M]
  const int64_t* slots;      // [M] physical KV slot (page * page_size + offset)
  __nv_bfloat16* q_out;     // [M][Hq][D]
  __nv_bfloat16* k_cache;   // [slots][Hkv][D]
  __nv_bfloat16* v_cache;
  float eps;
  long long num_slots;      // KV cache rows (debug bounds checks)
  int* status;              // error word (debug bounds checks; may be null)
  // optional RMSNorm row scale of the GEMM input (the norm weight folded into
  // the qkv weight): r[m] = rsqrt(sum_t rsq[t][m] / rsq_n + eps), rsq [rsq_tiles][M]
  const float* rsq;
  int rsq_tiles, rsq_n;
};
void qkv_rope_kv(const QkvRopeArgs& a, cudaStream_t st);

// SwiGLU of split-K partials of an interleaved gate|up weight whose input
// RMSNorm weight is folded in: h = silu(r*g) * (r*u), r from per-tile sums of
// squares rsq [rsq_tiles][M] of the GEMM input (n elements per row).
void swiglu_rowscale(const float* part, int nsplit, __nv_bfloat16* h, int M, int I, const float* rsq, int rsq_tiles,
                     int rsq_n, float eps, cudaStream_t st);
// x [M, N] (bf16, in place) += split-K partials part [nsplit][M][N] (split order,
// rounded like two bf16 ops) and per-tile row sums of squares into sumsq
// [ceil(N/128)][M]: the stand-alone form of the GEMM's in-kernel reduction.
void residual_split_reduce(const float* part, int nsplit, __nv_bfloat16* x, int M, int N, float* sumsq,
                           cudaStream_t st);
// Per-tile (128 columns) row sums of squares of x [M, N] into out [ceil(N/128)][M].
void tile_sumsq(const __nv_bfloat16* x, int M, int N, float* out, cudaStream_t st);

void embed(const int64_t* ids, const __nv_bfloat16* table, const __nv_bfloat16* cond, const unsigned char* cond_rows,
           int q_len, __nv_bfloat16* out, int M, int H, cudaStream_t st, long long vocab = 0, int* status = nullptr);

void topk_merge(const float* tv, const int* ti, int ntiles, int kt, int k, float* ov, int64_t* oi, int M,
                cudaStream_t st);

void greedy_accept(const int64_t* blocks, const int64_t* post, int B, int K, int64_t* commit, int64_t* corr,
                   const __nv_bfloat16* hidden, __nv_bfloat16* hid_out, int H, cudaStream_t st);

struct AttnArgs {
  const __nv_bfloat16* q;   // [T][Hq][D]
  const __nv_bfloat16* k_cache;  // [slots][Hkv][D]
  const __nv_bfloat16* v_cache;
  const int* block_table;   // [B][bt_stride] page ids
  int bt_stride;
  const int* rows;          // [T][3] (lim, lo, hi) absolute slots
  const int* kv_end;        // [B] keys beyond are never read
  int B, q_len, Hq, Hkv, head_dim, page_size;
  float scale;
  int chunk;                // keys per split (multiple of 64); one split when >= max kv
  int n_chunks;
  int invariant;            // batch-invariant path: same kernel whatever q_len (target decode)
  float* part_o;            // [n_chunks][T][Hq][D]
  float* part_ml;           // [n_chunks][T][Hq][2]
  __nv_bfloat16* out;       // [T][Hq][D]
  long long num_slots;      // KV cache rows (debug bounds checks)
  int* status;              // error word (debug bounds checks; may be null)
};
void attention(const AttnArgs& a, cudaStream_t st);        // cluster kernel (no partial buffers)
cudaError_t attention_split(const AttnArgs& a, cudaStream_t st);  // split-KV + combine (uses part_o / part_ml)
cudaError_t attention_combine(const AttnArgs& a, cudaStream_t st);  // merge part_o / part_ml chunks into out
bool attention_tc_supported(const AttnArgs& a);              // shapes the tcgen05 kernel serves
void attention_tc(const AttnArgs& a, cudaStream_t st);       // tcgen05/TMEM kernel (+ combine when split)

// ---- training kernels (train_kernels.cu)
void kl_ce_stats(const float* zt, const float* zs, int N, int C, int ldz, int v0, const int64_t* target, float* st,
                 cudaStream_t s);
void kl_ce_grad(const float* zt, const float* zs, int N, int C, int ldz, int v0, const int64_t* target,
                const float* lse_t, const float* lse_s, const float* w_kl, const float* w_ce, __nv_bfloat16* dz,
                int ld_dz, __nv_bfloat16* dzT, int ld_dzT, cudaStream_t s);
void adamw(float* p, const float* g, float* m, float* v, __nv_bfloat16* out, size_t n, float lr, float b1, float b2,
           float eps, float wd, int step, float grad_scale, cudaStream_t s);
void sumsq(const float* x, size_t n, float* out, cudaStream_t s);

}  // namespace d3d

namespace d3d {
// ---- cross-GPU handoff (handoff.cu)
void handoff_put(const void* src, void* dst_peer, size_t nbytes, int64_t* flag_peer, int64_t seq,
                 unsigned int* ticket, cudaStream_t st);
void handoff_wait(const int64_t* flag, int64_t seq, const void* src, void* dst, size_t nbytes, int* status,
                  unsigned long long limit_ns, cudaStream_t st);
void accept_send(const int64_t* blocks, const int64_t* post, int B, int K, const __nv_bfloat16* hidden, int H,
                 int64_t* out_peer, __nv_bfloat16* hid_peer, int64_t* flag_peer, int64_t seq, const int* gate,
                 cudaStream_t st);
constexpr int ARM_MAX_SRC = 8;
constexpr int SEL_MAX_ROWS = 64;
struct ArmArgs {
  const int64_t* flag[ARM_MAX_SRC];  // source inbox flags
  const int64_t* msg[ARM_MAX_SRC];   // the slot message seq lands in
  int64_t* head[ARM_MAX_SRC];        // pinned host copy of each message's first head_words
  int64_t seq[ARM_MAX_SRC];
  int row0[ARM_MAX_SRC];             // first merged row of each source
  int nb[ARM_MAX_SRC];               // rows expected from each source
  int n_src, K, head_words, page, bt_stride;
  const int64_t* tab;                // [B] expected sequence ids | [B] KV slots reserved per row
  const int32_t* block_table;
  const int64_t* seq_rows;
  int64_t scratch_slot;
  int64_t* ids;
  int64_t* pos;
  int64_t* slots;
  int32_t* rows;
  int32_t* kv_end;
  int* gate;
  int* status;                       // pinned [n_src + 1]
  unsigned long long limit_ns;
  // tensor-parallel targets: rank 0 (role 1) decides and publishes its
  // decision to every other rank (role 2), which follows it; role 0 alone
  int role;
  int n_follow;
  int64_t* dec_out[ARM_MAX_SRC];     // leader: each follower's decision record (peer memory)
  const int64_t* dec_in;             // follower: this rank's decision record
  int64_t epoch;
};
void verify_arm(const ArmArgs& a, cudaStream_t st);
struct SelectArgs {
  const int64_t* rflag;
  const int64_t* reply;
  int64_t rseq;
  int64_t* reply_host;
  int head_words, B, K, nk, a0, n_eos, ctrl, top_stride;
  const int64_t* tab;  // sid[B] | prefix[B] | n_limit[B] | keys[B][nk][2] | key_rows[B][nk] | eos | ctrl[B][2K]
  const int64_t* top;
  int64_t* out_slot[ARM_MAX_SRC];
  int64_t* out_flag[ARM_MAX_SRC];
  int64_t out_seq[ARM_MAX_SRC];
  int n_out;
  int* status;         // pinned [2]
  unsigned long long limit_ns;
};
void select_send(const SelectArgs& a, cudaStream_t st);
void* mailbox_alloc(size_t nbytes);
void mailbox_free(void* p);
void ipc_get_handle(void* p, unsigned char* out64);
void* ipc_open_handle(const unsigned char* in64);
void ipc_close_handle(void* p);
}  // namespace d3d

namespace d3d {
// ---- tensor-parallel exchange (tp.cu)
constexpr int TP_MAX = 8;
struct TpArgs {
  int tp, rank;
  int64_t* epoch;                 // this rank's forward counter (device)
  int64_t* flags[TP_MAX];         // every rank's flag array (peer-mapped): [exchange][source rank]
  uint8_t* parts[TP_MAX];         // every rank's exchange region (peer-mapped)
  int* status;
  unsigned long long timeout_ns;
};
void tp_epoch_bump(int64_t* epoch, cudaStream_t st);
void tp_signal(const TpArgs& a, int x, cudaStream_t st);
void add_rmsnorm_tp(const TpArgs& a, int x, size_t part_off, int nsplit, int pull, __nv_bfloat16* residual,
                    const __nv_bfloat16* w, __nv_bfloat16* out, int M, int N, float eps, cudaStream_t st);
void tp_publish_topk(const float* lv, const int64_t* li, int M, int k, int64_t id_offset, uint8_t* cand,
                     cudaStream_t st);
void topk_merge_tp(const TpArgs& a, int x, size_t cand_off, int M, int k, float* ov, int64_t* oi, cudaStream_t st);
}  // namespace d3d

namespace d3d {
// ---- sharded optimizer step fused with its collectives (fsdp.cu)
constexpr int FSDP_MAX = 8;
struct FsdpArgs {
  int world, rank;
  size_t lo, shard;                 // this rank's element range of the flattened model
  float* grads[FSDP_MAX];           // every rank's full fp32 gradient (peer-mapped)
  __nv_bfloat16* params[FSDP_MAX];  // every rank's full bf16 parameters (peer-mapped)
  int64_t* flags[FSDP_MAX];         // every rank's flags: [phase][source rank]
  int* status;
  unsigned long long timeout_ns;
};
void fsdp_signal(const FsdpArgs& a, int phase, int64_t e, cudaStream_t st);
void fsdp_reduce(const FsdpArgs& a, int64_t e, float* gshard, float* sumsq, cudaStream_t st);
void fsdp_update(const FsdpArgs& a, int64_t e, const float* gshard, float* p, float* m, float* v, float lr, float b1,
                 float b2, float eps, float wd, int step, float scale, unsigned int* ticket, cudaStream_t st);
void fsdp_wait(const FsdpArgs& a, int phase, int64_t e, cudaStream_t st);
void fsdp_gather(const FsdpArgs& a, size_t off, size_t n, __nv_bfloat16* dst, cudaStream_t st);
}  // namespace d3d
