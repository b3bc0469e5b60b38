// PyTorch bindings of the d3d_b200 sm_100a kernels.  Every op runs on the
// current CUDA stream and checks shapes/dtypes/alignment before launching.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "gemm.h"
#include "kernels.h"

using torch::Tensor;

namespace {

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")
#define CHECK_DT(t, dt) TORCH_CHECK((t).scalar_type() == (dt), #t " has wrong dtype")

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

inline __nv_bfloat16* bf(Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }
inline const __nv_bfloat16* cbf(const Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
inline int* status_ptr(const c10::optional<Tensor>& s) { return s ? s->data_ptr<int>() : nullptr; }

constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s bound on every in-kernel wait

// ``wn`` > 0 marks ``w`` as packed (see d3d_b200.ops.pack_weight): a
// [ceil(N/128) * ceil(K/64) * 128, 64] tensor of contiguous 16 KB tiles for a
// logical [wn, K] weight.
d3d::GemmArgs base_args(const Tensor& x, const Tensor& w, int bt, const c10::optional<Tensor>& status,
                        int64_t wn) {
  CHECK_CUDA(x);
  CHECK_CUDA(w);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(w, torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2, "gemm: x [M,K], w [N,K]");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1, "gemm: inner dim must be contiguous");
  d3d::GemmArgs a{};
  a.x = cbf(x);
  a.w = cbf(w);
  a.M = static_cast<int>(x.size(0));
  a.K = static_cast<int>(x.size(1));
  a.ldx = static_cast<int>(x.stride(0));
  if (wn > 0) {
    const int64_t tiles = (wn + 127) / 128 * ((a.K + 63) / 64);
    TORCH_CHECK(w.size(1) == 64 && w.size(0) == tiles * 128 && w.is_contiguous(), "gemm: bad packed weight");
    a.N = static_cast<int>(wn);
    a.ldw = 64;
    a.w_packed = 1;
  } else {
    TORCH_CHECK(x.size(1) == w.size(1), "gemm: K mismatch");
    a.N = static_cast<int>(w.size(0));
    a.ldw = static_cast<int>(w.stride(0));
  }
  a.bt = bt;
  a.splits = 1;
  a.topk = 1;
  a.status = status_ptr(status);
  a.timeout_ns = kTimeoutNs;
  return a;
}

void gemm_partial(Tensor x, Tensor w, Tensor out, int64_t splits, int64_t bt, c10::optional<Tensor> status,
                  int64_t wn) {
  const c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, static_cast<int>(bt), status, wn);
  CHECK_DT(out, torch::kFloat32);
  CHECK_CONTIG(out);
  TORCH_CHECK(out.numel() >= splits * a.M * a.N, "gemm_partial: out too small");
  a.mode = 0;
  a.splits = static_cast<int>(splits);
  a.out_f32 = out.data_ptr<float>();
  if (a.M == 0) return;
  d3d::gemm_launch(a, cur_stream());
}

// fp32 split-K partials reduced inside the GEMM: the last unit of each output
// tile adds the split sum to the bf16 residual ``resid`` [M, N] in place and
// writes the tile's per-row sums of squares ``sumsq`` [ceil(N/128), M];
// ``ticket`` is an int32 [>= ceil(N/128) * ceil(M/bt)] buffer of zeros.
void gemm_partial_fin(Tensor x, Tensor w, Tensor part, int64_t splits, int64_t bt, c10::optional<Tensor> status,
                      int64_t wn, Tensor resid, Tensor sumsq, Tensor ticket) {
  const c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, static_cast<int>(bt), status, wn);
  CHECK_DT(part, torch::kFloat32);
  CHECK_CONTIG(part);
  CHECK_DT(resid, torch::kBFloat16);
  CHECK_DT(sumsq, torch::kFloat32);
  CHECK_DT(ticket, torch::kInt32);
  TORCH_CHECK(part.numel() >= splits * a.M * a.N, "gemm_partial_fin: partials too small");
  TORCH_CHECK(resid.size(0) == a.M && resid.size(1) == a.N && resid.stride(1) == 1, "gemm_partial_fin: residual");
  const int ntn = (a.N + 127) / 128, ntm = (a.M + static_cast<int>(bt) - 1) / static_cast<int>(bt);
  TORCH_CHECK(sumsq.numel() >= static_cast<int64_t>(ntn) * a.M, "gemm_partial_fin: sumsq too small");
  TORCH_CHECK(ticket.numel() >= static_cast<int64_t>(ntn) * ntm, "gemm_partial_fin: ticket too small");
  a.mode = 4;
  a.splits = static_cast<int>(splits);
  a.out_f32 = part.data_ptr<float>();
  a.fin_x = bf(resid);
  a.fin_ldx = static_cast<int>(resid.stride(0));
  a.fin_sumsq = sumsq.data_ptr<float>();
  a.fin_ticket = reinterpret_cast<unsigned int*>(ticket.data_ptr<int>());
  if (a.M == 0) return;
  d3d::gemm_launch(a, cur_stream());
}

void gemm_bf16(Tensor x, Tensor w, Tensor out, c10::optional<Tensor> residual, int64_t bt,
               c10::optional<Tensor> status, int64_t wn) {
  const c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, static_cast<int>(bt), status, wn);
  CHECK_DT(out, torch::kBFloat16);
  TORCH_CHECK(out.size(0) == a.M && out.size(1) == a.N && out.stride(1) == 1, "gemm_bf16: out shape");
  a.mode = 1;
  a.out_bf16 = bf(out);
  a.ldc = static_cast<int>(out.stride(0));
  if (residual) {
    CHECK_DT(*residual, torch::kBFloat16);
    TORCH_CHECK(residual->stride(1) == 1, "residual inner dim must be contiguous");
    a.residual = cbf(*residual);
    a.ldr = static_cast<int>(residual->stride(0));
  }
  if (a.M == 0) return;
  d3d::gemm_launch(a, cur_stream());
}

// SwiGLU fused into the GEMM epilogue: w is the interleaved gate|up weight
// (d3d_b200.ops.pack_gate_up) of logical shape [wn = 2I, K]; out is [M, I].
void gemm_swiglu(Tensor x, Tensor w, Tensor out, int64_t bt, c10::optional<Tensor> status, int64_t wn) {
  const c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, static_cast<int>(bt), status, wn);
  CHECK_DT(out, torch::kBFloat16);
  TORCH_CHECK(out.size(0) == a.M && 2 * out.size(1) == a.N && out.stride(1) == 1, "gemm_swiglu: out shape");
  a.mode = 3;
  a.out_bf16 = bf(out);
  a.ldc = static_cast<int>(out.stride(0));
  if (a.M == 0) return;
  d3d::gemm_launch(a, cur_stream());
}

void gemm_topk(Tensor x, Tensor w, Tensor topv, Tensor topi, int64_t k, int64_t bt, c10::optional<Tensor> status,
               int64_t wn) {
  const c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, static_cast<int>(bt), status, wn);
  const int kt = k <= 1 ? 1 : (k <= 2 ? 2 : 4);
  const int ntiles = (a.N + 127) / 128;
  CHECK_DT(topv, torch::kFloat32);
  CHECK_DT(topi, torch::kInt32);
  TORCH_CHECK(topv.numel() >= static_cast<int64_t>(a.M) * ntiles * kt && topi.numel() >= topv.numel(),
              "gemm_topk: partial buffers too small");
  a.mode = 2;
  a.topk = kt;
  a.topv = topv.data_ptr<float>();
  a.topi = topi.data_ptr<int>();
  if (a.M == 0) return;
  d3d::gemm_launch(a, cur_stream());
}

void add_rmsnorm(c10::optional<Tensor> part, int64_t nsplit, Tensor residual, Tensor w, Tensor out, double eps) {
  const c10::cuda::CUDAGuard g(residual.device());
  CHECK_DT(residual, torch::kBFloat16);
  CHECK_CONTIG(residual);
  CHECK_CONTIG(out);
  const int M = static_cast<int>(residual.size(0)), N = static_cast<int>(residual.size(1));
  d3d::add_rmsnorm(part ? part->data_ptr<float>() : nullptr, static_cast<int>(nsplit), bf(residual), cbf(w), bf(out),
                   M, N, static_cast<float>(eps), cur_stream());
}

void swiglu(Tensor part, int64_t nsplit, Tensor h, bool interleaved) {
  const c10::cuda::CUDAGuard g(h.device());
  CHECK_CONTIG(h);
  CHECK_DT(part, torch::kFloat32);
  d3d::swiglu(part.data_ptr<float>(), static_cast<int>(nsplit), bf(h), static_cast<int>(h.size(0)),
              static_cast<int>(h.size(1)), interleaved, cur_stream());
}

void swiglu_rowscale(Tensor part, int64_t nsplit, Tensor h, Tensor rsq, int64_t rsq_n, double eps) {
  const c10::cuda::CUDAGuard g(h.device());
  CHECK_CONTIG(h);
  CHECK_DT(part, torch::kFloat32);
  CHECK_DT(rsq, torch::kFloat32);
  const int M = static_cast<int>(h.size(0));
  const int tiles = static_cast<int>((rsq_n + 127) / 128);
  TORCH_CHECK(rsq.numel() >= static_cast<int64_t>(tiles) * M, "swiglu_rowscale: sums of squares too small");
  d3d::swiglu_rowscale(part.data_ptr<float>(), static_cast<int>(nsplit), bf(h), M, static_cast<int>(h.size(1)),
                       rsq.data_ptr<float>(), tiles, static_cast<int>(rsq_n), static_cast<float>(eps), cur_stream());
}

void residual_split_reduce(Tensor part, int64_t nsplit, Tensor x, Tensor sumsq) {
  const c10::cuda::CUDAGuard g(x.device());
  CHECK_CONTIG(x);
  CHECK_DT(part, torch::kFloat32);
  CHECK_DT(sumsq, torch::kFloat32);
  const int M = static_cast<int>(x.size(0)), N = static_cast<int>(x.size(1));
  TORCH_CHECK(N % 4 == 0, "residual_split_reduce: row length must be a multiple of 4");
  TORCH_CHECK(part.numel() >= nsplit * static_cast<int64_t>(M) * N, "residual_split_reduce: partials too small");
  TORCH_CHECK(sumsq.numel() >= static_cast<int64_t>((N + 127) / 128) * M, "residual_split_reduce: sumsq too small");
  d3d::residual_split_reduce(part.data_ptr<float>(), static_cast<int>(nsplit), bf(x), M, N, sumsq.data_ptr<float>(),
                             cur_stream());
}

void tile_sumsq(Tensor x, Tensor out) {
  const c10::cuda::CUDAGuard g(x.device());
  CHECK_CONTIG(x);
  CHECK_DT(out, torch::kFloat32);
  const int M = static_cast<int>(x.size(0)), N = static_cast<int>(x.size(1));
  TORCH_CHECK(out.numel() >= static_cast<int64_t>((N + 127) / 128) * M, "tile_sumsq: out too small");
  d3d::tile_sumsq(cbf(x), M, N, out.data_ptr<float>(), cur_stream());
}

void qkv_rope_kv(c10::optional<Tensor> part, c10::optional<Tensor> y, int64_t nsplit, Tensor q_norm, Tensor k_norm,
                 Tensor inv_freq, Tensor positions, Tensor slots, Tensor q_out, Tensor k_cache, Tensor v_cache,
                 int64_t Hq, int64_t Hkv, int64_t D, double eps, c10::optional<Tensor> status,
                 c10::optional<Tensor> rsq, int64_t rsq_n) {
  const c10::cuda::CUDAGuard g(q_out.device());
  CHECK_DT(positions, torch::kInt64);
  CHECK_DT(slots, torch::kInt64);
  CHECK_CONTIG(q_out);
  TORCH_CHECK(D == 32 || D == 64 || D == 128, "head_dim must be 32, 64 or 128");
  d3d::QkvRopeArgs a{};
  a.part = part ? part->data_ptr<float>() : nullptr;
  a.y = y ? cbf(*y) : nullptr;
  TORCH_CHECK(a.part || a.y, "qkv_rope_kv needs partials or bf16 input");
  a.nsplit = static_cast<int>(nsplit);
  a.M = static_cast<int>(positions.numel());
  a.Hq = static_cast<int>(Hq);
  a.Hkv = static_cast<int>(Hkv);
  a.head_dim = static_cast<int>(D);
  a.q_norm = cbf(q_norm);
  a.k_norm = cbf(k_norm);
  a.inv_freq = inv_freq.data_ptr<float>();
  a.positions = positions.data_ptr<int64_t>();
  a.slots = slots.data_ptr<int64_t>();
  a.q_out = bf(q_out);
  a.k_cache = bf(k_cache);
  a.v_cache = bf(v_cache);
  a.eps = static_cast<float>(eps);
  a.num_slots = k_cache.size(0);
  a.status = status_ptr(status);
  if (rsq) {
    CHECK_DT(*rsq, torch::kFloat32);
    a.rsq = rsq->data_ptr<float>();
    a.rsq_n = static_cast<int>(rsq_n);
    a.rsq_tiles = static_cast<int>((rsq_n + 127) / 128);
    TORCH_CHECK(rsq->numel() >= static_cast<int64_t>(a.rsq_tiles) * a.M, "qkv_rope_kv: sums of squares too small");
  }
  d3d::qkv_rope_kv(a, cur_stream());
}

void embed(Tensor ids, Tensor table, c10::optional<Tensor> cond, c10::optional<Tensor> cond_rows, int64_t q_len,
           Tensor out, c10::optional<Tensor> status) {
  const c10::cuda::CUDAGuard g(out.device());
  CHECK_DT(ids, torch::kInt64);
  CHECK_CONTIG(table);
  CHECK_CONTIG(out);
  TORCH_CHECK(table.size(1) % 8 == 0, "hidden size must be a multiple of 8");
  d3d::embed(ids.data_ptr<int64_t>(), cbf(table), cond ? cbf(*cond) : nullptr,
             cond_rows ? cond_rows->data_ptr<uint8_t>() : nullptr, static_cast<int>(q_len), bf(out),
             static_cast<int>(ids.numel()), static_cast<int>(table.size(1)), cur_stream(), table.size(0),
             status_ptr(status));
}

void topk_merge(Tensor tv, Tensor ti, int64_t M, int64_t ntiles, int64_t kt, int64_t k, c10::optional<Tensor> ov,
                Tensor oi) {
  const c10::cuda::CUDAGuard g(oi.device());
  CHECK_DT(oi, torch::kInt64);
  d3d::topk_merge(tv.data_ptr<float>(), ti.data_ptr<int>(), static_cast<int>(ntiles), static_cast<int>(kt),
                  static_cast<int>(k), ov ? ov->data_ptr<float>() : nullptr, oi.data_ptr<int64_t>(),
                  static_cast<int>(M), cur_stream());
}

void greedy_accept(Tensor blocks, Tensor post, Tensor commit, Tensor corr, c10::optional<Tensor> hidden,
                   c10::optional<Tensor> hid_out) {
  const c10::cuda::CUDAGuard g(blocks.device());
  CHECK_DT(blocks, torch::kInt64);
  CHECK_DT(post, torch::kInt64);
  CHECK_CONTIG(blocks);
  CHECK_CONTIG(post);
  const int B = static_cast<int>(blocks.size(0)), K = static_cast<int>(blocks.size(1));
  int H = 0;
  if (hidden) H = static_cast<int>(hidden->size(-1));
  d3d::greedy_accept(blocks.data_ptr<int64_t>(), post.data_ptr<int64_t>(), B, K, commit.data_ptr<int64_t>(),
                     corr.data_ptr<int64_t>(), hidden ? cbf(*hidden) : nullptr,
                     hid_out ? bf(*hid_out) : nullptr, H, cur_stream());
}

void attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_table, Tensor rows, Tensor kv_end,
               int64_t B, int64_t q_len, int64_t Hq, int64_t Hkv, int64_t page_size, double scale, int64_t chunk,
               int64_t n_chunks, c10::optional<Tensor> part_o, c10::optional<Tensor> part_ml, Tensor out,
               bool invariant, c10::optional<Tensor> status, bool force_split) {
  const c10::cuda::CUDAGuard g(q.device());
  CHECK_CONTIG(q);
  CHECK_CONTIG(out);
  CHECK_DT(block_table, torch::kInt32);
  CHECK_DT(rows, torch::kInt32);
  CHECK_DT(kv_end, torch::kInt32);
  TORCH_CHECK(chunk % 64 == 0, "attention chunk must be a multiple of 64");
  TORCH_CHECK(chunk / page_size + 1 <= 1024, "attention chunk spans too many pages");
  TORCH_CHECK(n_chunks == 1 || (part_o && part_ml), "split attention needs partial buffers");
  TORCH_CHECK(n_chunks >= 1 && n_chunks <= 512, "attention: 1 <= n_chunks <= 512 (the combine kernel's limit)");
  d3d::AttnArgs a{};
  a.q = cbf(q);
  a.k_cache = cbf(k_cache);
  a.v_cache = cbf(v_cache);
  a.block_table = block_table.data_ptr<int>();
  a.bt_stride = static_cast<int>(block_table.stride(0));
  a.rows = rows.data_ptr<int>();
  a.kv_end = kv_end.data_ptr<int>();
  a.B = static_cast<int>(B);
  a.q_len = static_cast<int>(q_len);
  a.Hq = static_cast<int>(Hq);
  a.Hkv = static_cast<int>(Hkv);
  a.head_dim = static_cast<int>(q.size(-1));
  a.page_size = static_cast<int>(page_size);
  a.scale = static_cast<float>(scale);
  a.chunk = static_cast<int>(chunk);
  a.n_chunks = static_cast<int>(n_chunks);
  a.invariant = invariant ? 1 : 0;
  a.part_o = part_o ? part_o->data_ptr<float>() : nullptr;
  a.part_ml = part_ml ? part_ml->data_ptr<float>() : nullptr;
  a.out = bf(out);
  a.num_slots = k_cache.size(0);
  a.status = status_ptr(status);
  if (force_split) {
    const cudaError_t e = d3d::attention_split(a, cur_stream());
    TORCH_CHECK(e == cudaSuccess, "attention (split-KV): ", cudaGetErrorString(e));
    return;
  }
  d3d::attention(a, cur_stream());
}

// Whether d3d::attention takes the tcgen05/TMEM kernel for this shape.
bool attention_uses_tc(int64_t Hq, int64_t Hkv, int64_t head_dim, int64_t page_size, int64_t chunk,
                       int64_t n_chunks) {
  d3d::AttnArgs a{};
  a.Hq = static_cast<int>(Hq);
  a.Hkv = static_cast<int>(Hkv);
  a.head_dim = static_cast<int>(head_dim);
  a.page_size = static_cast<int>(page_size);
  a.chunk = static_cast<int>(chunk);
  a.n_chunks = static_cast<int>(n_chunks);
  float dummy = 0.f;
  a.part_o = a.part_ml = &dummy;
  a.num_slots = 1;
  return d3d::attention_tc_supported(a);
}

template <typename T>
T* opt_ptr(const c10::optional<Tensor>& t) {
  return t ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

void kl_ce_stats(c10::optional<Tensor> zt, Tensor zs, int64_t C, int64_t v0, c10::optional<Tensor> target,
                 Tensor st) {
  const c10::cuda::CUDAGuard g(zs.device());
  CHECK_DT(zs, torch::kFloat32);
  CHECK_DT(st, torch::kFloat32);
  TORCH_CHECK(zs.stride(1) == 1, "logit chunk rows must be contiguous");
  d3d::kl_ce_stats(opt_ptr<float>(zt), zs.data_ptr<float>(), static_cast<int>(zs.size(0)), static_cast<int>(C),
                   static_cast<int>(zs.stride(0)), static_cast<int>(v0), opt_ptr<int64_t>(target),
                   st.data_ptr<float>(), cur_stream());
}

void kl_ce_grad(c10::optional<Tensor> zt, Tensor zs, int64_t C, int64_t v0, c10::optional<Tensor> target,
                Tensor lse_t, Tensor lse_s, c10::optional<Tensor> w_kl, c10::optional<Tensor> w_ce,
                c10::optional<Tensor> dz, c10::optional<Tensor> dzT) {
  const c10::cuda::CUDAGuard g(zs.device());
  d3d::kl_ce_grad(opt_ptr<float>(zt), zs.data_ptr<float>(), static_cast<int>(zs.size(0)), static_cast<int>(C),
                  static_cast<int>(zs.stride(0)), static_cast<int>(v0), opt_ptr<int64_t>(target),
                  lse_t.data_ptr<float>(), lse_s.data_ptr<float>(), opt_ptr<float>(w_kl), opt_ptr<float>(w_ce),
                  opt_ptr<__nv_bfloat16>(dz), dz ? static_cast<int>(dz->stride(0)) : 0,
                  opt_ptr<__nv_bfloat16>(dzT), dzT ? static_cast<int>(dzT->stride(0)) : 0, cur_stream());
}

void adamw(Tensor p, Tensor grad, Tensor m, Tensor v, c10::optional<Tensor> out, double lr, double b1, double b2,
           double eps, double wd, int64_t step, double grad_scale) {
  const c10::cuda::CUDAGuard g(p.device());
  CHECK_DT(p, torch::kFloat32);
  CHECK_DT(grad, torch::kFloat32);
  TORCH_CHECK(p.numel() == grad.numel() && p.numel() == m.numel() && p.numel() == v.numel(), "adamw: sizes");
  TORCH_CHECK(!out || out->numel() == p.numel(), "adamw: out size");
  d3d::adamw(p.data_ptr<float>(), grad.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
             opt_ptr<__nv_bfloat16>(out), static_cast<size_t>(p.numel()), static_cast<float>(lr),
             static_cast<float>(b1), static_cast<float>(b2), static_cast<float>(eps), static_cast<float>(wd),
             static_cast<int>(step), static_cast<float>(grad_scale), cur_stream());
}

void sumsq(Tensor x, Tensor out) {
  const c10::cuda::CUDAGuard g(x.device());
  CHECK_DT(x, torch::kFloat32);
  d3d::sumsq(x.data_ptr<float>(), static_cast<size_t>(x.numel()), out.data_ptr<float>(), cur_stream());
}

// ---------------------------------------------------------------- handoff
// Mailboxes are raw device allocations (not from the caching allocator) so
// that CUDA IPC maps exactly them; Python holds them as integers and views
// them as uint8 tensors.
int64_t mailbox_alloc(int64_t nbytes, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  return reinterpret_cast<int64_t>(d3d::mailbox_alloc(static_cast<size_t>(nbytes)));
}
void mailbox_free(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  d3d::mailbox_free(reinterpret_cast<void*>(ptr));
}
Tensor mailbox_view(int64_t ptr, int64_t nbytes, int64_t device) {
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, static_cast<c10::DeviceIndex>(device));
  return torch::from_blob(reinterpret_cast<void*>(ptr), {nbytes}, opts);
}
py::bytes ipc_handle(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  unsigned char h[64];
  d3d::ipc_get_handle(reinterpret_cast<void*>(ptr), h);
  return py::bytes(reinterpret_cast<const char*>(h), 64);
}
int64_t ipc_open(py::bytes handle, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  std::string s = handle;
  TORCH_CHECK(s.size() == 64, "ipc handle must be 64 bytes");
  return reinterpret_cast<int64_t>(d3d::ipc_open_handle(reinterpret_cast<const unsigned char*>(s.data())));
}
void ipc_close(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  d3d::ipc_close_handle(reinterpret_cast<void*>(ptr));
}
void handoff_put(Tensor src, int64_t dst_ptr, int64_t flag_ptr, int64_t seq, c10::optional<Tensor> ticket) {
  TORCH_CHECK(!ticket || ticket->is_cuda(), "handoff_put: ticket must be on the GPU");
  const c10::cuda::CUDAGuard g(ticket ? ticket->device() : at::Device(at::kCUDA, at::cuda::current_device()));
  TORCH_CHECK(src.is_cuda() || src.is_pinned(), "handoff_put: src must be on the GPU or pinned");
  CHECK_CONTIG(src);
  TORCH_CHECK(reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0, "handoff_put: src not 16-byte aligned");
  const size_t nbytes = static_cast<size_t>(src.numel()) * src.element_size();
  TORCH_CHECK(nbytes % 16 == 0 && dst_ptr % 16 == 0, "handoff_put: 16-byte sizes and addresses");
  d3d::handoff_put(src.data_ptr(), reinterpret_cast<void*>(dst_ptr), nbytes, reinterpret_cast<int64_t*>(flag_ptr),
                   seq, ticket ? reinterpret_cast<unsigned int*>(ticket->data_ptr<int>()) : nullptr, cur_stream());
}
void handoff_wait(Tensor flag, int64_t seq, c10::optional<Tensor> src, c10::optional<Tensor> dst, Tensor status) {
  const c10::cuda::CUDAGuard g(flag.device());
  CHECK_DT(flag, torch::kInt64);
  CHECK_DT(status, torch::kInt32);
  // the kernel writes status and dst directly: device memory or pinned host memory only
  TORCH_CHECK(status.is_cuda() || status.is_pinned(), "handoff_wait: status must be on the GPU or pinned");
  TORCH_CHECK(!dst || dst->is_cuda() || dst->is_pinned(), "handoff_wait: dst must be on the GPU or pinned");
  TORCH_CHECK(!dst || dst->is_contiguous(), "handoff_wait: dst must be contiguous");
  TORCH_CHECK(!dst || reinterpret_cast<uintptr_t>(dst->data_ptr()) % 16 == 0, "handoff_wait: dst not 16-byte aligned");
  size_t nbytes = 0;
  if (src && dst) {
    nbytes = static_cast<size_t>(dst->numel()) * dst->element_size();
    TORCH_CHECK(static_cast<size_t>(src->numel()) * src->element_size() >= nbytes && nbytes % 16 == 0,
                "handoff_wait: payload sizes");
  }
  d3d::handoff_wait(flag.data_ptr<int64_t>(), seq, src ? src->data_ptr() : nullptr, dst ? dst->data_ptr() : nullptr,
                    nbytes, status.data_ptr<int>(), kTimeoutNs, cur_stream());
}
void accept_send(Tensor blocks, Tensor post, c10::optional<Tensor> hidden, int64_t out_ptr, int64_t hid_ptr,
                 int64_t flag_ptr, int64_t seq, c10::optional<Tensor> gate) {
  const c10::cuda::CUDAGuard g(blocks.device());
  CHECK_DT(blocks, torch::kInt64);
  CHECK_DT(post, torch::kInt64);
  CHECK_CONTIG(blocks);
  CHECK_CONTIG(post);
  const int B = static_cast<int>(blocks.size(0)), K = static_cast<int>(blocks.size(1));
  const int H = hidden ? static_cast<int>(hidden->size(-1)) : 0;
  d3d::accept_send(blocks.data_ptr<int64_t>(), post.data_ptr<int64_t>(), B, K, hidden ? cbf(*hidden) : nullptr, H,
                   reinterpret_cast<int64_t*>(out_ptr), reinterpret_cast<__nv_bfloat16*>(hid_ptr),
                   reinterpret_cast<int64_t*>(flag_ptr), seq, gate ? gate->data_ptr<int>() : nullptr, cur_stream());
}

// ``src``: int64 CPU [4, n_src] = inbox flag, message slot, pinned head copy
// (addresses) and expected sequence number per source; ``rows``: int64 CPU
// [2, n_src] = first merged row and row count per source.
void verify_arm(Tensor src, Tensor rows_of, int64_t K, int64_t head_words, int64_t page, Tensor tab,
                Tensor block_table, Tensor seq_rows, int64_t scratch_slot, Tensor ids, Tensor pos, Tensor slots,
                Tensor rows, Tensor kv_end, Tensor gate, Tensor status, int64_t role, c10::optional<Tensor> dec,
                int64_t epoch) {
  const c10::cuda::CUDAGuard g(ids.device());
  CHECK_DT(src, torch::kInt64);
  CHECK_DT(rows_of, torch::kInt64);
  CHECK_DT(tab, torch::kInt64);
  CHECK_DT(block_table, torch::kInt32);
  CHECK_DT(seq_rows, torch::kInt64);
  CHECK_DT(rows, torch::kInt32);
  CHECK_DT(kv_end, torch::kInt32);
  CHECK_DT(gate, torch::kInt32);
  CHECK_DT(status, torch::kInt32);
  TORCH_CHECK(status.is_pinned(), "verify_arm: status must be pinned host memory");
  const int n = static_cast<int>(src.size(1));
  TORCH_CHECK(src.dim() == 2 && src.size(0) == 4 && n >= 1 && n <= d3d::ARM_MAX_SRC, "verify_arm: bad source table");
  TORCH_CHECK(rows_of.dim() == 2 && rows_of.size(0) == 2 && rows_of.size(1) == n, "verify_arm: bad row table");
  TORCH_CHECK(status.numel() >= n + 1, "verify_arm: status too small");
  d3d::ArmArgs a{};
  auto sp = src.contiguous();
  auto rp = rows_of.contiguous();
  const int64_t* v = sp.data_ptr<int64_t>();
  const int64_t* rv = rp.data_ptr<int64_t>();
  int B = 0;
  for (int d = 0; d < n; ++d) {
    a.flag[d] = reinterpret_cast<const int64_t*>(v[d]);
    a.msg[d] = reinterpret_cast<const int64_t*>(v[n + d]);
    a.head[d] = reinterpret_cast<int64_t*>(v[2 * n + d]);
    a.seq[d] = v[3 * n + d];
    a.row0[d] = static_cast<int>(rv[d]);
    a.nb[d] = static_cast<int>(rv[n + d]);
    TORCH_CHECK(a.row0[d] == B, "verify_arm: sources must cover the rows in order");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(a.msg[d]) % 16 == 0 && reinterpret_cast<uintptr_t>(a.head[d]) % 16 == 0,
                "verify_arm: 16-byte aligned messages");
    B += a.nb[d];
  }
  TORCH_CHECK(tab.numel() >= 2 * B && seq_rows.numel() >= B && kv_end.numel() >= B, "verify_arm: row tables");
  TORCH_CHECK(ids.numel() >= B * K && pos.numel() >= B * K && slots.numel() >= B * K && rows.numel() >= 3 * B * K,
              "verify_arm: input buffers too small");
  a.n_src = n;
  a.K = static_cast<int>(K);
  a.head_words = static_cast<int>(head_words);
  a.page = static_cast<int>(page);
  a.bt_stride = static_cast<int>(block_table.size(1));
  a.tab = tab.data_ptr<int64_t>();
  a.block_table = block_table.data_ptr<int32_t>();
  a.seq_rows = seq_rows.data_ptr<int64_t>();
  a.scratch_slot = scratch_slot;
  a.ids = ids.data_ptr<int64_t>();
  a.pos = pos.data_ptr<int64_t>();
  a.slots = slots.data_ptr<int64_t>();
  a.rows = rows.data_ptr<int32_t>();
  a.kv_end = kv_end.data_ptr<int32_t>();
  a.gate = gate.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.limit_ns = kTimeoutNs;
  TORCH_CHECK(role >= 0 && role <= 2, "verify_arm: role 0 (alone), 1 (leader) or 2 (follower)");
  a.role = static_cast<int>(role);
  a.epoch = epoch;
  if (role != 0) {
    TORCH_CHECK(dec && dec->dtype() == torch::kInt64 && dec->dim() == 1, "verify_arm: decision record table");
    auto dp = dec->contiguous();
    const int64_t* dv = dp.data_ptr<int64_t>();
    if (role == 1) {
      TORCH_CHECK(dp.numel() <= d3d::ARM_MAX_SRC, "verify_arm: up to 8 followers");
      a.n_follow = static_cast<int>(dp.numel());
      for (int f = 0; f < a.n_follow; ++f) a.dec_out[f] = reinterpret_cast<int64_t*>(dv[f]);
    } else {
      TORCH_CHECK(dp.numel() == 1, "verify_arm: a follower reads one decision record");
      a.dec_in = reinterpret_cast<const int64_t*>(dv[0]);
    }
  }
  d3d::verify_arm(a, cur_stream());
}

// ``outs``: int64 CPU [3, n_out] = destination slot, destination flag
// (peer addresses mapped in this process) and sequence number per target rank.
void select_send(Tensor rflag, Tensor reply, int64_t rseq, Tensor reply_host, int64_t B, int64_t K, int64_t nk,
                 bool a0, int64_t n_eos, bool ctrl, c10::optional<Tensor> top, Tensor tab, Tensor outs,
                 Tensor status) {
  const c10::cuda::CUDAGuard g(tab.device());
  CHECK_DT(rflag, torch::kInt64);
  CHECK_DT(reply, torch::kInt64);
  CHECK_DT(reply_host, torch::kInt64);
  CHECK_DT(tab, torch::kInt64);
  CHECK_DT(outs, torch::kInt64);
  CHECK_DT(status, torch::kInt32);
  TORCH_CHECK(status.is_pinned() && reply_host.is_pinned(), "select_send: status and reply copy must be pinned");
  TORCH_CHECK(reply_host.numel() % 2 == 0 && reply.numel() >= reply_host.numel(), "select_send: reply sizes");
  TORCH_CHECK(ctrl || (top && top->dim() == 2), "select_send: the drafts' top ids are needed without controlled drafts");
  const int n = static_cast<int>(outs.size(1));
  TORCH_CHECK(outs.dim() == 2 && outs.size(0) == 3 && n >= 1 && n <= d3d::ARM_MAX_SRC, "select_send: bad outputs");
  TORCH_CHECK(tab.numel() >= 3 * B + B * nk * 3 + n_eos + (ctrl ? 2 * B * K : 0), "select_send: table too small");
  d3d::SelectArgs a{};
  a.rflag = rflag.data_ptr<int64_t>();
  a.reply = reply.data_ptr<int64_t>();
  a.rseq = rseq;
  a.reply_host = reply_host.data_ptr<int64_t>();
  a.head_words = static_cast<int>(reply_host.numel());
  a.B = static_cast<int>(B);
  a.K = static_cast<int>(K);
  a.nk = static_cast<int>(nk);
  a.a0 = a0 ? 1 : 0;
  a.n_eos = static_cast<int>(n_eos);
  a.ctrl = ctrl ? 1 : 0;
  if (top) {
    CHECK_DT(*top, torch::kInt64);
    a.top = top->data_ptr<int64_t>();
    a.top_stride = static_cast<int>(top->stride(0));
  }
  a.tab = tab.data_ptr<int64_t>();
  auto op = outs.contiguous();
  const int64_t* v = op.data_ptr<int64_t>();
  for (int o = 0; o < n; ++o) {
    a.out_slot[o] = reinterpret_cast<int64_t*>(v[o]);
    a.out_flag[o] = reinterpret_cast<int64_t*>(v[n + o]);
    a.out_seq[o] = v[2 * n + o];
  }
  a.n_out = n;
  a.status = status.data_ptr<int>();
  a.limit_ns = kTimeoutNs;
  d3d::select_send(a, cur_stream());
}

// ------------------------------------------------------------ tensor parallel
// ``ptrs`` is an int64 CPU tensor [2, tp]: row 0 = every rank's flag array,
// row 1 = every rank's exchange region (device addresses valid in this process).
d3d::TpArgs tp_args(Tensor ptrs, int64_t rank, Tensor epoch, c10::optional<Tensor> status) {
  TORCH_CHECK(ptrs.dim() == 2 && ptrs.size(0) == 2 && ptrs.size(1) <= d3d::TP_MAX, "tp: bad pointer table");
  CHECK_DT(ptrs, torch::kInt64);
  CHECK_DT(epoch, torch::kInt64);
  d3d::TpArgs a{};
  a.tp = static_cast<int>(ptrs.size(1));
  a.rank = static_cast<int>(rank);
  TORCH_CHECK(a.rank >= 0 && a.rank < a.tp, "tp: rank out of range");
  auto p = ptrs.contiguous().cpu();
  const int64_t* v = p.data_ptr<int64_t>();
  for (int j = 0; j < a.tp; ++j) {
    a.flags[j] = reinterpret_cast<int64_t*>(v[j]);
    a.parts[j] = reinterpret_cast<uint8_t*>(v[a.tp + j]);
  }
  a.epoch = epoch.data_ptr<int64_t>();
  a.status = status_ptr(status);
  a.timeout_ns = kTimeoutNs;
  return a;
}

// Row-parallel GEMM of a tensor-parallel rank: fp32 partials pushed into
// every rank's exchange region at ``part_off`` (slot rank * splits + split),
// flags raised for exchange ``x`` by the last CTA.
void gemm_partial_tp(Tensor x, Tensor w, Tensor ptrs, int64_t rank, Tensor epoch, Tensor ticket, int64_t xidx,
                     int64_t part_off, int64_t splits, int64_t bt, c10::optional<Tensor> status, int64_t wn,
                     bool pull) {
  const c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, static_cast<int>(bt), status, wn);
  const d3d::TpArgs t = tp_args(ptrs, rank, epoch, status);
  CHECK_DT(ticket, torch::kInt32);
  TORCH_CHECK(part_off % 16 == 0, "gemm_partial_tp: partial offset must be 16-byte aligned");
  a.mode = 0;
  a.splits = static_cast<int>(splits);
  a.tp = t.tp;
  a.tp_rank = t.rank;
  a.tp_x = static_cast<int>(xidx);
  a.tp_pull = pull ? 1 : 0;
  for (int r = 0; r < t.tp; ++r) {
    a.tp_out[r] = reinterpret_cast<float*>(t.parts[r] + part_off);
    a.tp_flags[r] = t.flags[r];
  }
  a.tp_epoch = t.epoch;
  a.tp_ticket = reinterpret_cast<unsigned int*>(ticket.data_ptr<int>());
  a.out_f32 = a.tp_out[t.rank];
  if (a.M == 0) return;
  d3d::gemm_launch(a, cur_stream());
}

void tp_epoch_bump(Tensor epoch) {
  const c10::cuda::CUDAGuard g(epoch.device());
  d3d::tp_epoch_bump(epoch.data_ptr<int64_t>(), cur_stream());
}

void tp_signal(Tensor ptrs, int64_t rank, Tensor epoch, int64_t x) {
  const c10::cuda::CUDAGuard g(epoch.device());
  d3d::tp_signal(tp_args(ptrs, rank, epoch, c10::nullopt), static_cast<int>(x), cur_stream());
}

void add_rmsnorm_tp(Tensor ptrs, int64_t rank, Tensor epoch, int64_t x, int64_t part_off, int64_t nsplit,
                    Tensor residual, Tensor w, Tensor out, double eps, c10::optional<Tensor> status, bool pull) {
  const c10::cuda::CUDAGuard g(residual.device());
  CHECK_DT(residual, torch::kBFloat16);
  CHECK_CONTIG(residual);
  CHECK_CONTIG(out);
  TORCH_CHECK(part_off % 16 == 0, "add_rmsnorm_tp: partial offset must be 16-byte aligned");
  d3d::add_rmsnorm_tp(tp_args(ptrs, rank, epoch, status), static_cast<int>(x), static_cast<size_t>(part_off),
                      static_cast<int>(nsplit), pull ? 1 : 0, bf(residual), cbf(w), bf(out), static_cast<int>(residual.size(0)),
                      static_cast<int>(residual.size(1)), static_cast<float>(eps), cur_stream());
}

void tp_publish_topk(Tensor lv, Tensor li, int64_t id_offset, Tensor cand) {
  const c10::cuda::CUDAGuard g(lv.device());
  CHECK_DT(lv, torch::kFloat32);
  CHECK_DT(li, torch::kInt64);
  CHECK_CONTIG(lv);
  CHECK_CONTIG(li);
  TORCH_CHECK(reinterpret_cast<uintptr_t>(cand.data_ptr()) % 16 == 0, "tp_publish_topk: slot alignment");
  d3d::tp_publish_topk(lv.data_ptr<float>(), li.data_ptr<int64_t>(), static_cast<int>(lv.size(0)),
                       static_cast<int>(lv.size(1)), id_offset, cand.data_ptr<uint8_t>(), cur_stream());
}

void topk_merge_tp(Tensor ptrs, int64_t rank, Tensor epoch, int64_t x, int64_t cand_off, int64_t M, int64_t k,
                   c10::optional<Tensor> ov, Tensor oi, c10::optional<Tensor> status) {
  const c10::cuda::CUDAGuard g(oi.device());
  CHECK_DT(oi, torch::kInt64);
  d3d::topk_merge_tp(tp_args(ptrs, rank, epoch, status), static_cast<int>(x), static_cast<size_t>(cand_off),
                     static_cast<int>(M), static_cast<int>(k), ov ? ov->data_ptr<float>() : nullptr,
                     oi.data_ptr<int64_t>(), cur_stream());
}

// ------------------------------------------------------ fused sharded optimizer
// ``ptrs``: int64 CPU tensor [3, world] = every rank's gradient buffer,
// parameter buffer and flag array (device addresses valid in this process).
d3d::FsdpArgs fsdp_args(Tensor ptrs, int64_t rank, int64_t lo, int64_t shard, c10::optional<Tensor> status) {
  TORCH_CHECK(ptrs.dim() == 2 && ptrs.size(0) == 3 && ptrs.size(1) <= d3d::FSDP_MAX, "fsdp: bad pointer table");
  CHECK_DT(ptrs, torch::kInt64);
  d3d::FsdpArgs a{};
  a.world = static_cast<int>(ptrs.size(1));
  a.rank = static_cast<int>(rank);
  TORCH_CHECK(a.rank >= 0 && a.rank < a.world, "fsdp: rank out of range");
  auto p = ptrs.contiguous().cpu();
  const int64_t* v = p.data_ptr<int64_t>();
  for (int j = 0; j < a.world; ++j) {
    a.grads[j] = reinterpret_cast<float*>(v[j]);
    a.params[j] = reinterpret_cast<__nv_bfloat16*>(v[a.world + j]);
    a.flags[j] = reinterpret_cast<int64_t*>(v[2 * a.world + j]);
  }
  a.lo = static_cast<size_t>(lo);
  a.shard = static_cast<size_t>(shard);
  a.status = status_ptr(status);
  a.timeout_ns = kTimeoutNs;
  return a;
}

void fsdp_signal(Tensor ptrs, int64_t rank, int64_t lo, int64_t shard, int64_t phase, int64_t e, Tensor like) {
  const c10::cuda::CUDAGuard g(like.device());
  d3d::fsdp_signal(fsdp_args(ptrs, rank, lo, shard, c10::nullopt), static_cast<int>(phase), e, cur_stream());
}

void fsdp_reduce(Tensor ptrs, int64_t rank, int64_t lo, int64_t shard, int64_t e, Tensor gshard, Tensor sumsq,
                 Tensor status) {
  const c10::cuda::CUDAGuard g(gshard.device());
  CHECK_DT(gshard, torch::kFloat32);
  CHECK_DT(sumsq, torch::kFloat32);
  TORCH_CHECK(gshard.numel() >= shard, "fsdp_reduce: shard buffer too small");
  d3d::fsdp_reduce(fsdp_args(ptrs, rank, lo, shard, status), e, gshard.data_ptr<float>(), sumsq.data_ptr<float>(),
                   cur_stream());
}

void fsdp_update(Tensor ptrs, int64_t rank, int64_t lo, int64_t shard, int64_t e, Tensor gshard, Tensor p, Tensor m,
                 Tensor v, double lr, double b1, double b2, double eps, double wd, int64_t step, double scale,
                 Tensor ticket, Tensor status) {
  const c10::cuda::CUDAGuard g(p.device());
  CHECK_DT(p, torch::kFloat32);
  TORCH_CHECK(p.numel() == shard && m.numel() == shard && v.numel() == shard, "fsdp_update: shard sizes");
  d3d::fsdp_update(fsdp_args(ptrs, rank, lo, shard, status), e, gshard.data_ptr<float>(), p.data_ptr<float>(),
                   m.data_ptr<float>(), v.data_ptr<float>(), static_cast<float>(lr), static_cast<float>(b1),
                   static_cast<float>(b2), static_cast<float>(eps), static_cast<float>(wd), static_cast<int>(step),
                   static_cast<float>(scale), reinterpret_cast<unsigned int*>(ticket.data_ptr<int>()), cur_stream());
}

void fsdp_gather(Tensor ptrs, int64_t rank, int64_t off, int64_t n, Tensor dst) {
  const c10::cuda::CUDAGuard g(dst.device());
  CHECK_DT(dst, torch::kBFloat16);
  CHECK_CONTIG(dst);
  auto a = fsdp_args(ptrs, rank, 0, 0, c10::nullopt);
  TORCH_CHECK(dst.numel() >= static_cast<int64_t>(a.world) * n, "fsdp_gather: destination too small");
  d3d::fsdp_gather(a, static_cast<size_t>(off), static_cast<size_t>(n), bf(dst), cur_stream());
}

void fsdp_wait(Tensor ptrs, int64_t rank, int64_t lo, int64_t shard, int64_t phase, int64_t e, Tensor status) {
  const c10::cuda::CUDAGuard g(status.device());
  d3d::fsdp_wait(fsdp_args(ptrs, rank, lo, shard, status), static_cast<int>(phase), e, cur_stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "d3d_b200 sm_100a kernels";
  m.def("gemm_partial", &gemm_partial, py::arg("x"), py::arg("w"), py::arg("out"), py::arg("splits"),
        py::arg("bt"), py::arg("status") = py::none(), py::arg("wn") = 0);
  m.def("gemm_bf16", &gemm_bf16, py::arg("x"), py::arg("w"), py::arg("out"), py::arg("residual") = py::none(),
        py::arg("bt") = 16, py::arg("status") = py::none(), py::arg("wn") = 0);
  m.def("gemm_topk", &gemm_topk, py::arg("x"), py::arg("w"), py::arg("topv"), py::arg("topi"), py::arg("k"),
        py::arg("bt"), py::arg("status") = py::none(), py::arg("wn") = 0);
  m.def("add_rmsnorm", &add_rmsnorm);
  m.def("swiglu", &swiglu, py::arg("part"), py::arg("nsplit"), py::arg("h"), py::arg("interleaved") = false);
  m.def("gemm_swiglu", &gemm_swiglu, py::arg("x"), py::arg("w"), py::arg("out"), py::arg("bt"),
        py::arg("status") = py::none(), py::arg("wn") = 0);
  m.def("qkv_rope_kv", &qkv_rope_kv, py::arg("part"), py::arg("y"), py::arg("nsplit"), py::arg("q_norm"),
        py::arg("k_norm"), py::arg("inv_freq"), py::arg("positions"), py::arg("slots"), py::arg("q_out"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("eps"),
        py::arg("status") = py::none(), py::arg("rsq") = py::none(), py::arg("rsq_n") = 0);
  m.def("swiglu_rowscale", &swiglu_rowscale);
  m.def("tile_sumsq", &tile_sumsq);
  m.def("residual_split_reduce", &residual_split_reduce);
  m.def("embed", &embed, py::arg("ids"), py::arg("table"), py::arg("cond"), py::arg("cond_rows"), py::arg("q_len"),
        py::arg("out"), py::arg("status") = py::none());
  m.def("topk_merge", &topk_merge);
  m.def("greedy_accept", &greedy_accept);
  m.def("attention_uses_tc", &attention_uses_tc);
  m.def("fsdp_gather", &fsdp_gather);
  m.def("gemm_partial_fin", &gemm_partial_fin);
  m.def("attention", &attention, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("block_table"),
        py::arg("rows"), py::arg("kv_end"), py::arg("B"), py::arg("q_len"), py::arg("Hq"), py::arg("Hkv"),
        py::arg("page_size"), py::arg("scale"), py::arg("chunk"), py::arg("n_chunks"), py::arg("part_o"),
        py::arg("part_ml"), py::arg("out"), py::arg("invariant") = false, py::arg("status") = py::none(),
        py::arg("force_split") = false);
  m.def("gemm_stages", &d3d::gemm_stages);
  m.def("kl_ce_stats", &kl_ce_stats);
  m.def("kl_ce_grad", &kl_ce_grad);
  m.def("adamw", &adamw);
  m.def("sumsq", &sumsq);
  m.def("gemm_ctas_per_sm", &d3d::gemm_ctas_per_sm);
  m.def("mailbox_alloc", &mailbox_alloc);
  m.def("mailbox_free", &mailbox_free);
  m.def("mailbox_view", &mailbox_view);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("handoff_put", &handoff_put, py::arg("src"), py::arg("dst_ptr"), py::arg("flag_ptr"), py::arg("seq"),
        py::arg("ticket") = py::none());
  m.def("handoff_wait", &handoff_wait, py::arg("flag"), py::arg("seq"), py::arg("src"), py::arg("dst"),
        py::arg("status"));
  m.def("accept_send", &accept_send, py::arg("blocks"), py::arg("post"), py::arg("hidden"), py::arg("out_ptr"),
        py::arg("hid_ptr"), py::arg("flag_ptr"), py::arg("seq"), py::arg("gate") = py::none());
  m.def("verify_arm", &verify_arm, py::arg("src"), py::arg("rows_of"), py::arg("K"), py::arg("head_words"),
        py::arg("page"), py::arg("tab"), py::arg("block_table"), py::arg("seq_rows"), py::arg("scratch_slot"),
        py::arg("ids"), py::arg("pos"), py::arg("slots"), py::arg("rows"), py::arg("kv_end"), py::arg("gate"),
        py::arg("status"), py::arg("role") = 0, py::arg("dec") = py::none(), py::arg("epoch") = 0);
  m.def("select_send", &select_send);
  m.def("tp_epoch_bump", &tp_epoch_bump);
  m.def("gemm_partial_tp", &gemm_partial_tp, py::arg("x"), py::arg("w"), py::arg("ptrs"), py::arg("rank"),
        py::arg("epoch"), py::arg("ticket"), py::arg("xidx"), py::arg("part_off"), py::arg("splits"),
        py::arg("bt"), py::arg("status") = py::none(), py::arg("wn") = 0, py::arg("pull") = false);
  m.def("tp_signal", &tp_signal);
  m.def("add_rmsnorm_tp", &add_rmsnorm_tp, py::arg("ptrs"), py::arg("rank"), py::arg("epoch"), py::arg("x"),
        py::arg("part_off"), py::arg("nsplit"), py::arg("residual"), py::arg("w"), py::arg("out"), py::arg("eps"),
        py::arg("status") = py::none(), py::arg("pull") = false);
  m.def("tp_publish_topk", &tp_publish_topk);
  m.def("fsdp_signal", &fsdp_signal);
  m.def("fsdp_reduce", &fsdp_reduce);
  m.def("fsdp_update", &fsdp_update);
  m.def("fsdp_wait", &fsdp_wait);
  m.def("topk_merge_tp", &topk_merge_tp, py::arg("ptrs"), py::arg("rank"), py::arg("epoch"), py::arg("x"),
        py::arg("cand_off"), py::arg("M"), py::arg("k"), py::arg("ov"), py::arg("oi"), py::arg("status") = py::none());
}
