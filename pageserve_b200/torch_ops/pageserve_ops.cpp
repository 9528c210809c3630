// torch.ops.pageserve_b200.* — the hot-path operators registered with the
// PyTorch dispatcher (CUDA kernels + Meta shape functions for tracing), each a
// thin call into the plain extern "C" core (include/pageserve_b200.h,
// libpageserve_b200.so). No CPU kernels are registered: a CPU tensor raises
// the dispatcher's "no kernel for CPU" error (no CPU fallback).
//
// Operator names and arguments follow the reference's Python functions
// (engine/paged_attention.py, engine/quantization.py, engine/model.py); the
// batched forms take device-resident int32 metadata (graph-capturable).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "../../include/pageserve_b200.h"

namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return PS_F32;
    case at::kBFloat16: return PS_BF16;
    case at::kHalf: return PS_F16;
    case at::kChar: return PS_I8;
    default: TORCH_CHECK(false, "pageserve_b200: unsupported dtype ", t.scalar_type());
  }
  return -1;
}

ps_stream_t stream_of(const at::Tensor& t) {
  return reinterpret_cast<ps_stream_t>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void check(int rc, const char* what) {
  if (rc == PS_OK) return;
  const char* msg = ps_last_error();
  TORCH_CHECK_INDEX(rc != PS_ERR_INDEX, what, ": ", msg);
  TORCH_CHECK_NOT_IMPLEMENTED(rc != PS_ERR_UNSUPPORTED, what, ": ", msg);
  TORCH_CHECK(false, what, " failed (", rc, "): ", msg);
}

void* ptr(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

void need_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "pageserve_b200: ", name, " must be a CUDA tensor (no CPU fallback)");
  TORCH_CHECK(t.is_contiguous(), "pageserve_b200: ", name, " must be contiguous");
}

// ---------------------------------------------------------------- CUDA ----

void write_kv(at::Tensor k_cache, at::Tensor v_cache, const at::Tensor& block_table, int64_t block_size,
              int64_t start_pos, const at::Tensor& k, const at::Tensor& v) {
  need_cuda(k_cache, "k_cache"); need_cuda(v_cache, "v_cache"); need_cuda(k, "k"); need_cuda(v, "v");
  need_cuda(block_table, "block_table");
  TORCH_CHECK(block_table.scalar_type() == at::kInt, "block_table must be int32");
  c10::cuda::CUDAGuard g(k_cache.device());
  check(ps_write_kv(k_cache.data_ptr(), v_cache.data_ptr(), block_table.data_ptr<int32_t>(), block_table.numel(),
                    k_cache.size(0), block_size, k_cache.size(2), k_cache.size(3), dtype_code(k), start_pos,
                    k.size(0), k.data_ptr(), v.data_ptr(), stream_of(k)),
        "write_kv");
}

at::Tensor paged_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                           const at::Tensor& block_tables, const at::Tensor& cu_q, const at::Tensor& start_pos,
                           int64_t max_q_len, int64_t max_ctx) {
  need_cuda(q, "q"); need_cuda(k_cache, "k_cache"); need_cuda(v_cache, "v_cache");
  need_cuda(block_tables, "block_tables"); need_cuda(cu_q, "cu_q"); need_cuda(start_pos, "start_pos");
  c10::cuda::CUDAGuard g(q.device());
  const int B = start_pos.numel(), Hq = q.size(1), D = q.size(2), Hkv = k_cache.size(2);
  at::Tensor out = at::empty_like(q);
  const size_t ws_bytes = ps_paged_attention_workspace_size(B, max_q_len, max_ctx, Hq, Hkv, D);
  at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes > 0 ? ws_bytes : 1)}, q.options().dtype(at::kByte));
  check(ps_paged_attention(out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                           block_tables.data_ptr<int32_t>(), block_tables.size(1), cu_q.data_ptr<int32_t>(),
                           start_pos.data_ptr<int32_t>(), B, q.size(0), max_q_len, max_ctx, k_cache.size(0),
                           k_cache.size(1), Hq, Hkv, D, dtype_code(q), ws.data_ptr(), ws_bytes, stream_of(q)),
        "paged_attention");
  return out;
}

std::tuple<at::Tensor, at::Tensor> quantize_per_channel(const at::Tensor& w) {
  need_cuda(w, "weight");
  c10::cuda::CUDAGuard g(w.device());
  at::Tensor q = at::empty({w.size(0), w.size(1)}, w.options().dtype(at::kChar));
  at::Tensor scale = at::empty({w.size(0), 1}, w.options().dtype(at::kFloat));
  check(ps_quantize_per_channel(q.data_ptr<int8_t>(), scale.data_ptr<float>(), w.data_ptr(), dtype_code(w),
                                w.size(0), w.size(1), stream_of(w)),
        "quantize_per_channel");
  return {q, scale};
}

at::Tensor tile_int8_weight(const at::Tensor& q) {
  need_cuda(q, "q");
  c10::cuda::CUDAGuard g(q.device());
  at::Tensor t = at::empty({static_cast<int64_t>(ps_tiled_int8_weight_bytes(q.size(0), q.size(1)))},
                           q.options().dtype(at::kChar));
  check(ps_tile_int8_weight(t.data_ptr<int8_t>(), q.data_ptr<int8_t>(), q.size(0), q.size(1), stream_of(q)),
        "tile_int8_weight");
  return t;
}

at::Tensor w8a16_linear(const at::Tensor& x, const at::Tensor& q_tiled, const at::Tensor& scale, int64_t N,
                        const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual) {
  need_cuda(x, "x"); need_cuda(q_tiled, "q_tiled"); need_cuda(scale, "scale");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t K = x.size(-1), M = x.numel() / K;
  auto sizes = x.sizes().vec();
  sizes.back() = N;
  at::Tensor y = at::empty(sizes, x.options());
  const size_t ws_bytes = ps_w8a16_linear_tiled_workspace_size(M, N, K);
  at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes > 0 ? ws_bytes : 1)}, x.options().dtype(at::kByte));
  check(ps_w8a16_linear_tiled(y.data_ptr(), x.data_ptr(), q_tiled.data_ptr<int8_t>(), scale.data_ptr<float>(),
                              ptr(bias), ptr(residual), M, N, K, dtype_code(x), ws.data_ptr(), ws_bytes,
                              stream_of(x)),
        "w8a16_linear");
  return y;
}

at::Tensor linear16(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                    const c10::optional<at::Tensor>& residual) {
  need_cuda(x, "x"); need_cuda(w, "w");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t K = x.size(-1), M = x.numel() / K, N = w.size(0);
  auto sizes = x.sizes().vec();
  sizes.back() = N;
  at::Tensor y = at::empty(sizes, x.options());
  const size_t ws_bytes = ps_w8a16_linear_tiled_workspace_size(M, N, K);
  at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes > 0 ? ws_bytes : 1)}, x.options().dtype(at::kByte));
  check(ps_linear(y.data_ptr(), x.data_ptr(), w.data_ptr(), ptr(bias), ptr(residual), M, N, K, dtype_code(x),
                  ws.data_ptr(), ws_bytes, stream_of(x)),
        "linear16");
  return y;
}

at::Tensor linear_swiglu(const at::Tensor& x, const at::Tensor& q_tiled, const at::Tensor& scale, int64_t N2) {
  need_cuda(x, "x"); need_cuda(q_tiled, "q_tiled"); need_cuda(scale, "scale");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t K = x.size(-1), M = x.numel() / K;
  auto sizes = x.sizes().vec();
  sizes.back() = N2 / 2;
  at::Tensor y = at::empty(sizes, x.options());
  check(ps_linear_swiglu(y.data_ptr(), x.data_ptr(), nullptr, PS_I8, q_tiled.data_ptr<int8_t>(),
                         scale.data_ptr<float>(), M, N2, K, dtype_code(x), stream_of(x)),
        "linear_swiglu");
  return y;
}

at::Tensor rms_norm(const at::Tensor& x, const at::Tensor& weight, double eps) {
  need_cuda(x, "x"); need_cuda(weight, "weight");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t H = x.size(-1);
  at::Tensor y = at::empty_like(x);
  at::Tensor w = weight.to(x.scalar_type()).contiguous();
  check(ps_rmsnorm(y.data_ptr(), nullptr, x.data_ptr(), nullptr, w.data_ptr(), static_cast<float>(eps),
                   x.numel() / H, H, dtype_code(x), stream_of(x)),
        "rms_norm");
  return y;
}

std::tuple<at::Tensor, at::Tensor> add_rms_norm(const at::Tensor& x, const at::Tensor& residual,
                                                const at::Tensor& weight, double eps) {
  need_cuda(x, "x"); need_cuda(residual, "residual"); need_cuda(weight, "weight");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t H = x.size(-1);
  at::Tensor y = at::empty_like(x), sum = at::empty_like(x);
  at::Tensor w = weight.to(x.scalar_type()).contiguous();
  check(ps_rmsnorm(y.data_ptr(), sum.data_ptr(), x.data_ptr(), residual.data_ptr(), w.data_ptr(),
                   static_cast<float>(eps), x.numel() / H, H, dtype_code(x), stream_of(x)),
        "add_rms_norm");
  return {y, sum};
}

at::Tensor apply_rope(const at::Tensor& x, const at::Tensor& cos, const at::Tensor& sin) {
  need_cuda(x, "x"); need_cuda(cos, "cos"); need_cuda(sin, "sin");
  c10::cuda::CUDAGuard g(x.device());
  at::Tensor out = at::empty_like(x);
  at::Tensor c = cos.to(x.scalar_type()).contiguous(), s = sin.to(x.scalar_type()).contiguous();
  check(ps_apply_rope(out.data_ptr(), x.data_ptr(), c.data_ptr(), s.data_ptr(), x.size(0), x.size(1), x.size(2),
                      dtype_code(x), stream_of(x)),
        "apply_rope");
  return out;
}

at::Tensor embedding(const at::Tensor& ids, const at::Tensor& table) {
  need_cuda(ids, "ids"); need_cuda(table, "table");
  TORCH_CHECK(ids.scalar_type() == at::kLong, "ids must be int64");
  c10::cuda::CUDAGuard g(table.device());
  at::Tensor out = at::empty({ids.numel(), table.size(1)}, table.options());
  check(ps_embedding(out.data_ptr(), ids.data_ptr<int64_t>(), table.data_ptr(), ids.numel(), table.size(1),
                     table.size(0), dtype_code(table), stream_of(table)),
        "embedding");
  return out;
}

at::Tensor argmax(const at::Tensor& logits) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "argmax: 2-D CUDA logits rows");
  c10::cuda::CUDAGuard g(logits.device());
  at::Tensor out = at::empty({logits.size(0)}, logits.options().dtype(at::kInt));
  check(ps_argmax(out.data_ptr<int32_t>(), logits.data_ptr(), logits.size(0), logits.size(1), logits.stride(0),
                  dtype_code(logits), stream_of(logits)),
        "argmax");
  return out;
}

std::tuple<at::Tensor, at::Tensor> topk(const at::Tensor& logits, int64_t k) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "topk: 2-D CUDA logits rows");
  c10::cuda::CUDAGuard g(logits.device());
  at::Tensor vals = at::empty({logits.size(0), k}, logits.options().dtype(at::kFloat));
  at::Tensor idx = at::empty({logits.size(0), k}, logits.options().dtype(at::kInt));
  check(ps_topk(vals.data_ptr<float>(), idx.data_ptr<int32_t>(), logits.data_ptr(), logits.size(0), logits.size(1),
                logits.stride(0), k, dtype_code(logits), stream_of(logits)),
        "topk");
  return {vals, idx};
}

void copy_kv_blocks(at::Tensor k_cache, at::Tensor v_cache, const at::Tensor& pairs) {
  need_cuda(k_cache, "k_cache"); need_cuda(v_cache, "v_cache"); need_cuda(pairs, "pairs");
  TORCH_CHECK(k_cache.dim() == 5 && pairs.scalar_type() == at::kInt, "copy_kv_blocks: (L, NB, bs, Hkv, D) caches, "
              "int32 (n, 2) pairs");
  c10::cuda::CUDAGuard g(k_cache.device());
  check(ps_copy_kv_blocks(k_cache.data_ptr(), v_cache.data_ptr(), pairs.data_ptr<int32_t>(), pairs.numel() / 2,
                          k_cache.size(0), k_cache.size(1), k_cache.size(2), k_cache.size(3), k_cache.size(4),
                          dtype_code(k_cache), stream_of(k_cache)),
        "copy_kv_blocks");
}

// ---------------------------------------------------------------- Meta ----
// Output shapes only (torch.compile / fake-tensor tracing).

at::Tensor paged_attention_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                const at::Tensor&, const at::Tensor&, int64_t, int64_t) {
  return at::empty_like(q);
}
std::tuple<at::Tensor, at::Tensor> quantize_meta(const at::Tensor& w) {
  return {at::empty({w.size(0), w.size(1)}, w.options().dtype(at::kChar)),
          at::empty({w.size(0), 1}, w.options().dtype(at::kFloat))};
}
at::Tensor w8a16_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&, int64_t N,
                      const c10::optional<at::Tensor>&, const c10::optional<at::Tensor>&) {
  auto s = x.sizes().vec();
  s.back() = N;
  return at::empty(s, x.options());
}
at::Tensor linear16_meta(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>&,
                         const c10::optional<at::Tensor>&) {
  auto s = x.sizes().vec();
  s.back() = w.size(0);
  return at::empty(s, x.options());
}
at::Tensor swiglu_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&, int64_t N2) {
  auto s = x.sizes().vec();
  s.back() = N2 / 2;
  return at::empty(s, x.options());
}
at::Tensor rms_norm_meta(const at::Tensor& x, const at::Tensor&, double) { return at::empty_like(x); }
std::tuple<at::Tensor, at::Tensor> add_rms_norm_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&,
                                                     double) {
  return {at::empty_like(x), at::empty_like(x)};
}
at::Tensor apply_rope_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&) { return at::empty_like(x); }
at::Tensor argmax_meta(const at::Tensor& l) { return at::empty({l.size(0)}, l.options().dtype(at::kInt)); }
std::tuple<at::Tensor, at::Tensor> topk_meta(const at::Tensor& l, int64_t k) {
  return {at::empty({l.size(0), k}, l.options().dtype(at::kFloat)),
          at::empty({l.size(0), k}, l.options().dtype(at::kInt))};
}

}  // namespace

TORCH_LIBRARY(pageserve_b200, m) {
  m.def("write_kv(Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor block_table, int block_size, int start_pos, "
        "Tensor k, Tensor v) -> ()");
  m.def("paged_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables, Tensor cu_q, "
        "Tensor start_pos, int max_q_len, int max_ctx) -> Tensor");
  m.def("quantize_per_channel(Tensor weight) -> (Tensor, Tensor)");
  m.def("tile_int8_weight(Tensor q) -> Tensor");
  m.def("w8a16_linear(Tensor x, Tensor q_tiled, Tensor scale, int N, Tensor? bias=None, Tensor? residual=None) "
        "-> Tensor");
  m.def("linear16(Tensor x, Tensor w, Tensor? bias=None, Tensor? residual=None) -> Tensor");
  m.def("linear_swiglu(Tensor x, Tensor q_tiled, Tensor scale, int N2) -> Tensor");
  m.def("rms_norm(Tensor x, Tensor weight, float eps) -> Tensor");
  m.def("add_rms_norm(Tensor x, Tensor residual, Tensor weight, float eps) -> (Tensor, Tensor)");
  m.def("apply_rope(Tensor x, Tensor cos, Tensor sin) -> Tensor");
  m.def("embedding(Tensor ids, Tensor table) -> Tensor");
  m.def("argmax(Tensor logits) -> Tensor");
  m.def("topk(Tensor logits, int k) -> (Tensor, Tensor)");
  m.def("copy_kv_blocks(Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor pairs) -> ()");
}

TORCH_LIBRARY_IMPL(pageserve_b200, CUDA, m) {
  m.impl("write_kv", &write_kv);
  m.impl("paged_attention", &paged_attention);
  m.impl("quantize_per_channel", &quantize_per_channel);
  m.impl("tile_int8_weight", &tile_int8_weight);
  m.impl("w8a16_linear", &w8a16_linear);
  m.impl("linear16", &linear16);
  m.impl("linear_swiglu", &linear_swiglu);
  m.impl("rms_norm", &rms_norm);
  m.impl("add_rms_norm", &add_rms_norm);
  m.impl("apply_rope", &apply_rope);
  m.impl("embedding", &embedding);
  m.impl("argmax", &argmax);
  m.impl("topk", &topk);
  m.impl("copy_kv_blocks", &copy_kv_blocks);
}

TORCH_LIBRARY_IMPL(pageserve_b200, Meta, m) {
  m.impl("paged_attention", &paged_attention_meta);
  m.impl("quantize_per_channel", &quantize_meta);
  m.impl("w8a16_linear", &w8a16_meta);
  m.impl("linear16", &linear16_meta);
  m.impl("linear_swiglu", &swiglu_meta);
  m.impl("rms_norm", &rms_norm_meta);
  m.impl("add_rms_norm", &add_rms_norm_meta);
  m.impl("apply_rope", &apply_rope_meta);
  m.impl("argmax", &argmax_meta);
  m.impl("topk", &topk_meta);
}
