// C entry points of the linear kernels: pick the CUDA-core streaming kernel
// for small M and the tcgen05 tensor-core kernel above it.
#include <cstdlib>

#include "linear.cuh"

namespace {

// Largest M served by the CUDA-core streaming kernel; above it the tcgen05
// kernel runs. PS_SIMT_MAX_M overrides it (tuning).
int simt_max_m() {
  static const int v = [] {
    const char* e = std::getenv("PS_SIMT_MAX_M");
    return e ? std::atoi(e) : 1;
  }();
  return v;
}

int linear_any(void* y, const void* x, const void* w, int wdtype, const float* scale, const void* bias,
               const void* resid, int M, int N, int K, int dtype, void* ws, size_t ws_bytes, ps_stream_t stream,
               const char* name) {
  if (M < 0 || N <= 0 || K <= 0) {
    ps_host::set_error("%s: invalid sizes M=%d N=%d K=%d", name, M, N, K);
    return PS_ERR_INVALID;
  }
  if (!y || !x || !w) {
    ps_host::set_error("%s: null pointer", name);
    return PS_ERR_INVALID;
  }
  if (M == 0) return PS_OK;
  if (!ps_host::aligned(y, 4) || !ps_host::aligned(x, 16) || !ps_host::aligned(w, 16) ||
      !ps_host::aligned(resid, 4) || !ps_host::aligned(bias, 4)) {
    ps_host::set_error("%s: x and w must be 16-byte aligned", name);
    return PS_ERR_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (wdtype == PS_I8 && M <= ps_host::mma_max_m() && dtype != PS_F32 && ps_host::aligned(resid, 2) &&
      ps_host::aligned(bias, 2)) {
    const int rc = ps_host::linear_mma(y, x, static_cast<const int8_t*>(w), false, scale, bias, resid, M, N, K, dtype,
                                       false, s);
    if (rc != PS_ERR_UNSUPPORTED) return rc;
  }
  if (M > simt_max_m() && dtype != PS_F32) {
    const int rc = ps_host::linear_tc(y, x, w, wdtype, scale, bias, resid, M, N, K, dtype, ws, ws_bytes, s);
    if (rc != PS_ERR_UNSUPPORTED) return rc;
  }
  return ps_host::linear_simt(y, x, w, wdtype, scale, bias, resid, M, N, K, dtype, s);
}

}  // namespace

namespace ps_host {
int mma_max_m() {
  static const int v = [] {
    const char* e = std::getenv("PS_MMA_MAX_M");
    const int m = e ? std::atoi(e) : kMmaDefaultMaxM;
    return m < 0 ? 0 : (m > kMmaMaxM ? kMmaMaxM : m);
  }();
  return v;
}
}  // namespace ps_host

extern "C" {

size_t ps_w8a16_linear_workspace_size(int M, int N, int K) {
  return M > simt_max_m() ? ps_host::linear_tc_workspace(M, N, K) : 0;
}

int ps_w8a16_linear(void* y, const void* x, const int8_t* q, const float* scale, const void* bias,
                    const void* resid, int M, int N, int K, int dtype, void* ws, size_t ws_bytes,
                    ps_stream_t stream) {
  if (!scale) {
    ps_host::set_error("w8a16_linear: scale is NULL");
    return PS_ERR_INVALID;
  }
  return linear_any(y, x, q, PS_I8, scale, bias, resid, M, N, K, dtype, ws, ws_bytes, stream, "w8a16_linear");
}

size_t ps_tiled_int8_weight_bytes(int N, int K) { return N > 0 && K > 0 ? ps_host::tiled_int8_bytes(N, K) : 0; }

int ps_tile_int8_weight(int8_t* dst, const int8_t* q, int N, int K, ps_stream_t stream) {
  if (N <= 0 || K <= 0 || !dst || !q || !ps_host::aligned(dst, 16)) {
    ps_host::set_error("tile_int8_weight: invalid arguments");
    return PS_ERR_INVALID;
  }
  return ps_host::tile_int8(dst, q, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int ps_w8a16_linear_tiled(void* y, const void* x, const int8_t* q_tiled, const float* scale, const void* bias,
                          const void* resid, int M, int N, int K, int dtype, void* ws, size_t ws_bytes,
                          ps_stream_t stream) {
  if (M < 0 || N <= 0 || K <= 0 || !y || !x || !q_tiled || !scale) {
    ps_host::set_error("w8a16_linear_tiled: invalid arguments (M=%d N=%d K=%d)", M, N, K);
    return PS_ERR_INVALID;
  }
  if (M == 0) return PS_OK;
  if (dtype != PS_BF16 && dtype != PS_F16) {
    ps_host::set_error("w8a16_linear_tiled: dtype must be bf16 or f16");
    return PS_ERR_UNSUPPORTED;
  }
  if (!ps_host::aligned(y, 16) || !ps_host::aligned(x, 16) || !ps_host::aligned(q_tiled, 16) ||
      !ps_host::aligned(scale, 16) || !ps_host::aligned(resid, 16) || !ps_host::aligned(bias, 16) || K % 16 != 0) {
    ps_host::set_error("w8a16_linear_tiled: tensors must be 16-byte aligned and K a multiple of 16");
    return PS_ERR_INVALID;
  }
  if (M <= ps_host::mma_max_m()) {
    const int rc = ps_host::linear_mma(y, x, q_tiled, true, scale, bias, resid, M, N, K, dtype, false,
                                       reinterpret_cast<cudaStream_t>(stream));
    if (rc != PS_ERR_UNSUPPORTED) return rc;
  }
  return ps_host::linear_tc(y, x, q_tiled, PS_I8, scale, bias, resid, M, N, K, dtype, ws, ws_bytes,
                            reinterpret_cast<cudaStream_t>(stream), q_tiled);
}

size_t ps_w8a16_linear_tiled_workspace_size(int M, int N, int K) { return ps_host::linear_tc_workspace(M, N, K); }

static int linear_push_any(const void* x, const void* w, int wdtype, const int8_t* w_tiled, const float* scale,
                           int M, int N, int K, int dtype, void* const* rank_bufs, int world, int rank, int set,
                           int max_tokens, void* ws, size_t ws_bytes, ps_stream_t stream, bool scatter) {
  const bool int8 = wdtype == PS_I8;
  if (M <= 0 || N <= 0 || K <= 0 || M > max_tokens || !x || (int8 ? (!w_tiled || !scale) : !w)) {
    ps_host::set_error("linear_push: invalid arguments (M=%d N=%d K=%d max_tokens=%d)", M, N, K, max_tokens);
    return PS_ERR_INVALID;
  }
  if ((dtype != PS_BF16 && dtype != PS_F16) || (!int8 && wdtype != dtype)) {
    ps_host::set_error("linear_push: bf16/f16 activations with int8 or same-type weights");
    return PS_ERR_UNSUPPORTED;
  }
  if (!ps_host::aligned(x, 16) || !ps_host::aligned(w, 16) || !ps_host::aligned(w_tiled, 16) ||
      !ps_host::aligned(scale, 16) || K % 16 != 0 || N % 8 != 0) {
    ps_host::set_error("linear_push: tensors must be 16-byte aligned, K a multiple of 16, N of 8");
    return PS_ERR_INVALID;
  }
  ps::PushTargets pt;
  const int rc = ps_host::push_targets(&pt, rank_bufs, world, rank, set, max_tokens, N, 2, scatter);
  if (rc != PS_OK) return rc;
  const int8_t* wt = int8 ? w_tiled : nullptr;
  if (int8 && M <= ps_host::mma_max_m()) {
    const int r1 = ps_host::linear_mma(nullptr, x, w_tiled, true, scale, nullptr, nullptr, M, N, K, dtype, false,
                                       reinterpret_cast<cudaStream_t>(stream), &pt);
    if (r1 != PS_ERR_UNSUPPORTED) return r1;
  }
  const int r2 = ps_host::linear_tc(nullptr, x, int8 ? static_cast<const void*>(w_tiled) : w, wdtype, scale, nullptr,
                                    nullptr, M, N, K, dtype, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream),
                                    wt, &pt);
  if (r2 == PS_ERR_UNSUPPORTED) ps_host::set_error("linear_push: no tensor-core configuration for this shape");
  return r2;
}

int ps_linear_push(const void* x, const void* w, int wdtype, const int8_t* w_tiled, const float* scale, int M, int N,
                   int K, int dtype, void* const* rank_bufs, int world, int rank, int set, int max_tokens, void* ws,
                   size_t ws_bytes, ps_stream_t stream) {
  return linear_push_any(x, w, wdtype, w_tiled, scale, M, N, K, dtype, rank_bufs, world, rank, set, max_tokens, ws,
                         ws_bytes, stream, false);
}

int ps_linear_push_scatter(const void* x, const void* w, int wdtype, const int8_t* w_tiled, const float* scale, int M,
                           int N, int K, int dtype, void* const* rank_bufs, int world, int rank, int set,
                           int max_tokens, void* ws, size_t ws_bytes, ps_stream_t stream) {
  return linear_push_any(x, w, wdtype, w_tiled, scale, M, N, K, dtype, rank_bufs, world, rank, set, max_tokens, ws,
                         ws_bytes, stream, true);
}

int ps_linear_swiglu(void* y, const void* x, const void* w, int wdtype, const int8_t* w_tiled, const float* scale,
                     int M, int N2, int K, int dtype, ps_stream_t stream) {
  const bool int8 = wdtype == PS_I8;
  if (M < 0 || N2 <= 0 || K <= 0 || !y || !x || (int8 ? (!w_tiled || !scale) : !w)) {
    ps_host::set_error("linear_swiglu: invalid arguments (M=%d N2=%d K=%d)", M, N2, K);
    return PS_ERR_INVALID;
  }
  if (M == 0) return PS_OK;
  if ((dtype != PS_BF16 && dtype != PS_F16) || (!int8 && wdtype != dtype)) {
    ps_host::set_error("linear_swiglu: bf16/f16 activations with int8 or same-type weights");
    return PS_ERR_UNSUPPORTED;
  }
  if (N2 % 16 != 0 || K % 16 != 0 || !ps_host::aligned(y, 16) || !ps_host::aligned(x, 16) ||
      !ps_host::aligned(w, 16) || !ps_host::aligned(w_tiled, 16) || !ps_host::aligned(scale, 16)) {
    ps_host::set_error("linear_swiglu: 2*intermediate must be a multiple of 16, K of 16, tensors 16-byte aligned");
    return PS_ERR_INVALID;
  }
  if (int8 && M <= ps_host::mma_max_m()) {
    const int r1 = ps_host::linear_mma(y, x, w_tiled, true, scale, nullptr, nullptr, M, N2, K, dtype, true,
                                       reinterpret_cast<cudaStream_t>(stream));
    if (r1 != PS_ERR_UNSUPPORTED) return r1;
  }
  const int rc = ps_host::linear_tc(y, x, int8 ? static_cast<const void*>(w_tiled) : w, wdtype, scale, nullptr,
                                    nullptr, M, N2, K, dtype, nullptr, 0, reinterpret_cast<cudaStream_t>(stream),
                                    int8 ? w_tiled : nullptr, nullptr, true);
  if (rc == PS_ERR_UNSUPPORTED) ps_host::set_error("linear_swiglu: no tensor-core configuration for this shape");
  return rc;
}

int ps_linear(void* y, const void* x, const void* w, const void* bias, const void* resid, int M, int N, int K,
              int dtype, void* ws, size_t ws_bytes, ps_stream_t stream) {
  return linear_any(y, x, w, dtype, nullptr, bias, resid, M, N, K, dtype, ws, ws_bytes, stream, "linear");
}

}  // extern "C"
