// C entry points of the linear kernels: pick the CUDA-core streaming kernel
// for small M and the tcgen05 tensor-core kernel above it.
#include "linear.cuh"

namespace {

constexpr int kSimtMaxM = 16;

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
  if (M > kSimtMaxM && dtype != PS_F32) {
    const int rc = ps_host::linear_tc(y, x, w, wdtype, scale, bias, resid, M, N, K, dtype, ws, ws_bytes, s);
    if (rc != PS_ERR_UNSUPPORTED) return rc;
  }
  return ps_host::linear_simt(y, x, w, wdtype, scale, bias, resid, M, N, K, dtype, s);
}

}  // namespace

extern "C" {

size_t ps_w8a16_linear_workspace_size(int M, int N, int K) {
  return M > kSimtMaxM ? ps_host::linear_tc_workspace(M, N, K) : 0;
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

int ps_linear(void* y, const void* x, const void* w, const void* bias, const void* resid, int M, int N, int K,
              int dtype, void* ws, size_t ws_bytes, ps_stream_t stream) {
  return linear_any(y, x, w, dtype, nullptr, bias, resid, M, N, K, dtype, ws, ws_bytes, stream, "linear");
}

}  // extern "C"
