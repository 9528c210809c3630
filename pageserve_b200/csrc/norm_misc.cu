// Residual + RMSNorm, embedding gather, greedy argmax, SwiGLU gating and
// on-device per-channel int8 quantization (engine/model.py:29-34, 159,
// 184-193; engine/quantization.py:16-23; server.py:51 of the reference).
// All HBM-bound, one pass over the data, 16-byte vector accesses.
#include <cfloat>

#include "common.cuh"

namespace {

using namespace ps;

constexpr int kNormThreads = 256;

// One CTA per row. r = x (+ residual, rounded to T) ; y = r * rsqrt(mean(r^2)+eps) * w.
template <typename T, int MAXV>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(T* __restrict__ y, T* __restrict__ resid_out,
                                                               const T* __restrict__ x, const T* __restrict__ resid,
                                                               const T* __restrict__ w, float eps, int H) {
  pdl_wait();
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T);
  const int row = blockIdx.x;
  const int nvec = H / VEC;
  const T* xr = x + static_cast<long long>(row) * H;
  float v[MAXV][VEC];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int c = threadIdx.x + j * kNormThreads;
    if (c < nvec) {
      uint4 u = reinterpret_cast<const uint4*>(xr)[c];
      const T* xe = reinterpret_cast<const T*>(&u);
      if (resid) {
        uint4 ru = reinterpret_cast<const uint4*>(resid + static_cast<long long>(row) * H)[c];
        const T* re = reinterpret_cast<const T*>(&ru);
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          oe[i] = from_f32<T>(to_f32(xe[i]) + to_f32(re[i]));
          v[j][i] = to_f32(oe[i]);
        }
        if (resid_out) reinterpret_cast<uint4*>(resid_out + static_cast<long long>(row) * H)[c] = o;
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) v[j][i] = to_f32(xe[i]);
      }
#pragma unroll
      for (int i = 0; i < VEC; ++i) ss += v[j][i] * v[j][i];
    }
  }
  __shared__ float red[kNormThreads / 32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / static_cast<float>(H) + eps);
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int c = threadIdx.x + j * kNormThreads;
    if (c < nvec) {
      uint4 wu = reinterpret_cast<const uint4*>(w)[c];
      const T* we = reinterpret_cast<const T*>(&wu);
      float o[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) o[i] = v[j][i] * inv * to_f32(we[i]);
      uint4 ou;
      T* oe = reinterpret_cast<T*>(&ou);
#pragma unroll
      for (int i = 0; i < VEC; ++i) oe[i] = from_f32<T>(o[i]);
      reinterpret_cast<uint4*>(y + static_cast<long long>(row) * H)[c] = ou;
    }
  }
}

template <typename T>
__global__ void embedding_kernel(T* __restrict__ out, const int64_t* __restrict__ ids, const T* __restrict__ table,
                                 int H, int vocab, int* status) {
  pdl_wait();
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T);
  const int t = blockIdx.x;
  const long long id = ids[t];
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(t) * H);
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) record_error(status, kErrTokenId);
    for (int c = threadIdx.x; c < H / VEC; c += blockDim.x) dst[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + id * H);
  for (int c = threadIdx.x; c < H / VEC; c += blockDim.x) dst[c] = src[c];
}

// First index of the row maximum (torch.argmax semantics for finite input).
// One CTA per row; 16-byte loads, four in flight per thread (the row is read
// once, HBM bound), then a (value, index) tree reduction with first-index
// tie-breaking.
PS_DEVICE void argmax_merge(float& best, int& bidx, float ob, int oi) {
  if (ob > best || (ob == best && oi < bidx)) {
    best = ob;
    bidx = oi;
  }
}

template <typename T>
__global__ void __launch_bounds__(1024) argmax_kernel(int32_t* __restrict__ out, const T* __restrict__ logits,
                                                      int V, int ld) {
  pdl_wait();
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T);
  const int row = blockIdx.x;
  const T* lr = logits + static_cast<long long>(row) * ld;
  float best = -FLT_MAX;
  int bidx = 0x7fffffff;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(lr) % 16) == 0;
  int tail = 0;
  if (vec_ok) {
    const int nv = V / VEC;
    const uint4* lv = reinterpret_cast<const uint4*>(lr);
    constexpr int U = 4;
    for (int base = threadIdx.x; base < nv; base += blockDim.x * U) {
      uint4 u[U];
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const int c = base + j * blockDim.x;
        u[j] = c < nv ? __ldg(lv + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const int c = base + j * blockDim.x;
        if (c < nv) {
          const T* e = reinterpret_cast<const T*>(&u[j]);
#pragma unroll
          for (int i = 0; i < VEC; ++i) argmax_merge(best, bidx, to_f32(e[i]), c * VEC + i);
        }
      }
    }
    tail = nv * VEC;
  }
  for (int i = tail + threadIdx.x; i < V; i += blockDim.x) argmax_merge(best, bidx, to_f32(lr[i]), i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
    argmax_merge(best, bidx, ob, oi);
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sb[warp] = best;
    si[warp] = bidx;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -FLT_MAX;
    bidx = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
      argmax_merge(best, bidx, ob, oi);
    }
    if (lane == 0) out[row] = bidx == 0x7fffffff ? 0 : bidx;
  }
}

template <typename T>
__global__ void silu_mul_kernel(T* __restrict__ out, const T* __restrict__ gu, int M, int I) {
  constexpr int VEC = 16 / sizeof(T);
  const long long nv = static_cast<long long>(M) * (I / VEC);
  for (long long w = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; w < nv;
       w += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long m = w / (I / VEC);
    const int c = static_cast<int>(w - m * (I / VEC));
    const uint4 gvec = reinterpret_cast<const uint4*>(gu + m * 2 * I)[c];
    const uint4 uvec = reinterpret_cast<const uint4*>(gu + m * 2 * I + I)[c];
    float g[VEC], u[VEC], o[VEC];
    unpack8<T>(gvec, g);
    unpack8<T>(uvec, u);
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = silu_mul_f32(g[i], u[i]);
    reinterpret_cast<uint4*>(out + m * I)[c] = pack8<T>(o);
  }
}

// quantize_per_channel: one CTA per output row.
template <typename T>
__global__ void quantize_kernel(int8_t* __restrict__ q, float* __restrict__ scale, const T* __restrict__ w, int K) {
  const int n = blockIdx.x;
  const T* wr = w + static_cast<long long>(n) * K;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(to_f32(wr[k])));
  amax = warp_max(amax);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float s = fmaxf(red[0], 1e-8f) / 127.0f;  // IEEE division, as torch
  if (threadIdx.x == 0) scale[n] = s;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float r = rintf(to_f32(wr[k]) / s);
    r = fminf(fmaxf(r, -127.f), 127.f);
    q[static_cast<long long>(n) * K + k] = static_cast<int8_t>(r);
  }
}

int vec_of(int dtype) { return dtype == PS_F32 ? 4 : 8; }

}  // namespace

extern "C" {

int ps_rmsnorm(void* y, void* resid_out, const void* x, const void* resid, const void* w, float eps, int M, int H,
               int dtype, ps_stream_t stream) {
  if (M < 0 || H <= 0 || !y || !x || !w) {
    ps_host::set_error("rmsnorm: invalid arguments");
    return PS_ERR_INVALID;
  }
  if (M == 0) return PS_OK;
  const int vec = vec_of(dtype);
  if (H % vec != 0) {
    ps_host::set_error("rmsnorm: hidden size %d not a multiple of %d", H, vec);
    return PS_ERR_UNSUPPORTED;
  }
  if (!ps_host::aligned(y, 16) || !ps_host::aligned(resid_out, 16) || !ps_host::aligned(x, 16) ||
      !ps_host::aligned(resid, 16) || !ps_host::aligned(w, 16)) {
    ps_host::set_error("rmsnorm: tensors must be 16-byte aligned");
    return PS_ERR_INVALID;
  }
  const int nvec = H / vec;
  const int per_thread = (nvec + kNormThreads - 1) / kNormThreads;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
#define PS_NORM(T, MV)                                                                                     \
  ps_host::launch(rmsnorm_kernel<T, MV>, M, kNormThreads, 0, s, static_cast<T*>(y), static_cast<T*>(resid_out),        \
                                                    static_cast<const T*>(x), static_cast<const T*>(resid), \
                                                    static_cast<const T*>(w), eps, H)
#define PS_NORM_T(T)            \
  if (per_thread <= 1) PS_NORM(T, 1); \
  else if (per_thread <= 2) PS_NORM(T, 2); \
  else if (per_thread <= 4) PS_NORM(T, 4); \
  else if (per_thread <= 8) PS_NORM(T, 8); \
  else { ps_host::set_error("rmsnorm: hidden size %d too large", H); return PS_ERR_UNSUPPORTED; }
  switch (dtype) {
    case PS_F32: PS_NORM_T(float); break;
    case PS_BF16: PS_NORM_T(__nv_bfloat16); break;
    case PS_F16: PS_NORM_T(__half); break;
    default: ps_host::set_error("rmsnorm: unsupported dtype"); return PS_ERR_UNSUPPORTED;
  }
#undef PS_NORM_T
#undef PS_NORM
  ps_host::count_launch();
  return ps_host::check_launch("rmsnorm");
}

int ps_embedding(void* out, const int64_t* ids, const void* table, int T, int H, int vocab, int dtype,
                 ps_stream_t stream) {
  if (T < 0 || H <= 0 || H % vec_of(dtype) != 0) {
    ps_host::set_error("embedding: invalid sizes");
    return PS_ERR_INVALID;
  }
  if (T == 0) return PS_OK;
  if (!ps_host::aligned(out, 16) || !ps_host::aligned(table, 16) || !ps_host::aligned(ids, 8)) {
    ps_host::set_error("embedding: out/table must be 16-byte aligned");
    return PS_ERR_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* st = ps_host::status_word(PS_TU_MISC);
  switch (dtype) {
    case PS_F32: ps_host::launch(embedding_kernel<float>, T, 128, 0, s, static_cast<float*>(out), ids, static_cast<const float*>(table), H, vocab, st); break;
    case PS_BF16: ps_host::launch(embedding_kernel<__nv_bfloat16>, T, 128, 0, s, static_cast<__nv_bfloat16*>(out), ids, static_cast<const __nv_bfloat16*>(table), H, vocab, st); break;
    case PS_F16: ps_host::launch(embedding_kernel<__half>, T, 128, 0, s, static_cast<__half*>(out), ids, static_cast<const __half*>(table), H, vocab, st); break;
    default: ps_host::set_error("embedding: unsupported dtype"); return PS_ERR_UNSUPPORTED;
  }
  ps_host::count_launch();
  return ps_host::check_launch("embedding");
}

int ps_argmax(int32_t* out, const void* logits, int M, int V, int ld, int dtype, ps_stream_t stream) {
  if (M < 0 || V <= 0 || ld < V) {
    ps_host::set_error("argmax: invalid sizes");
    return PS_ERR_INVALID;
  }
  if (M == 0) return PS_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PS_F32: ps_host::launch(argmax_kernel<float>, M, 1024, 0, s, out, static_cast<const float*>(logits), V, ld); break;
    case PS_BF16: ps_host::launch(argmax_kernel<__nv_bfloat16>, M, 1024, 0, s, out, static_cast<const __nv_bfloat16*>(logits), V, ld); break;
    case PS_F16: ps_host::launch(argmax_kernel<__half>, M, 1024, 0, s, out, static_cast<const __half*>(logits), V, ld); break;
    default: ps_host::set_error("argmax: unsupported dtype"); return PS_ERR_UNSUPPORTED;
  }
  ps_host::count_launch();
  return ps_host::check_launch("argmax");
}

int ps_silu_mul(void* out, const void* gu, int M, int I, int dtype, ps_stream_t stream) {
  if (M < 0 || I <= 0 || I % 8 != 0) {
    ps_host::set_error("silu_mul: intermediate size must be a multiple of 8");
    return PS_ERR_INVALID;
  }
  if (M == 0) return PS_OK;
  if (!ps_host::aligned(out, 16) || !ps_host::aligned(gu, 16)) {
    ps_host::set_error("silu_mul: tensors must be 16-byte aligned");
    return PS_ERR_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long nv = static_cast<long long>(M) * I / 8;
  long long g = (nv + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  switch (dtype) {
    case PS_BF16: silu_mul_kernel<__nv_bfloat16><<<static_cast<int>(g), 256, 0, s>>>(static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(gu), M, I); break;
    case PS_F16: silu_mul_kernel<__half><<<static_cast<int>(g), 256, 0, s>>>(static_cast<__half*>(out), static_cast<const __half*>(gu), M, I); break;
    default: ps_host::set_error("silu_mul: dtype must be bf16 or f16"); return PS_ERR_UNSUPPORTED;
  }
  ps_host::count_launch();
  return ps_host::check_launch("silu_mul");
}

int ps_quantize_per_channel(int8_t* q, float* scale, const void* w, int dtype, int N, int K, ps_stream_t stream) {
  if (N < 0 || K <= 0) {
    ps_host::set_error("quantize_per_channel: invalid sizes");
    return PS_ERR_INVALID;
  }
  if (N == 0) return PS_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PS_F32: quantize_kernel<float><<<N, 256, 0, s>>>(q, scale, static_cast<const float*>(w), K); break;
    case PS_BF16: quantize_kernel<__nv_bfloat16><<<N, 256, 0, s>>>(q, scale, static_cast<const __nv_bfloat16*>(w), K); break;
    case PS_F16: quantize_kernel<__half><<<N, 256, 0, s>>>(q, scale, static_cast<const __half*>(w), K); break;
    default: ps_host::set_error("quantize_per_channel: unsupported dtype"); return PS_ERR_UNSUPPORTED;
  }
  ps_host::count_launch();
  return ps_host::check_launch("quantize_per_channel");
}

}  // extern "C"
