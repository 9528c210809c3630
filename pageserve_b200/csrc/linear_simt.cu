// Weight-streaming linear on CUDA cores for small M (decode of a few
// sequences): y[m,n] = scale[n] * sum_k x[m,k] * w[n,k] + bias[n] + resid[m,n]
// (engine/quantization.py:26-50 + F.linear at engine/model.py:168-193 of the
// reference). Bandwidth bound: every weight byte is read once with 16-byte
// loads; int8 is widened in registers (never materialised), fp32 accumulate,
// the per-channel scale is applied once per output after the K reduction.
//
// Each warp owns kRowsPerWarp output rows and strides K in 16-byte lane
// chunks; activations (a few KB) come through L1.
#include "common.cuh"
#include "linear.cuh"

namespace {

using namespace ps;

constexpr int kWarpsPerCta = 8;
constexpr int kRowsPerWarp = 2;
constexpr int kMaxTok = 8;

// 16 int8 -> 16 floats. Byte b maps to float 2^23 + (b ^ 0x80) through the
// exponent field; subtracting 2^23 + 128 recovers the signed value exactly.
PS_DEVICE void widen16(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x ^ 0x80808080u, u.y ^ 0x80808080u, u.z ^ 0x80808080u, u.w ^ 0x80808080u};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t bits = __byte_perm(w[j], 0x4B000000u, 0x7640u | i);  // [byte i, 0, 0, 0x4B]
      f[j * 4 + i] = __uint_as_float(bits) - 8388736.0f;
    }
  }
}

template <typename TW>
struct WTraits;
template <>
struct WTraits<int8_t> {
  static constexpr int kElems = 16;
  static PS_DEVICE void load(const int8_t* p, float* f) { widen16(*reinterpret_cast<const uint4*>(p), f); }
};
template <>
struct WTraits<__nv_bfloat16> {
  static constexpr int kElems = 8;
  static PS_DEVICE void load(const __nv_bfloat16* p, float* f) { unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(p), f); }
};
template <>
struct WTraits<__half> {
  static constexpr int kElems = 8;
  static PS_DEVICE void load(const __half* p, float* f) { unpack8<__half>(*reinterpret_cast<const uint4*>(p), f); }
};

template <typename TX>
PS_DEVICE void load_x(const TX* p, float* f, int n) {
#pragma unroll
  for (int c = 0; c < n; c += 8) {
    if constexpr (sizeof(TX) == 4) {
      const float4 a = *reinterpret_cast<const float4*>(p + c);
      const float4 b = *reinterpret_cast<const float4*>(p + c + 4);
      f[c + 0] = a.x; f[c + 1] = a.y; f[c + 2] = a.z; f[c + 3] = a.w;
      f[c + 4] = b.x; f[c + 5] = b.y; f[c + 6] = b.z; f[c + 7] = b.w;
    } else {
      unpack8<TX>(*reinterpret_cast<const uint4*>(p + c), f + c);
    }
  }
}

template <typename TX, typename TW, int MT>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
    linear_simt_kernel(TX* __restrict__ y, const TX* __restrict__ x, const TW* __restrict__ w,
                       const float* __restrict__ scale, const TX* __restrict__ bias, const TX* __restrict__ resid,
                       int M, int N, int K) {
  constexpr int E = WTraits<TW>::kElems;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = (blockIdx.x * kWarpsPerCta + warp) * kRowsPerWarp;
  if (n0 >= N) return;
  for (int m0 = blockIdx.y * MT; m0 < M; m0 += gridDim.y * MT) {
    float acc[kRowsPerWarp][MT];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
      for (int t = 0; t < MT; ++t) acc[r][t] = 0.f;
    for (int k = lane * E; k < K; k += 32 * E) {
      float wf[kRowsPerWarp][E];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        if (n0 + r < N) WTraits<TW>::load(w + static_cast<long long>(n0 + r) * K + k, wf[r]);
        else
#pragma unroll
          for (int i = 0; i < E; ++i) wf[r][i] = 0.f;
      }
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        if (m0 + t < M) {
          float xf[E];
          load_x<TX>(x + static_cast<long long>(m0 + t) * K + k, xf, E);
#pragma unroll
          for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
            for (int i = 0; i < E; ++i) acc[r][t] = fmaf(xf[i], wf[r][i], acc[r][t]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
      for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum(acc[r][t]);
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const int n = n0 + r;
        if (n >= N) continue;
        const float sc = scale ? scale[n] : 1.f;
        const float bs = bias ? to_f32(bias[n]) : 0.f;
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const int m = m0 + t;
          if (m >= M) continue;
          float v = acc[r][t] * sc + bs;
          if (resid) {
            // the reference adds the residual to the dtype-rounded product
            v = to_f32(from_f32<TX>(v)) + to_f32(resid[static_cast<long long>(m) * N + n]);
          }
          y[static_cast<long long>(m) * N + n] = from_f32<TX>(v);
        }
      }
    }
  }
}

template <typename TX, typename TW>
int launch_simt(void* y, const void* x, const void* w, const float* scale, const void* bias, const void* resid, int M,
                int N, int K, cudaStream_t s) {
  constexpr int MT = kMaxTok;
  const int rows_per_cta = kWarpsPerCta * kRowsPerWarp;
  dim3 grid((N + rows_per_cta - 1) / rows_per_cta, 1);
  // spread token groups over grid.y only when N alone cannot fill the GPU
  const int mgroups = (M + MT - 1) / MT;
  int gy = 1;
  while (gy < mgroups && static_cast<long long>(grid.x) * gy < 148LL * 8) ++gy;
  grid.y = gy;
  if (M <= 1) {
    linear_simt_kernel<TX, TW, 1><<<grid, kWarpsPerCta * 32, 0, s>>>(
        static_cast<TX*>(y), static_cast<const TX*>(x), static_cast<const TW*>(w), scale,
        static_cast<const TX*>(bias), static_cast<const TX*>(resid), M, N, K);
  } else if (M <= 4) {
    linear_simt_kernel<TX, TW, 4><<<grid, kWarpsPerCta * 32, 0, s>>>(
        static_cast<TX*>(y), static_cast<const TX*>(x), static_cast<const TW*>(w), scale,
        static_cast<const TX*>(bias), static_cast<const TX*>(resid), M, N, K);
  } else {
    linear_simt_kernel<TX, TW, MT><<<grid, kWarpsPerCta * 32, 0, s>>>(
        static_cast<TX*>(y), static_cast<const TX*>(x), static_cast<const TW*>(w), scale,
        static_cast<const TX*>(bias), static_cast<const TX*>(resid), M, N, K);
  }
  ps_host::count_launch();
  return ps_host::check_launch("linear_simt");
}

}  // namespace

namespace ps_host {

int linear_simt(void* y, const void* x, const void* w, int wdtype, const float* scale, const void* bias,
                const void* resid, int M, int N, int K, int dtype, cudaStream_t s) {
  const int e = wdtype == PS_I8 ? 16 : 8;
  if (K % e != 0) {
    set_error("linear: in_features %d must be a multiple of %d", K, e);
    return PS_ERR_UNSUPPORTED;
  }
  if (wdtype == PS_I8) {
    switch (dtype) {
      case PS_F32: return launch_simt<float, int8_t>(y, x, w, scale, bias, resid, M, N, K, s);
      case PS_BF16: return launch_simt<__nv_bfloat16, int8_t>(y, x, w, scale, bias, resid, M, N, K, s);
      case PS_F16: return launch_simt<__half, int8_t>(y, x, w, scale, bias, resid, M, N, K, s);
    }
  } else if (wdtype == PS_BF16 && dtype == PS_BF16) {
    return launch_simt<__nv_bfloat16, __nv_bfloat16>(y, x, w, scale, bias, resid, M, N, K, s);
  } else if (wdtype == PS_F16 && dtype == PS_F16) {
    return launch_simt<__half, __half>(y, x, w, scale, bias, resid, M, N, K, s);
  }
  set_error("linear: unsupported dtype combination (x %d, w %d)", dtype, wdtype);
  return PS_ERR_UNSUPPORTED;
}

}  // namespace ps_host
