// Small-M W8A16 linear (M <= 32 tokens: decode batches) on mma.sync, bound by
// the weight stream: y[m,n] = scale[n] * sum_k x[m,k] * q[n,k] + bias[n]
// (+ resid[m,n]) — engine/quantization.py:26-50 + F.linear at
// engine/model.py:168-193 — or, in SwiGLU mode (rows interleaved gate/up),
// y[m,i] = silu(gate) * up (engine/model.py:188-190).
//
// One CTA = 16 weight rows x all of K; its 8 warps take every 8th 64-wide
// k-tile and reduce through shared memory in warp order (deterministic).
// The int8 weight is read once, 16 bytes per lane (a 16-row x 64-byte tile
// slice is one contiguous 1 KB in the pre-tiled layout), widened exactly to
// bf16/f16 in registers and fed to m16n8k16 MMAs with the tokens as N.
// Inside each 64-wide k-tile the reduction order over k is permuted so that
// lane (g, c) owns physical k [16c, 16c+16) of rows g and g+8: for k-step s
// its logical MMA positions (2c, 2c+1, 2c+8, 2c+9) hold physical
// (16c+4s .. 16c+4s+3), in both A (weights) and B (activations), so every
// lane issues whole 16-byte loads and no data moves between lanes.
#include <cstdlib>
#include <cstring>

#include "linear.cuh"
#include "widen.cuh"

namespace {

using namespace ps;

constexpr int kKT = 64;

template <typename T>
PS_DEVICE void widen16(const uint4& in, uint4& lo, uint4& hi) {
  if constexpr (std::is_same<T, __half>::value) widen16_f16(in, lo, hi);
  else widen16_bf16(in, lo, hi);
}

PS_DEVICE uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// NT = 8-token MMA tiles (M <= 8 * NT); W = warps per CTA (they split K).
// tiled: q_tiled in 8 KB blocks [N/128][K/64][128][64] with chunk c of row r
// at slot c ^ ((r >> 1) & 3); else q row-major [N][K]. The grid strides over
// 16-row groups so every SM stays busy to the end; each warp keeps kDepth of
// its k-tiles' weight loads in flight ahead of the MMAs (deeper when few row
// groups leave fewer warps per SM).
template <typename T, int NT, int W, int kDepth>
__global__ void __launch_bounds__(W * 32) linear_mma_kernel(
    T* __restrict__ y, const T* __restrict__ x, const int8_t* __restrict__ q, int tiled,
    const float* __restrict__ scale, const T* __restrict__ bias, const T* __restrict__ resid, int M, int N, int K,
    int swiglu, const PushTargets push) {
  __shared__ float red[W][16][NT * 8 + 1];
  pdl_trigger();
  bool waited = false;  // the first weight loads go out before waiting for the previous kernel
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int k_tiles = (K + kKT - 1) / kKT;
  const int groups = (N + 15) / 16;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int rg = blockIdx.x; rg < groups; rg += gridDim.x) {
    const int n0 = rg * 16;
    const int r0 = n0 + g, r1 = n0 + g + 8;
    // weight pointers of this lane's two rows at k-tile 0
    const int8_t* w0;
    const int8_t* w1;
    long long wstep;
    if (tiled) {
      const int blk = n0 >> 7;
      const int in0 = (n0 & 127) + g, in1 = in0 + 8;
      const int8_t* base = q + static_cast<long long>(blk) * k_tiles * 8192;
      w0 = base + in0 * 64 + ((c ^ ((in0 >> 1) & 3)) << 4);
      w1 = base + in1 * 64 + ((c ^ ((in1 >> 1) & 3)) << 4);
      wstep = 8192;
    } else {
      w0 = q + static_cast<long long>(r0 < N ? r0 : 0) * K + 16 * c;
      w1 = q + static_cast<long long>(r1 < N ? r1 : 0) * K + 16 * c;
      wstep = kKT;
    }
    const bool ok0 = tiled || r0 < N, ok1 = tiled || r1 < N;  // padded rows of the tiled layout are zero
    auto load_w = [&](int kt, uint4& a, uint4& b) {
      const bool in = kt < k_tiles && kt * kKT + 16 * c < K;  // K % 16 == 0: a group is wholly in or out
      a = (in && ok0) ? ldg_stream(w0 + kt * wstep) : zero;
      b = (in && ok1) ? ldg_stream(w1 + kt * wstep) : zero;
    };

    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[t][e] = 0.f;
    // this warp's next kDepth k-tiles of weights are always in flight
    uint4 qa[kDepth], qb[kDepth];
#pragma unroll
    for (int i = 0; i < kDepth; ++i) load_w(warp + i * W, qa[i], qb[i]);
    if (!waited) {
      pdl_wait();  // activations and outputs belong to earlier kernels
      waited = true;
    }
    for (int kt0 = warp; kt0 < k_tiles; kt0 += kDepth * W) {
#pragma unroll
      for (int i = 0; i < kDepth; ++i) {
        const int kt = kt0 + i * W;
        if (kt >= k_tiles) break;
        const uint4 q0 = qa[i], q1 = qb[i];
        load_w(kt + kDepth * W, qa[i], qb[i]);
        const int k = kt * kKT + 16 * c;  // physical k of this lane's 16-element group
        const bool kin = k < K;
        uint4 a0lo, a0hi, a1lo, a1hi;
        widen16<T>(q0, a0lo, a0hi);
        widen16<T>(q1, a1lo, a1hi);
        const uint32_t A0[8] = {a0lo.x, a0lo.y, a0lo.z, a0lo.w, a0hi.x, a0hi.y, a0hi.z, a0hi.w};
        const uint32_t A1[8] = {a1lo.x, a1lo.y, a1lo.z, a1lo.w, a1hi.x, a1hi.y, a1hi.z, a1hi.w};
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int m = t * 8 + g;
          uint4 xa = zero, xb = zero;
          if (kin && m < M) {
            const uint4* xp = reinterpret_cast<const uint4*>(x + static_cast<long long>(m) * K + k);
            xa = __ldg(xp);
            xb = __ldg(xp + 1);
          }
          const uint32_t X[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint32_t a[4] = {A0[2 * s], A1[2 * s], A0[2 * s + 1], A1[2 * s + 1]};
            const uint32_t b[2] = {X[2 * s], X[2 * s + 1]};
            mma_16816<T>(acc[t], a, b);
          }
        }
      }
    }
    // C fragment: (row g, tokens 2c, 2c+1) and (row g + 8, same tokens)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      red[warp][g][t * 8 + 2 * c] = acc[t][0];
      red[warp][g][t * 8 + 2 * c + 1] = acc[t][1];
      red[warp][g + 8][t * 8 + 2 * c] = acc[t][2];
      red[warp][g + 8][t * 8 + 2 * c + 1] = acc[t][3];
    }
    __syncthreads();
    if (!swiglu) {
      for (int i = threadIdx.x; i < 16 * M; i += W * 32) {
        const int r = i & 15, m = i >> 4;
        const int n = n0 + r;
        if (n >= N) continue;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) v += red[w][r][m];
        v = v * scale[n] + (bias ? to_f32(bias[n]) : 0.f);
        const long long o = static_cast<long long>(m) * N + n;
        if (resid) v = to_f32(from_f32<T>(v)) + to_f32(resid[o]);
        if (push.world > 0) {
          if (push.slice) {  // two-shot: the owner of column n only
            const int d = n / push.slice;
            static_cast<T*>(push.dst[d])[push_offset(push, m, n, N, d)] = from_f32<T>(v);
          } else {
            for (int d = 0; d < push.world; ++d) static_cast<T*>(push.dst[d])[o] = from_f32<T>(v);  // every rank's slot
          }
        } else {
          y[o] = from_f32<T>(v);
        }
      }
    } else {
      // rows 2i / 2i+1 = gate / up of channel n0/2 + i; each rounded to dtype
      const int I = N / 2;
      for (int i = threadIdx.x; i < 8 * M; i += W * 32) {
        const int pr = i & 7, m = i >> 3;
        const int n = n0 + 2 * pr;
        if (n >= N) continue;
        float gv = 0.f, uv = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) {
          gv += red[w][2 * pr][m];
          uv += red[w][2 * pr + 1][m];
        }
        gv = to_f32(from_f32<T>(gv * scale[n] + (bias ? to_f32(bias[n]) : 0.f)));
        uv = to_f32(from_f32<T>(uv * scale[n + 1] + (bias ? to_f32(bias[n + 1]) : 0.f)));
        y[static_cast<long long>(m) * I + n / 2] = from_f32<T>(silu_mul_f32(gv, uv));
      }
    }
    __syncthreads();  // red is reused by the next row group
  }
  if (!waited) pdl_wait();
  if (push.world > 0) push_arrive(push);
}

// k-tiles of weight loads each warp keeps in flight (PS_MMA_DEPTH = 2, 4 or
// 8 overrides the default for tuning).
int mma_depth() {
  static const int v = [] {
    const char* e = std::getenv("PS_MMA_DEPTH");
    return e ? std::atoi(e) : 0;
  }();
  return v;
}

template <typename T, int W>
int launch_w(void* y, const void* x, const int8_t* q, bool tiled, const float* scale, const void* bias,
             const void* resid, int M, int N, int K, bool swiglu, const PushTargets& pt, cudaStream_t s) {
  const int groups = (N + 15) / 16;
  // persistent grid: as many CTAs as can be resident (occupancy of this
  // instantiation, queried once), striding over the row groups
  auto grid_for = [&](auto kern) {
    static int per_sm = 0;
    if (per_sm == 0) {
      int n = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, W * 32, 0) != cudaSuccess || n < 1) {
        (void)cudaGetLastError();
        n = 1;
      }
      int dev = 0, sms = 148;
      if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      per_sm = n * sms;
    }
    return dim3(groups < per_sm ? groups : per_sm);
  };
#define PS_MMA_LAUNCH(NT)                                                                                         \
  if (mma_depth() >= 8) PS_MMA_LAUNCH_D(NT, 8)                                                                    \
  else if (mma_depth() >= 4 || W > 8) PS_MMA_LAUNCH_D(NT, 4)                                                      \
  else PS_MMA_LAUNCH_D(NT, 2)
#define PS_MMA_LAUNCH_D(NT, DEPTH)                                                                                \
  {                                                                                                               \
    auto kern = linear_mma_kernel<T, NT, W, DEPTH>;                                                               \
    ps_host::launch(kern, grid_for(kern), W * 32, 0, s, static_cast<T*>(y), static_cast<const T*>(x), q, tiled ? 1 : 0, scale, \
                                           static_cast<const T*>(bias), static_cast<const T*>(resid), M, N, K,    \
                                           swiglu ? 1 : 0, pt);                                                   \
  }
  if (M <= 8) PS_MMA_LAUNCH(1)
  else if (M <= 16) PS_MMA_LAUNCH(2)
  else PS_MMA_LAUNCH(4)
#undef PS_MMA_LAUNCH
#undef PS_MMA_LAUNCH_D
  ps_host::count_launch();
  return ps_host::check_launch("linear_mma");
}

template <typename T>
int launch_t(void* y, const void* x, const int8_t* q, bool tiled, const float* scale, const void* bias,
             const void* resid, int M, int N, int K, bool swiglu, const PushTargets& pt, cudaStream_t s) {
  // few row groups (narrow outputs, long K): 16 warps split K, for more loads in flight
  const int groups = (N + 15) / 16;
  if (groups < 2 * 148) return launch_w<T, 16>(y, x, q, tiled, scale, bias, resid, M, N, K, swiglu, pt, s);
  return launch_w<T, 8>(y, x, q, tiled, scale, bias, resid, M, N, K, swiglu, pt, s);
}

}  // namespace

namespace ps_host {

int linear_mma(void* y, const void* x, const int8_t* q, bool tiled, const float* scale, const void* bias,
               const void* resid, int M, int N, int K, int dtype, bool swiglu, cudaStream_t s,
               const ps::PushTargets* push) {
  if (M < 1 || M > kMmaMaxM || K % 16 != 0 || (swiglu && (N % 2 != 0 || resid || push)) || !scale)
    return PS_ERR_UNSUPPORTED;
  if (!aligned(x, 16) || !aligned(q, 16)) return PS_ERR_UNSUPPORTED;
  ps::PushTargets pt;
  std::memset(&pt, 0, sizeof(pt));
  if (push) pt = *push;
  if (dtype == PS_BF16) return launch_t<__nv_bfloat16>(y, x, q, tiled, scale, bias, resid, M, N, K, swiglu, pt, s);
  if (dtype == PS_F16) return launch_t<__half>(y, x, q, tiled, scale, bias, resid, M, N, K, swiglu, pt, s);
  return PS_ERR_UNSUPPORTED;
}

}  // namespace ps_host
