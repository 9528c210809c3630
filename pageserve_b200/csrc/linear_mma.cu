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

// plain / residual / TP-push store of output element (m, n) (v: fp32 after scale)
template <typename T>
PS_DEVICE void mma_store(T* y, const T* bias, const T* resid, const PushTargets& push, float v, int m, int n,
                         int N) {
  if (bias) v += to_f32(bias[n]);
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

// Narrow outputs with a long K (the down projection at decode sizes): the
// same product as linear_mma_kernel (same k permutation inside a k-tile, the
// W warps of a CTA split a 16-row group's k-tiles and reduce in warp order),
// with the loads moved out of registers into a per-warp cp.async ring in
// shared memory. Each lane copies its own 16-byte pieces (2 of weights, 2 per
// 8-token tile of activations) kDepth k-tiles ahead and later reads back only
// what it copied itself, so the ring needs no barrier, and the activation
// loads leave the MMA chain (in the register kernel each k-tile waits for its
// activations from L2, a long chain when K is long). The ring runs on across
// the CTA's row groups. Weights are copied with .cg (L2 only: read once),
// activations with .ca (L1: every group re-reads them); pieces past K or M
// are zero-filled.
PS_DEVICE void ring_cp16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
PS_DEVICE void ring_cp16_l1(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
PS_DEVICE void ring_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
PS_DEVICE void ring_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
PS_DEVICE uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
  return v;
}

// ring layout: [kDepth][W][2 + 2 * NT][32 lanes] x 16 bytes — piece 0/1 = rows
// g / g + 8 of the weights, piece 2 + 2t + h = half h of the activations of
// token t * 8 + g; one ld.shared.v4 of a piece by a warp is 512 contiguous bytes
template <int NT, int W, int kDepth>
constexpr int ring_bytes() {
  return kDepth * W * (2 + 2 * NT) * 512;
}

template <typename T, int NT, int W, int kDepth>
__global__ void __launch_bounds__(W * 32) linear_mma_ring_kernel(
    T* __restrict__ y, const T* __restrict__ x, const int8_t* __restrict__ q, int tiled,
    const float* __restrict__ scale, const T* __restrict__ bias, const T* __restrict__ resid, int M, int N, int K,
    int swiglu, const PushTargets push) {
  constexpr int kPieces = 2 + 2 * NT;
  constexpr uint32_t kSlot = W * kPieces * 512;  // bytes from one ring slot to the next
  extern __shared__ __align__(16) uint4 ring[];
  __shared__ float red[W][16][NT * 8 + 1];
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int k_tiles = (K + kKT - 1) / kKT;
  const int kpw = (k_tiles + W - 1) / W;  // k-tiles per warp and group (the ones past K read as zeros)
  const int groups = (N + 15) / 16;
  const long long wstride = (tiled ? 8192ll : static_cast<long long>(kKT)) * W;  // weight bytes per step
  const uint32_t base = smem_u32(ring) + warp * (kPieces * 512) + lane * 16;  // this lane's piece 0 of slot 0
  const uint32_t ring_end = base + kDepth * kSlot;

  // producer: group prg, step pi (k-tile warp + pi * W), this lane's element
  // offset pk of the k-tile, weight row pointers at that k-tile
  int prg = blockIdx.x, pi = 0;
  int pk = warp * kKT + 16 * c;
  const int8_t* pw0 = q;
  const int8_t* pw1 = q;
  bool pok0 = false, pok1 = false;
  auto rows_of = [&](int rg) {
    const int n0 = rg * 16;
    if (tiled) {
      const int in0 = (n0 & 127) + g, in1 = in0 + 8;
      const int8_t* b = q + (static_cast<long long>(n0 >> 7) * k_tiles + warp) * 8192;
      pw0 = b + in0 * 64 + ((c ^ ((in0 >> 1) & 3)) << 4);
      pw1 = b + in1 * 64 + ((c ^ ((in1 >> 1) & 3)) << 4);
      pok0 = pok1 = true;  // padded rows of the tiled layout are zero
    } else {
      const int r0 = n0 + g, r1 = r0 + 8;
      pok0 = r0 < N;
      pok1 = r1 < N;
      pw0 = q + static_cast<long long>(pok0 ? r0 : 0) * K + warp * kKT + 16 * c;
      pw1 = q + static_cast<long long>(pok1 ? r1 : 0) * K + warp * kKT + 16 * c;
    }
  };
  if (prg < groups) rows_of(prg);
  // activation rows of this lane (token t * 8 + g)
  const T* px[NT];
  bool pm[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    pm[t] = t * 8 + g < M;
    px[t] = x + static_cast<long long>(pm[t] ? t * 8 + g : 0) * K;
  }
  auto issue_w = [&](uint32_t a) {
    const bool in = prg < groups && pk < K;
    ring_cp16(a, in && pok0 ? pw0 : q, in && pok0 ? 16 : 0);
    ring_cp16(a + 512, in && pok1 ? pw1 : q, in && pok1 ? 16 : 0);
  };
  auto issue_x = [&](uint32_t a) {
    const bool in = prg < groups && pk < K;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const bool ok = in && pm[t];
      const T* src = ok ? px[t] + pk : x;
      ring_cp16_l1(a + (2 + 2 * t) * 512, src, ok ? 16 : 0);
      ring_cp16_l1(a + (3 + 2 * t) * 512, ok ? src + 8 : x, ok ? 16 : 0);
    }
  };
  auto advance = [&] {
    pw0 += wstride;
    pw1 += wstride;
    pk += W * kKT;
    if (++pi == kpw) {
      pi = 0;
      pk = warp * kKT + 16 * c;
      prg += gridDim.x;
      if (prg < groups) rows_of(prg);
    }
  };
  // prologue: the weights of the first kDepth steps go out before waiting for
  // the previous kernel (the activations are its output); commit group d
  // completes step d
  {
    const int prg0 = prg, pi0 = pi, pk0 = pk;
    uint32_t a = base;
#pragma unroll
    for (int d = 0; d < kDepth; ++d, a += kSlot) {
      issue_w(a);
      advance();
    }
    pdl_wait();
    prg = prg0;
    pi = pi0;
    pk = pk0;
    if (prg < groups) rows_of(prg);
    a = base;
#pragma unroll
    for (int d = 0; d < kDepth; ++d, a += kSlot) {
      issue_x(a);
      ring_commit();
      advance();
    }
  }

  uint32_t ca = base;  // consumer slot of this lane
  for (int rg = blockIdx.x; rg < groups; rg += gridDim.x) {
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[t][e] = 0.f;
    for (int i = 0; i < kpw; ++i) {
      ring_wait<kDepth - 1>();  // this step's copies (committed kDepth - 1 groups ago) have landed
      uint4 a0lo, a0hi, a1lo, a1hi;
      widen16<T>(lds128(ca), a0lo, a0hi);
      widen16<T>(lds128(ca + 512), a1lo, a1hi);
      const uint32_t A0[8] = {a0lo.x, a0lo.y, a0lo.z, a0lo.w, a0hi.x, a0hi.y, a0hi.z, a0hi.w};
      const uint32_t A1[8] = {a1lo.x, a1lo.y, a1lo.z, a1lo.w, a1hi.x, a1hi.y, a1hi.z, a1hi.w};
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint4 xa = lds128(ca + (2 + 2 * t) * 512), xb = lds128(ca + (3 + 2 * t) * 512);
        const uint32_t X[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint32_t a[4] = {A0[2 * s], A1[2 * s], A0[2 * s + 1], A1[2 * s + 1]};
          const uint32_t b[2] = {X[2 * s], X[2 * s + 1]};
          mma_16816<T>(acc[t], a, b);
        }
      }
      // refill the slot just read (its values are in registers: the MMAs used them)
      issue_w(ca);
      issue_x(ca);
      ring_commit();
      advance();
      ca += kSlot;
      if (ca == ring_end) ca = base;
    }
    // the group's warps reduce in warp order through shared memory
    const int n0 = rg * 16;
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
        mma_store<T>(y, bias, resid, push, v * scale[n], m, n, N);
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
    __syncthreads();  // red is reused by the next group
  }
  ring_wait<0>();
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

// 1 (default): the cp.async ring kernel where it is faster (narrow outputs,
// long K, M <= 8); PS_MMA_RING=0 keeps every shape on the register kernel
bool mma_ring() {
  static const bool v = [] {
    const char* e = std::getenv("PS_MMA_RING");
    return !e || std::atoi(e) != 0;
  }();
  return v;
}

template <typename T, int NT, int W, int kDepth>
int launch_ring(void* y, const void* x, const int8_t* q, bool tiled, const float* scale, const void* bias,
                const void* resid, int M, int N, int K, bool swiglu, const PushTargets& pt, cudaStream_t s) {
  static_assert(ring_bytes<NT, W, kDepth>() + W * 16 * (NT * 8 + 1) * 4 <= 200 * 1024, "ring too large");
  auto kern = linear_mma_ring_kernel<T, NT, W, kDepth>;
  constexpr int kSmem = ring_bytes<NT, W, kDepth>();
  // resident CTAs of this instantiation on the device, queried once
  static const int resident = [&] {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess) {
      (void)cudaGetLastError();
      return 0;
    }
    int n = 0, dev = 0, sms = 148;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, W * 32, kSmem) != cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      n = 1;
    }
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return n * sms;
  }();
  if (resident == 0) {
    ps_host::set_error("linear_mma: cannot reserve %d bytes of shared memory", kSmem);
    return PS_ERR_CUDA;
  }
  const int groups = (N + 15) / 16;
  ps_host::launch(kern, dim3(groups < resident ? groups : resident), W * 32, kSmem, s, static_cast<T*>(y),
                  static_cast<const T*>(x), q, tiled ? 1 : 0, scale, static_cast<const T*>(bias),
                  static_cast<const T*>(resid), M, N, K, swiglu ? 1 : 0, pt);
  ps_host::count_launch();
  return ps_host::check_launch("linear_mma");
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
  const int groups = (N + 15) / 16, k_tiles = (K + kKT - 1) / kKT;
  // narrow outputs with a long K at M <= 8 (the down projection): the cp.async
  // ring, whose activation loads stay out of the MMA chain (measured 14%
  // faster there; elsewhere the register-prefetch kernel is as fast or faster)
  if (mma_ring() && M <= 8 && groups < 2 * 148 && k_tiles >= 8 * 16)
    return launch_ring<T, 1, 16, 4>(y, x, q, tiled, scale, bias, resid, M, N, K, swiglu, pt, s);
  // few row groups (narrow outputs, long K): 16 warps split K, for more loads in flight
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
