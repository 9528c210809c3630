// W8A16 (and 16-bit-weight) linear on the 5th-generation tensor cores:
//   y[m,n] = scale[n] * sum_k x[m,k] * w[n,k] + bias[n] (+ resid[m,n])
// (engine/quantization.py:26-50 + F.linear, engine/model.py:168-193 of the
// reference).
//
// Orientation ("swap AB"): the MMA's 128-row M dimension walks the weight's
// output channels and its N dimension walks the tokens, so one CTA owns a
// 128-channel weight slab for a tile of up to 256 tokens and every weight byte
// is fetched and widened once per token tile. Decode batches (tens of tokens)
// stream the int8 weight at HBM speed; prefill tiles run tensor-bound.
//
// Roles (192 threads):
//   warp 0        TMA producer: int8 weight tile (128 x 64 B) and the bf16
//                 activation tile (BM x 128 B, 128B-swizzled) per stage
//   warp 1        TMEM allocator; one elected lane issues tcgen05.mma
//                 (M=128, N=BM, K=16) x 4 per stage, commits to mbarriers
//   warps 2..5    widen int8 -> bf16 (exact: |q| <= 127) into the
//                 128B-swizzled K-major UMMA operand layout, then run the
//                 epilogue from TMEM (scale, bias, residual, store / split-K
//                 reduction)
// The per-channel scale is applied once per output after accumulation, so
// the tensor-core operand is the exact integer weight.
//
// Every mbarrier wait is bounded (about a second of clock64 cycles): on
// timeout the kernel records kErrTimeout in the status word, stops issuing
// work, releases its TMEM and returns.
#include <cudaTypedefs.h>

#include <mutex>

#include "linear.cuh"

namespace {

using namespace ps;

constexpr int kThreads = 192;
constexpr int kBN = 128;  // weight rows per CTA (MMA M)
constexpr int kBK = 64;   // K elements per stage (128 bytes of bf16 = one swizzle atom row)
constexpr long long kWaitCycles = 2000000000LL;

// ------------------------------------------------------------- PTX bits --
PS_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
PS_DEVICE void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
PS_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
PS_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait. Returns false (and raises the CTA abort flag) on timeout or
// when another role already aborted.
PS_DEVICE bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      record_error(status, kErrTimeout);
      return false;
    }
  }
  return true;
}

PS_DEVICE void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

PS_DEVICE void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
PS_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PS_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 128B-swizzled K-major shared-memory matrix descriptor (SM100 format:
// start>>4 @0, LBO>>4 @16, SBO>>4 @32, version 1 @46, layout 2 = SW128 @61).
PS_DEVICE uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1024 >> 4) << 32;  // 8-row group stride
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// kind::f16 instruction descriptor: f32 accumulate, A/B = bf16 (1) or f16
// (0), both K-major, N>>3 @17, M>>4 @24.
__host__ __device__ constexpr uint32_t instr_desc(bool bf16, int m, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

PS_DEVICE void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
PS_DEVICE void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

PS_DEVICE void tmem_ld16(uint32_t addr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 signed bytes -> 16 bf16 (exact). For byte b = s*128 + u (two's
// complement, u = low 7 bits): value = (128 + u) - (128 + 128*s); both
// terms are exact bf16 built by byte permutes, one packed subtract per pair.
PS_DEVICE void widen16_bf16(const uint4& in, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {in.x, in.y, in.z, in.w};
  uint32_t out[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t low7 = w[j] & 0x7F7F7F7Fu;
    const uint32_t sign = w[j] & 0x80808080u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // bytes 2h, 2h+1 -> bf16 pair {0x43 : byte}
      const uint32_t sel = h ? 0x4342u : 0x4140u;
      const uint32_t a = __byte_perm(low7, 0x43434343u, sel);
      const uint32_t b = __byte_perm(sign, 0x43434343u, sel);
      uint32_t r;
      asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
      out[j * 2 + h] = r;
    }
  }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
}
PS_DEVICE void widen16_f16(const uint4& in, uint4& lo, uint4& hi) {
  // f16: 0x6400 | byte = 1024 + byte; subtract 1024 + 128 after flipping the sign bit.
  const uint32_t w[4] = {in.x ^ 0x80808080u, in.y ^ 0x80808080u, in.z ^ 0x80808080u, in.w ^ 0x80808080u};
  uint32_t out[8];
  const uint32_t bias = 0x64806480u;  // 1152.0 in both halves
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t a = __byte_perm(w[j], 0x64646464u, h ? 0x4342u : 0x4140u);
      uint32_t r;
      asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(bias));
      out[j * 2 + h] = r;
    }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
}

struct TcParams {
  void* y;
  const float* scale;
  const void* bias;
  const void* resid;
  float* ws;        // split-K fp32 partial sums [M][N] (kept zeroed)
  int* counters;    // split-K arrival counters [m_tiles][n_tiles] (kept zeroed)
  int* status;
  int M, N, K;
  int k_tiles;      // total K tiles of 64
  int k_tiles_per_split;
  int splits;
};

template <typename T, bool kInt8, int BM, int STAGES>
struct Smem {
  static constexpr int kA = kBN * kBK * 2;       // bf16 weight operand
  static constexpr int kW8 = kInt8 ? kBN * kBK : 0;  // raw int8 weight
  static constexpr int kX = BM * kBK * 2;        // activation operand
  static constexpr int kStage = kA + kW8 + kX;
  static constexpr int kBytes = STAGES * kStage + 1024 /*align*/ + 256 /*barriers*/;
};

template <typename T, bool kInt8, int BM, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                     const TcParams p) {
  using S = Smem<T, kInt8, BM, STAGES>;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  // stage s: [A bf16 | X bf16 | W int8]; A and X are 1024-aligned
  auto a_addr = [&](int s) { return base + s * S::kStage; };
  auto x_addr = [&](int s) { return base + s * S::kStage + S::kA; };
  auto w8_addr = [&](int s) { return base + s * S::kStage + S::kA + S::kX; };
  const uint32_t bars = base + STAGES * S::kStage;
  auto tma_full = [&](int s) { return bars + 8 * s; };
  auto deq_full = [&](int s) { return bars + 8 * (STAGES + s); };
  auto mma_done = [&](int s) { return bars + 8 * (2 * STAGES + s); };
  const uint32_t acc_full = bars + 8 * (3 * STAGES);
  unsigned char* misc = gbase + STAGES * S::kStage + 8 * (3 * STAGES + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 4);
  int* last_flag = reinterpret_cast<int*>(misc + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN;
  const int m0 = blockIdx.y * BM;
  const int split = blockIdx.z;
  const int kt0 = split * p.k_tiles_per_split;
  const int kt1 = min(p.k_tiles, kt0 + p.k_tiles_per_split);
  const int nkt = kt1 - kt0;
  constexpr int kTmemCols = BM <= 32 ? 32 : (BM <= 64 ? 64 : (BM <= 128 ? 128 : 256));

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    *last_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(tma_full(s), 1);
      mbar_init(deq_full(s), kInt8 ? 4 : 1);
      mbar_init(mma_done(s), 1);
    }
    mbar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------- TMA producer --
    // The whole warp walks the loop (keeps it converged); lane 0 issues.
    constexpr uint32_t kTx = S::kX + (kInt8 ? S::kW8 : S::kA);
    for (int i = 0; i < nkt; ++i) {
      const int s = i % STAGES;
      if (i >= STAGES) {
        const bool ok = mbar_wait(mma_done(s), ((i / STAGES) - 1) & 1, abort_flag, p.status);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      if (lane == 0) {
        mbar_expect_tx(tma_full(s), kTx);
        const int kx = (kt0 + i) * kBK;
        tma_load_2d(kInt8 ? w8_addr(s) : a_addr(s), &wmap, tma_full(s), kx, n0);
        tma_load_2d(x_addr(s), &xmap, tma_full(s), kx, m0);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer --
    constexpr uint32_t idesc = instr_desc(!std::is_same<T, __half>::value, kBN, BM);
    bool ok = nkt > 0;
    for (int i = 0; i < nkt; ++i) {
      const int s = i % STAGES;
      ok = __all_sync(0xffffffffu, mbar_wait(kInt8 ? deq_full(s) : tma_full(s), (i / STAGES) & 1, abort_flag,
                                             p.status));
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t ad = smem_desc_sw128(a_addr(s) + kk * 32);
          const uint64_t bd = smem_desc_sw128(x_addr(s) + kk * 32);
          mma_f16(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(mma_done(s));
      }
      __syncwarp();
    }
    if (ok && lane == 0) mma_commit(acc_full);
    __syncwarp();
  } else {
    // --------------------------------------- int8 -> bf16 widening warps --
    const int t = threadIdx.x - 64;  // 0..127
    if (kInt8) {
      for (int i = 0; i < nkt; ++i) {
        const int s = i % STAGES;
        if (!__all_sync(0xffffffffu, mbar_wait(tma_full(s), (i / STAGES) & 1, abort_flag, p.status))) break;
        const unsigned char* w8 = gbase + (w8_addr(s) - base);
        unsigned char* a = gbase + (a_addr(s) - base);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int id = t + 128 * j;  // 512 chunks of 16 int8
          const int r = id >> 2;
          const int c16 = id & 3;
          const uint4 in = *reinterpret_cast<const uint4*>(w8 + r * 64 + c16 * 16);
          uint4 lo, hi;
          if constexpr (std::is_same<T, __half>::value) widen16_f16(in, lo, hi);
          else widen16_bf16(in, lo, hi);
          const int c0 = (2 * c16) ^ (r & 7), c1 = (2 * c16 + 1) ^ (r & 7);
          *reinterpret_cast<uint4*>(a + r * 128 + c0 * 16) = lo;
          *reinterpret_cast<uint4*>(a + r * 128 + c1 * 16) = hi;
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(deq_full(s));
      }
    }
    // ------------------------------------------------------------ epilogue --
    const bool ok = __all_sync(0xffffffffu, nkt > 0 && mbar_wait(acc_full, 0, abort_flag, p.status));
    tc_fence_after();
    const int q = warp & 3;            // TMEM lane quarter this warp may read
    const int row = q * 32 + lane;     // weight row within the tile
    const int n = n0 + row;
    const T* bias = static_cast<const T*>(p.bias);
    const T* resid = static_cast<const T*>(p.resid);
    T* y = static_cast<T*>(p.y);
    const float sc = (n < p.N && p.scale) ? p.scale[n] : 1.f;
    const float bs = (n < p.N && bias) ? to_f32(bias[n]) : 0.f;
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < BM; c += 16) {
        float v[16];
        __syncwarp();
        tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c, v);
        if (n < p.N) {
          if (p.splits == 1) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = m0 + c + j;
              if (m < p.M) {
                float o = v[j] * sc + bs;
                if (resid) o = to_f32(from_f32<T>(o)) + to_f32(resid[static_cast<long long>(m) * p.N + n]);
                y[static_cast<long long>(m) * p.N + n] = from_f32<T>(o);
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = m0 + c + j;
              if (m < p.M) atomicAdd(p.ws + static_cast<long long>(m) * p.N + n, v[j]);
            }
          }
        }
      }
    }
    if (p.splits > 1) {
      // last CTA of this tile finishes: apply scale/bias/residual, re-zero.
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (t == 0) {
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        const int prev = atomicAdd(p.counters + tile, 1);
        *last_flag = (prev == p.splits - 1) ? 1 : 0;
        if (*last_flag) p.counters[tile] = 0;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*last_flag && n < p.N) {
        __threadfence();
        const int mend = min(p.M, m0 + BM);
        for (int m = m0; m < mend; ++m) {
          float* w = p.ws + static_cast<long long>(m) * p.N + n;
          const float acc = __ldcg(w);
          *w = 0.f;
          float o = acc * sc + bs;
          if (resid) o = to_f32(from_f32<T>(o)) + to_f32(resid[static_cast<long long>(m) * p.N + n]);
          y[static_cast<long long>(m) * p.N + n] = from_f32<T>(o);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ------------------------------------------------------------- host side --
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_map(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int esize, int rows, int cols, int box_cols,
              int box_rows, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * esize};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Plan {
  int bm, m_tiles, n_tiles, k_tiles, splits, per_split;
};

Plan plan(int M, int N, int K) {
  Plan pl{};
  // token tile: one tile up to 256, else equal tiles of a multiple of 16
  const int mt = (M + 255) / 256;
  int bm = (M + mt - 1) / mt;
  bm = (bm + 15) / 16 * 16;
  if (bm < 16) bm = 16;
  pl.bm = bm <= 32 ? 32 : (bm <= 64 ? 64 : (bm <= 128 ? 128 : (bm <= 192 ? 192 : 256)));
  pl.m_tiles = (M + pl.bm - 1) / pl.bm;
  pl.n_tiles = (N + kBN - 1) / kBN;
  pl.k_tiles = (K + kBK - 1) / kBK;
  const int tiles = pl.m_tiles * pl.n_tiles;
  int splits = 1;
  if (tiles < 148) {
    splits = (148 + tiles - 1) / tiles;
    const int max_split = pl.k_tiles / 4 > 0 ? pl.k_tiles / 4 : 1;  // >= 4 K tiles per CTA
    if (splits > max_split) splits = max_split;
  }
  pl.per_split = (pl.k_tiles + splits - 1) / splits;
  pl.splits = (pl.k_tiles + pl.per_split - 1) / pl.per_split;
  return pl;
}

size_t ws_bytes(const Plan& pl, int M, int N) {
  if (pl.splits <= 1) return 0;
  return 256 + static_cast<size_t>(pl.m_tiles) * pl.n_tiles * sizeof(int) + static_cast<size_t>(M) * N * 4 + 256;
}

template <typename T, bool kInt8, int BM>
int launch_bm(const CUtensorMap& wm, const CUtensorMap& xm, const TcParams& p, const Plan& pl, cudaStream_t s) {
  constexpr int stage = Smem<T, kInt8, BM, 1>::kStage;
  constexpr int stages = (200 * 1024) / stage > 8 ? 8 : (200 * 1024) / stage;
  using S = Smem<T, kInt8, BM, stages>;
  auto kern = linear_tc_kernel<T, kInt8, BM, stages>;
  static bool attr_set = false;  // one attribute call per instantiation
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes) != cudaSuccess) {
      ps_host::set_error("linear_tc: cannot reserve %d bytes of shared memory", S::kBytes);
      return PS_ERR_CUDA;
    }
    attr_set = true;
  }
  dim3 grid(pl.n_tiles, pl.m_tiles, pl.splits);
  kern<<<grid, kThreads, S::kBytes, s>>>(wm, xm, p);
  ps_host::count_launch();
  return ps_host::check_launch("linear_tc");
}

template <typename T, bool kInt8>
int launch_t(const CUtensorMap& wm, const CUtensorMap& xm, const TcParams& p, const Plan& pl, cudaStream_t s) {
  switch (pl.bm) {
    case 32: return launch_bm<T, kInt8, 32>(wm, xm, p, pl, s);
    case 64: return launch_bm<T, kInt8, 64>(wm, xm, p, pl, s);
    case 128: return launch_bm<T, kInt8, 128>(wm, xm, p, pl, s);
    case 192: return launch_bm<T, kInt8, 192>(wm, xm, p, pl, s);
    default: return launch_bm<T, kInt8, 256>(wm, xm, p, pl, s);
  }
}

}  // namespace

namespace ps_host {

size_t linear_tc_workspace(int M, int N, int K) {
  const Plan pl = plan(M, N, K);
  return ws_bytes(pl, M, N);
}

int linear_tc(void* y, const void* x, const void* w, int wdtype, const float* scale, const void* bias,
              const void* resid, int M, int N, int K, int dtype, void* workspace, size_t workspace_bytes,
              cudaStream_t s) {
  if (dtype != PS_BF16 && dtype != PS_F16) return PS_ERR_UNSUPPORTED;
  const bool int8 = wdtype == PS_I8;
  if (!int8 && wdtype != dtype) return PS_ERR_UNSUPPORTED;
  // TMA: global row strides must be multiples of 16 bytes
  if (K % 16 != 0 || !aligned(x, 16) || !aligned(w, 16)) return PS_ERR_UNSUPPORTED;
  const Plan pl = plan(M, N, K);
  TcParams p{};
  p.y = y;
  p.scale = scale;
  p.bias = bias;
  p.resid = resid;
  p.status = status_word(PS_TU_GEMM);
  p.M = M;
  p.N = N;
  p.K = K;
  p.k_tiles = pl.k_tiles;
  p.k_tiles_per_split = pl.per_split;
  p.splits = pl.splits;
  if (pl.splits > 1) {
    const size_t need = ws_bytes(pl, M, N);
    if (!workspace || workspace_bytes < need) {
      set_error("linear: split-K workspace of %zu bytes needed, %zu given", need, workspace_bytes);
      return PS_ERR_INVALID;
    }
    uintptr_t a = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~static_cast<uintptr_t>(255);
    p.counters = reinterpret_cast<int*>(a);
    p.ws = reinterpret_cast<float*>((a + pl.m_tiles * pl.n_tiles * sizeof(int) + 255) & ~static_cast<uintptr_t>(255));
  }
  const CUtensorMapDataType xdt = dtype == PS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap wm, xm;
  bool ok = make_map(&xm, x, xdt, 2, M, K, kBK, pl.bm, CU_TENSOR_MAP_SWIZZLE_128B);
  if (int8) ok = ok && make_map(&wm, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K, kBK, kBN, CU_TENSOR_MAP_SWIZZLE_NONE);
  else ok = ok && make_map(&wm, w, xdt, 2, N, K, kBK, kBN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok) {
    set_error("linear: cuTensorMapEncodeTiled failed (M=%d N=%d K=%d)", M, N, K);
    return PS_ERR_CUDA;
  }
  if (dtype == PS_BF16) return int8 ? launch_t<__nv_bfloat16, true>(wm, xm, p, pl, s)
                                    : launch_t<__nv_bfloat16, false>(wm, xm, p, pl, s);
  return int8 ? launch_t<__half, true>(wm, xm, p, pl, s) : launch_t<__half, false>(wm, xm, p, pl, s);
}

}  // namespace ps_host
