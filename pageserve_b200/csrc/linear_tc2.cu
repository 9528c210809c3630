// W8A16 linear on CTA pairs (engine/quantization.py:26-50 + F.linear,
// engine/model.py:168-193 of the reference):
//   y[m,n] = scale[n] * sum_k x[m,k] * w[n,k] + bias[n] (+ resid[m,n])
// or, for interleaved gate/up rows, y[m,i] = silu(gate) * up.
//
// The two CTAs of a (2,1,1) cluster run one tcgen05.mma.cta_group::2 per
// 16-deep K step: M = 256 weight rows (128 per SM, each CTA's widened rows in
// its own TMEM), N = BM tokens (each CTA stages half the token tile in its
// shared memory), the 256 x BM fp32 accumulator split across the two SMs'
// TMEM. Per SM this is the operand traffic of a 256-row slab on one SM, but
// with half the accumulator, so every SM keeps TWO accumulators and the grid
// is persistent: while the epilogue warps drain tile t from one accumulator,
// the MMA already runs tile t+1 into the other, and the producers stream its
// operands. Tiles are handed out round-robin (pair p takes p, p + P, ...),
// slab-major, so the pairs that run at the same time share weight slabs in L2.
//
// Roles (352 threads per CTA):
//   warp 0      weight producer: one contiguous 8 KB bulk copy per k-tile (this
//               CTA's 128 rows of the pre-tiled int8 weight) into a deep ring
//   warp 1      TMEM allocator (cta_group::2, both CTAs); in the leader CTA
//               (cluster rank 0) one lane issues the pair's MMAs and commits
//               their completion to the barriers of both CTAs
//   warp 2      activation producer: TMA of this CTA's BM/2 token rows x 64 K
//               (128B swizzle); both CTAs' copies complete on the leader's
//               barrier (the .cta_group::2 form of the TMA load)
//   warps 3..6  widen int8 -> bf16/f16 (exact) into the TMEM A ring (one row
//               per lane) and arrive on the leader's A-ready barrier
//   warps 7..10 epilogue: TMEM -> scale, bias, residual (TMA-loaded into the
//               output tile) or SiLU*up -> 16-bit tile in shared memory -> one
//               TMA store, then release the accumulator to the leader
//
// Every mbarrier wait is bounded (about a second of clock64 cycles): on
// timeout the CTA records kErrTimeout in the status word and stops issuing.
// Teardown waits (bounded) for its own copies and MMAs, then both CTAs meet
// at a cluster barrier before they free TMEM, so no CTA exits while its peer
// can still touch its shared memory or TMEM.
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "linear.cuh"
#include "tc_ptx.cuh"
#include "widen.cuh"

namespace {

using namespace ps;

constexpr int kT2Threads = 352;
constexpr int kT2BK = 64;              // K elements per k-tile
constexpr int kT2Budget = 216 * 1024;  // shared memory of one CTA

// Pipeline event timestamps (clock64) of both CTAs of pair 0 for latency
// analysis; compiled only with -DPS_TRACE (never in the shipped library).
#ifdef PS_TRACE
__device__ unsigned long long g_tc2_trace[4096];
#define PS_T2(slot, cond)                                                          \
  do {                                                                             \
    if ((cond) && blockIdx.x < 2 && (slot) < 2048)                                 \
      g_tc2_trace[blockIdx.x * 2048 + (slot)] = clock64();                         \
  } while (0)
#else
#define PS_T2(slot, cond) \
  do {                    \
  } while (0)
#endif

template <int BM>
struct Cfg2 {
  static constexpr int kW = 8192;                // 128 rows x 64 int8
  static constexpr int kXh = (BM / 2) * 128;  // BM/2 token rows x 64 K x 16-bit
  static constexpr int kOut = BM * 256;          // [BM][128] 16-bit output tile
  // activation ring: 8 stages (a pair's activation copy takes ~1 us to land
  // on the leader's barrier, several k-tiles of MMA at this tile shape)
  static constexpr int kRX = 8;
  static constexpr int kRW0 = (kT2Budget - kRX * kXh - kOut) / kW;
  static constexpr int kRW = kRW0 > 16 ? 16 : kRW0;  // weight ring
  static constexpr int kOffX = 0;
  static constexpr int kOffOut = kOffX + kRX * kXh;
  static constexpr int kOffW = kOffOut + kOut;
  static constexpr int kOffBar = kOffW + kRW * kW;
  static constexpr int kBytes = kOffBar + 8 * 64 + 64 + 1024;  // + alignment slack
  // TMEM: two accumulators of BM columns, then the widened-A ring
  // An A stage holds kAK k-tiles (32 columns each): one handoff (and one
  // arrival on the leader's barrier) per kAK k-tiles.
  static constexpr int kAK = 2;
  static constexpr int kACols = 32 * kAK;
  static constexpr int kACol0 = 2 * BM;
  static constexpr int kATm = (512 - 2 * BM) / kACols >= 4 ? 4 : (512 - 2 * BM) / kACols;
  static_assert(BM % 32 == 0 && BM >= 64 && BM <= 192, "token tile");
  static_assert(kATm >= 2 && 2 * BM + kATm * kACols <= 512, "TMEM columns");
  static_assert(kXh % 1024 == 0 && kOut % 1024 == 0, "1024-byte aligned stages");
  static_assert(kRW >= 4, "weight ring");
  static_assert(kBytes <= 227 * 1024, "shared memory plan");
};

struct Tc2Params {
  const int8_t* wt;  // pre-tiled int8 weight [N/128][K/64][128][64]
  const float* scale;
  const void* bias;
  const void* resid;
  int* status;
  int M, N, K;
  int k_tiles;
  int m_tiles;
  int tiles;   // (N / 256) * m_tiles
  int swiglu;  // interleaved gate/up rows -> y [M][N/2]
};

struct Tc2Maps {
  CUtensorMap x;    // activations [M][K], box 64 x BM/2, 128B swizzle
  CUtensorMap y;    // output [M][N] (box 128 x BM) or [M][N/2] (box 64 x BM)
  CUtensorMap res;  // residual [M][N], box 128 x BM
};

// TMA load whose completion is signalled on a barrier of either CTA of the
// pair (`bar` is a shared::cluster address).
PS_DEVICE void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// Pair MMA with A from TMEM (both CTAs' TMEM at the same address).
PS_DEVICE void mma2_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Arrive (once) on the barrier at shared::cluster address `bar` when every
// pair MMA issued so far by this thread has completed.
PS_DEVICE void commit2(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// The same on the barrier at this offset in both CTAs of the pair: one
// commit to the local barrier, one to the peer's through the cluster window.
PS_DEVICE void commit2_pair(uint32_t bar, uint32_t peer_off) {
  commit2(bar);
  commit2(bar + peer_off);
}

// Arrive on a barrier of either CTA of the cluster (default .release.cta
// semantics). The data it publishes is TMEM written by tcgen05.st (completed
// by tcgen05.wait::st and ordered by tcgen05.fence::before_thread_sync) or
// TMEM already read by tcgen05.ld, not generic memory, so no cluster-scope
// release is needed; a .release.cluster arrive measured ~0.9 us here, which
// serialised the widen -> MMA pipeline.
PS_DEVICE void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Barrier 2 among the 4 epilogue warps (warps 7..10).
PS_DEVICE void epi2_bar() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

// Bounded wait for a phase that must complete (teardown): ignores the abort
// flag, gives up after kWaitCycles.
PS_DEVICE void drain_wait(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) break;
  }
}

template <typename T, int BM>
__global__ void __launch_bounds__(kT2Threads, 1)
    linear_tc2_kernel(const __grid_constant__ Tc2Maps maps, const Tc2Params p) {
  using C = Cfg2<BM>;
  constexpr int RW = C::kRW, RX = C::kRX, AS = C::kATm;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  auto x_addr = [&](int s) { return base + C::kOffX + s * C::kXh; };
  auto w_addr = [&](int s) { return base + C::kOffW + s * C::kW; };
  const uint32_t out_sa = base + C::kOffOut;
  const uint32_t bars = base + C::kOffBar;
  auto w_full = [&](int s) { return bars + 8 * s; };
  auto w_empty = [&](int s) { return bars + 8 * (16 + s); };
  auto x_full = [&](int s) { return bars + 8 * (32 + s); };
  auto x_empty = [&](int s) { return bars + 8 * (40 + s); };
  auto a_full = [&](int s) { return bars + 8 * (48 + s); };
  auto a_empty = [&](int s) { return bars + 8 * (52 + s); };
  auto acc_full = [&](int b) { return bars + 8 * (56 + b); };
  auto acc_empty = [&](int b) { return bars + 8 * (58 + b); };
  const uint32_t res_full = bars + 8 * 60;
  const uint32_t drain = bars + 8 * 61;
  unsigned char* misc = gbase + C::kOffBar + 8 * 64;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());  // 0: leader (issues the MMAs)
  const int pair = static_cast<int>(blockIdx.x) >> 1;
  const int npairs = static_cast<int>(gridDim.x) >> 1;
  const int KT = p.k_tiles;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < RW; ++s) {
      mbar_init(w_full(s), 1);
      mbar_init(w_empty(s), 4);
    }
    for (int s = 0; s < RX; ++s) {
      mbar_init(x_full(s), 1);   // the leader's arrive.expect_tx; both halves' bytes
      mbar_init(x_empty(s), 1);  // the leader's MMA commit
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init(a_full(s), 8);   // 4 widen warps of each CTA
      mbar_init(a_empty(s), 1);  // the leader's MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);   // the leader's MMA commit
      mbar_init(acc_empty(b), 2);  // one arrival per CTA's epilogue
    }
    mbar_init(res_full, 1);
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  PS_T2(0, threadIdx.x == 0);
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  PS_T2(1, threadIdx.x == 0);
  // Programmatic dependent launch: the weight producer streams the (never
  // written) weights while the previous kernel finishes; every other role
  // waits for it before reading activations / residuals or writing.
  pdl_trigger();
  if (warp != 0) pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------- weight producer --
    int g = 0;
    for (int tile = pair; tile < p.tiles; tile += npairs) {
      const int nt = tile / p.m_tiles;
      const int8_t* src = p.wt + static_cast<long long>(nt * 2 + rank) * KT * 8192;
      bool ok = true;
      for (int i = 0; i < KT; ++i, ++g) {
        const int s = g % RW;
        if (g >= RW && !warp_wait(w_empty(s), ((g / RW) - 1) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        PS_T2(8 + (g & 255) * 8 + 0, lane == 0);
        if (lane == 0) {
          mbar_expect_tx(w_full(s), 8192);
          bulk_load(w_addr(s), src + static_cast<long long>(i) * 8192, 8192, w_full(s));
        }
        __syncwarp();
      }
      if (!ok) break;
    }
    // teardown: the last copy into every stage has landed
    if (lane == 0)
      for (int s = 0; s < RW && s < g; ++s) drain_wait(w_full(s), ((g - 1 - s) / RW) & 1);
  } else if (warp == 2) {
    // --------------------------------------------- activation producer --
    int g = 0;
    const uint32_t lead = mapa_shared(x_full(0), 0);  // leader's x_full(0); stages are 8 bytes apart
    for (int tile = pair; tile < p.tiles; tile += npairs) {
      const int mt = tile % p.m_tiles;
      const int row0 = mt * BM + rank * (BM / 2);
      bool ok = true;
      for (int i = 0; i < KT; ++i, ++g) {
        const int s = g % RX;
        if (g >= RX && !warp_wait(x_empty(s), ((g / RX) - 1) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        PS_T2(8 + (g & 255) * 8 + 1, lane == 0);
        if (lane == 0) {
          if (rank == 0) mbar_expect_tx(x_full(s), 2 * C::kXh);
          tma_load_2d_pair(x_addr(s), &maps.x, lead + 8 * s, i * kT2BK, row0);
        }
        __syncwarp();
      }
      if (!ok) break;
    }
    if (rank == 0 && lane == 0)
      for (int s = 0; s < RX && s < g; ++s) drain_wait(x_full(s), ((g - 1 - s) / RX) & 1);
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer --
    if (rank == 0) {
      constexpr uint32_t idesc = instr_desc(!std::is_same<T, __half>::value, 256, BM);
      const uint32_t peer_off = mapa_shared(bars, 1) - bars;  // leader -> peer barrier offset
      int g = 0, ga = 0, it = 0;  // k-tiles, A stages, tiles of this pair so far
      bool issued = false, ok = true;
      for (int tile = pair; ok && tile < p.tiles; tile += npairs, ++it) {
        const int b = it & 1;
        if (it >= 2) ok = warp_wait(acc_empty(b), ((it >> 1) - 1) & 1, abort_flag, p.status);
        if (!ok) break;
        tc_fence_after();
        for (int i = 0; ok && i < KT; i += C::kAK, ++ga) {
          const int sa = ga % AS;
          const int kc = KT - i < C::kAK ? KT - i : C::kAK;
          ok = warp_wait(a_full(sa), (ga / AS) & 1, abort_flag, p.status);
          for (int j = 0; ok && j < kc; ++j, ++g) {
            const int sx = g % RX;
            ok = warp_wait(x_full(sx), (g / RX) & 1, abort_flag, p.status);
            if (!ok) break;
            tc_fence_after();
            PS_T2(8 + (g & 255) * 8 + 4, lane == 0);
            if (lane == 0) {
#pragma unroll
              for (int kk = 0; kk < kT2BK / 16; ++kk)
                mma2_ts(tmem + b * BM, tmem + C::kACol0 + sa * C::kACols + j * 32 + kk * 8,
                        smem_desc_sw128(x_addr(sx) + kk * 32), idesc, (i + j > 0 || kk > 0) ? 1u : 0u);
              commit2_pair(x_empty(sx), peer_off);
            }
            issued = true;
            __syncwarp();
          }
          if (ok && lane == 0) {
            commit2_pair(a_empty(sa), peer_off);
          }
          __syncwarp();
        }
        if (ok && lane == 0) {
          commit2_pair(acc_full(b), peer_off);
        }
        __syncwarp();
      }
      // teardown: every issued MMA has completed before TMEM is freed
      if (issued) {
        if (lane == 0) commit2(drain);
        __syncwarp();
        if (lane == 0) drain_wait(drain, 0);
        __syncwarp();
      }
    }
  } else if (warp <= 6) {
    // ------------------------------------- int8 -> 16-bit widening into TMEM --
    const int q = warp & 3;  // TMEM lane quarter (warps 3..6 -> 3, 0, 1, 2)
    const int rin = q * 32 + lane;
    const int swz = (rin >> 1) & 3;  // chunk slot swizzle of the tiled layout
    // the peer signals the leader's barrier through the cluster window; the
    // leader arrives on its own barrier locally (a cluster-window arrive costs
    // a round trip, ~0.3 us, that the next release-ordered op would wait for)
    const uint32_t lead = mapa_shared(a_full(0), 0);
    int g = 0, ga = 0;
    bool ok = true;
    for (int tile = pair; ok && tile < p.tiles; tile += npairs) {
      for (int i = 0; ok && i < KT; i += C::kAK, ++ga) {
        const int sa = ga % AS;
        const int kc = KT - i < C::kAK ? KT - i : C::kAK;
        if (ga >= AS) ok = warp_wait(a_empty(sa), ((ga / AS) - 1) & 1, abort_flag, p.status);
        for (int j = 0; ok && j < kc; ++j, ++g) {
          const int sw = g % RW;
          ok = warp_wait(w_full(sw), (g / RW) & 1, abort_flag, p.status);
          if (!ok) break;
          tc_fence_after();
          PS_T2(8 + (g & 255) * 8 + 2, threadIdx.x == 96);
          const unsigned char* row = gbase + (w_addr(sw) - base) + rin * 64;
          uint32_t words[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 in = *reinterpret_cast<const uint4*>(row + ((c ^ swz) << 4));
            uint4 lo, hi;
            if constexpr (std::is_same<T, __half>::value) widen16_f16(in, lo, hi);
            else widen16_bf16(in, lo, hi);
            words[c * 8 + 0] = lo.x; words[c * 8 + 1] = lo.y; words[c * 8 + 2] = lo.z; words[c * 8 + 3] = lo.w;
            words[c * 8 + 4] = hi.x; words[c * 8 + 5] = hi.y; words[c * 8 + 6] = hi.z; words[c * 8 + 7] = hi.w;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(w_empty(sw));  // this weight stage is read
          const uint32_t ta = tmem + (static_cast<uint32_t>(q * 32) << 16) + C::kACol0 + sa * C::kACols + j * 32;
          tmem_st16(ta, words);
          tmem_st16(ta + 16, words + 16);
          PS_T2(8 + (g & 255) * 8 + 3, threadIdx.x == 96);
        }
        if (!ok) break;
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(a_full(sa));
          else mbar_arrive_cluster(lead + 8 * sa);
        }
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    const int q = warp & 3;  // TMEM lane quarter (warps 7..10 -> 3, 0, 1, 2)
    const bool e0 = threadIdx.x == 7 * 32;
    const uint32_t lead_empty = mapa_shared(acc_empty(0), 0);
    const T* bias = static_cast<const T*>(p.bias);
    T* out_tile = reinterpret_cast<T*>(gbase + C::kOffOut);
    int it = 0;
    for (int tile = pair; tile < p.tiles; tile += npairs, ++it) {
      const int b = it & 1;
      const int nt = tile / p.m_tiles, mt = tile % p.m_tiles;
      const int n0 = nt * 256 + rank * 128;  // this CTA's first output row
      const int m0 = mt * BM;
      if (!warp_wait(acc_full(b), (it >> 1) & 1, abort_flag, p.status)) break;
      tc_fence_after();
      PS_T2(2 + 2 * (it & 1), e0 && it < 2);
      if (e0) bulk_wait_read_all();  // the previous tile's store has read the output tile
      epi2_bar();
      bool res_ok = true;
      if (p.resid) {
        if (e0) {
          mbar_expect_tx(res_full, BM * 256);
          tma_load_2d(out_sa, &maps.res, res_full, n0, m0);
        }
        res_ok = warp_wait(res_full, it & 1, abort_flag, p.status);
      }
      const int n = n0 + q * 32 + lane;  // this lane's output row (always < N: N % 256 == 0)
      const float sc = p.scale[n];
      const float bs = bias ? to_f32(bias[n]) : 0.f;
#pragma unroll 1
      for (int c = 0; c < BM; c += 32) {
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + b * BM + c, v);
        if (p.swiglu) {
          // lanes 2k / 2k+1 hold gate / up of intermediate channel
          // (n0 + q*32)/2 + k: each rounded to the linear's dtype, then
          // silu(gate) * up in float32; the pair splits the 32 tokens (even
          // lane 0..15, odd lane 16..31).
          const bool odd = lane & 1;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float mine_lo = to_f32(from_f32<T>(v[j] * sc + bs));
            const float mine_hi = to_f32(from_f32<T>(v[j + 16] * sc + bs));
            const float other = __shfl_xor_sync(0xffffffffu, odd ? mine_lo : mine_hi, 1);
            const float gate = odd ? other : mine_lo;
            const float up = odd ? mine_hi : other;
            out_tile[(c + j + (odd ? 16 : 0)) * 64 + q * 16 + (lane >> 1)] = from_f32<T>(silu_mul_f32(gate, up));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float o = v[j] * sc + bs;
            T* e = out_tile + (c + j) * 128 + q * 32 + lane;
            if (p.resid && res_ok) o = to_f32(from_f32<T>(o)) + to_f32(*e);
            *e = from_f32<T>(o);
          }
        }
      }
      tc_fence_before();
      fence_proxy_async();  // generic tile writes -> the TMA store
      epi2_bar();           // all 4 warps' TMEM reads and tile writes are done
      PS_T2(3 + 2 * (it & 1), e0 && it < 2);
      if (e0) {
        mbar_arrive_cluster(lead_empty + 8 * b);
        tma_store_2d(&maps.y, out_sa, p.swiglu ? n0 / 2 : n0, m0);
        bulk_commit();
      }
    }
    if (e0) bulk_wait_all();
  }
  // ------------------------------------------------------------ teardown --
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA exits while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

template <typename T, int BM>
int launch2(const Tc2Maps& maps, const Tc2Params& p, cudaStream_t s) {
  using C = Cfg2<BM>;
  auto kern = linear_tc2_kernel<T, BM>;
  static int max_pairs = 0;  // resident clusters of this instantiation (queried once)
  if (max_pairs == 0) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes) != cudaSuccess) {
      ps_host::set_error("linear_tc2: cannot reserve %d bytes of shared memory", C::kBytes);
      return PS_ERR_CUDA;
    }
    cudaLaunchConfig_t qc = {};
    qc.gridDim = dim3(2);
    qc.blockDim = dim3(kT2Threads);
    qc.dynamicSmemBytes = C::kBytes;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 2;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    qc.attrs = qa;
    qc.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &qc) != cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      ps_host::set_error("linear_tc2: no resident CTA pair");
      return PS_ERR_CUDA;
    }
    max_pairs = n;
  }
  const int pairs = p.tiles < max_pairs ? p.tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kT2Threads);
  cfg.dynamicSmemBytes = C::kBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = 2;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = 1;
  ++na;
  if (ps_host::pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps, p);
  if (e != cudaSuccess) {
    ps_host::set_error("linear_tc2: launch failed: %s", cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  ps_host::count_launch();
  return ps_host::check_launch("linear_tc2");
}

// Token tile: the BM in {128, 192} with the least padded work (ties: 192).
int pick_bm(int M) {
  const int t128 = (M + 127) / 128 * 128, t192 = (M + 191) / 192 * 192;
  return t192 <= t128 ? 192 : 128;
}

}  // namespace

#ifdef PS_TRACE
extern "C" PS_API int ps_debug_tc2_trace(unsigned long long* host, int n) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, g_tc2_trace, sizeof(unsigned long long) * n));
}
#endif

namespace ps_host {

// PS_TC2: unset / 0 = off (default: the single-CTA kernel measured faster
// on every shape of the step), 1 = on for the shapes below, 2 = wherever
// legal. Read on every call, so tests can switch it per case.
int tc2_mode() {
  const char* e = std::getenv("PS_TC2");
  if (!e) return 0;
  const int v = std::atoi(e);
  return v == 1 || v == 2 ? v : 0;
}

bool linear_tc2_eligible(int M, int N, int K, bool int8, const int8_t* w_tiled, bool push, int dtype) {
  const int mode = tc2_mode();
  if (mode == 0 || !int8 || !w_tiled || push || M <= 0 || N % 256 != 0 || K % 16 != 0) return false;
  if (dtype != PS_BF16 && dtype != PS_F16) return false;
  if (mode == 2) return true;  // forced (tests)
  // one full round of pairs at least: fewer tiles leave SMs idle, where the
  // single-CTA kernel's split-K does better
  const int bm = pick_bm(M);
  const long long tiles = static_cast<long long>(N / 256) * ((M + bm - 1) / bm);
  return M >= 96 && tiles >= 74;
}

int linear_tc2(void* y, const void* x, const int8_t* w_tiled, const float* scale, const void* bias,
               const void* resid, int M, int N, int K, int dtype, cudaStream_t s, bool swiglu) {
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(resid, 16) || !aligned(bias, 16) || !aligned(scale, 16) ||
      !aligned(w_tiled, 16) || (swiglu && resid))
    return PS_ERR_UNSUPPORTED;
  const int bm = pick_bm(M);
  Tc2Params p{};
  p.wt = w_tiled;
  p.scale = scale;
  p.bias = bias;
  p.resid = resid;
  p.status = status_word(PS_TU_GEMM);
  p.M = M;
  p.N = N;
  p.K = K;
  p.k_tiles = (K + kT2BK - 1) / kT2BK;
  p.m_tiles = (M + bm - 1) / bm;
  p.tiles = (N / 256) * p.m_tiles;
  p.swiglu = swiglu ? 1 : 0;
  const CUtensorMapDataType xdt =
      dtype == PS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  Tc2Maps maps;
  std::memset(&maps, 0, sizeof(maps));
  bool ok = make_map(&maps.x, x, xdt, 2, M, K, kT2BK, bm / 2, CU_TENSOR_MAP_SWIZZLE_128B);
  if (swiglu) ok = ok && make_map(&maps.y, y, xdt, 2, M, N / 2, 64, bm, CU_TENSOR_MAP_SWIZZLE_NONE);
  else ok = ok && make_map(&maps.y, y, xdt, 2, M, N, 128, bm, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (resid) ok = ok && make_map(&maps.res, resid, xdt, 2, M, N, 128, bm, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!ok) {
    set_error("linear_tc2: cuTensorMapEncodeTiled failed (M=%d N=%d K=%d)", M, N, K);
    return PS_ERR_CUDA;
  }
  if (dtype == PS_BF16)
    return bm == 192 ? launch2<__nv_bfloat16, 192>(maps, p, s) : launch2<__nv_bfloat16, 128>(maps, p, s);
  return bm == 192 ? launch2<__half, 192>(maps, p, s) : launch2<__half, 128>(maps, p, s);
}

}  // namespace ps_host
