// W8A16 (and 16-bit-weight) linear on the 5th-generation tensor cores:
//   y[m,n] = scale[n] * sum_k x[m,k] * w[n,k] + bias[n] (+ resid[m,n])
// (engine/quantization.py:26-50 + F.linear, engine/model.py:168-193 of the
// reference).
//
// Orientation ("swap AB"): the MMA's 128-row M dimension walks the weight's
// output channels and its N dimension walks the tokens, so a CTA owns a slab
// of NSUB*128 output channels for a tile of BM (<= 256) tokens and every
// weight byte is fetched and widened once per token tile. With NSUB = 2 two
// M=128 MMAs share each activation tile (half the activation traffic per
// flop); decode-sized batches use NSUB = 1 for more CTAs.
//
// Roles (352 threads), each ring with its own full/empty mbarrier pair:
//   warp 0      weight producer: one contiguous 8 KB bulk copy per 128-row
//               block of the pre-tiled int8 weight (a 2-D TMA for row-major
//               int8, or the 16-bit tile straight into the operand ring)
//   warp 1      TMEM allocator; one elected lane issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BM, K=16),
//               NSUB x 4 per k-tile, and commits to the rings' empty barriers
//   warp 2      activation producer: TMA of the bf16 tile (BM x 128 B,
//               128B swizzle) into its ring
//   warps 3..10 widen int8 -> bf16 (exact: |q| <= 127) straight into a
//               2..4-deep ring of MMA A operands in tensor memory (tcgen05.st; one
//               weight row per lane, K packed two bf16 per column), running up
//               to that many k-tiles ahead of the MMA, which reads A from TMEM
//               (tcgen05.mma ... [a_tmem]) and only the activations from
//               shared memory; then they run the epilogue
// Epilogue without a K split: the accumulators are read from TMEM
// (tcgen05.ld 32x32b; warp w reads lane quarter w%4), scaled, biased,
// residual-added (the residual tile TMA-loaded into the output tile first)
// or SiLU*up-combined, rounded into a token-major 16-bit tile and TMA-stored
// (to y, or to every rank's receive slot when pushing).
// The weight stream runs ahead independently of the MMA, so HBM latency is
// hidden by the weight ring depth rather than by the MMA's commit chain.
// Keeping the widened weights in TMEM takes their write and the MMA's read
// (64 KB per k-tile at 256 rows) off shared memory, whose bandwidth bounds
// this loop. bf16/f16 weights (the lm_head) skip the widening: TMA lands
// them in shared memory as the MMA's A operand directly.
// Small-N shapes split K across CTAs: the splits of one output tile form a
// thread-block cluster along z; after the main loop each CTA stages its fp32
// partial tile, bulk-copies token-row slice j to cluster CTA j
// (cp.async.bulk shared::cta -> shared::cluster), and each CTA sums its
// slice over the splits in fixed order, so the partial sums never leave the
// chip and no second kernel runs.
//
// Every mbarrier wait is bounded (about a second of clock64 cycles): on
// timeout the kernel records kErrTimeout in the status word, stops issuing
// work, releases its TMEM and returns.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "linear.cuh"
#include "tc_ptx.cuh"
#include "widen.cuh"

namespace {

using namespace ps;

constexpr int kThreads = 352;
constexpr int kDeqWarps = 8;
constexpr int kBK = 64;  // K elements per k-tile (128 bytes of bf16 = one swizzle row)
constexpr int kSmemBudget = 216 * 1024;

// Pipeline event timestamps of CTA (0,0,0) for latency analysis; compiled
// only with -DPS_TRACE (never in the shipped library).
#ifdef PS_TRACE
__device__ unsigned long long g_tc_trace[4096];
#define PS_TC_TRACE(slot, cond)                                                    \
  do {                                                                             \
    if ((cond) && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)           \
      g_tc_trace[(slot)] = clock64();                                              \
  } while (0)
#else
#define PS_TC_TRACE(slot, cond) \
  do {                          \
  } while (0)
#endif

// Barrier 1 among the 8 epilogue warps (warps 3..10).
PS_DEVICE void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

struct TcParams {
  const int8_t* wt;  // int8 weight pre-tiled in 8 KB blocks [N/128][K/64][128][64] (or null: row-major via TMA)
  int n_blocks;      // ceil(N / 128)
  void* y;
  const float* scale;
  const void* bias;
  const void* resid;
  int* status;
  int M, N, K;
  int k_tiles;      // total K tiles of 64
  int k_tiles_per_split;
  int splits;       // split-K CTAs per output tile = cluster size along z (1: no cluster)
  int tma_out;      // splits == 1 and N % 8 == 0: outputs leave by TMA stores (OutMaps)
  int swiglu;       // rows interleaved (2i gate_i, 2i+1 up_i): y[m][i] = silu(gate) * up, width N / 2
  int stagger;      // rotate each CTA's k-tile order (see kt_of in the kernel)
  float* ws;        // splits > 1: fp32 partial tiles [tile][split][NSUB][BM][128] in global memory (null: DSMEM)
  PushTargets push;  // world > 0: the final output goes to every rank's receive slot instead of y
};

// Tensor maps of the TMA-stored outputs (bf16/f16 [rows][N], box 128 x BM).
struct OutMaps {
  CUtensorMap y;                // output [M][N]
  CUtensorMap res;              // residual [M][N]
  CUtensorMap dst[kMaxWorld];   // push: every rank's slot [max_tokens][N]
};

// Shared-memory plan of one configuration.
template <bool kInt8, int NSUB, int BM>
struct Cfg {
  static constexpr int kBN = 128 * NSUB;
  static constexpr int kW = kInt8 ? kBN * kBK : kBN * kBK * 2;  // weight ring stage
  static constexpr int kX = BM * kBK * 2;                        // activation ring stage
  static constexpr int kA = 0;                                   // widened operands live in TMEM
  static constexpr int kAS = 0;
  static constexpr int kAccCols = NSUB * BM;                       // fp32 accumulators
  static constexpr int kACols = kInt8 ? NSUB * (kBK / 2) : 0;      // one TMEM A stage (2 bf16 per column)
  static constexpr int kStage = BM * 128 * 4;                     // epilogue fp32 stage [BM][128]
  static constexpr int kRX0 = (120 * 1024) / kX;
  static constexpr int kRX = kRX0 < 2 ? 2 : (kRX0 > 8 ? 8 : kRX0);
  // Pre-tiled int8 weights arrive as one bulk copy of kJ consecutive k-tiles
  // per 128-row block (contiguous in the tiled layout): a thread issues about
  // one bulk copy per ~675 cycles whatever its size (measured on B200), so
  // 8 KB copies would cap the weight stream below the MMA rate. The ring has
  // kRW k-tile slots in groups of kJ, one full/empty barrier pair per group.
  static constexpr int kJ = kInt8 ? 2 : 1;
  static constexpr int kRW0 = (kSmemBudget - kAS * kA - kRX * kX) / kW;
  static constexpr int kRW1 = kRW0 > 8 * kJ ? 8 * kJ : kRW0;
  static constexpr int kRW = (kRW1 / kJ) * kJ < 2 * kJ ? 2 * kJ : (kRW1 / kJ) * kJ;
  // layout (1024-aligned rings first): A | W | X | barriers. The epilogue's
  // stage reuses the rings, idle once the main loop is done.
  static constexpr int kOffA = 0;
  static constexpr int kOffW = kOffA + kAS * kA;
  static constexpr int kOffX = kOffW + kRW * kW;
  static constexpr int kOffStage = kOffW;
  static constexpr int kOffBar = kOffX + kRX * kX;
  static constexpr int kBytes = kOffBar + 512 + 1024;
  // widened-A stages in TMEM: as many as fit beside the accumulators (2..4);
  // small token tiles get a deeper ring, which hides the widen -> MMA ->
  // commit round trip when the MMAs are short
  static constexpr int kATm = kInt8 ? ((512 - kAccCols) / kACols >= 4 ? 4 : ((512 - kAccCols) / kACols >= 3 ? 3 : 2))
                                    : 2;
  static constexpr int kTmemNeed = kAccCols + kATm * kACols;  // accumulators + the A stages
  static constexpr int kTmemCols = kTmemNeed <= 32 ? 32 : (kTmemNeed <= 64 ? 64 : (kTmemNeed <= 128 ? 128 :
                                   (kTmemNeed <= 256 ? 256 : 512)));
  static_assert(kBytes <= 227 * 1024, "shared memory plan too large");
  static constexpr int kRings = kRW * kW + kRX * kX;
  static_assert(kRings >= kStage, "epilogue stage aliases the rings");
  static_assert(kRings >= NSUB * BM * 256, "TMA output tiles alias the rings");
  static_assert(kTmemNeed <= 512, "TMEM columns");
  static_assert(kW % 1024 == 0 && kX % 1024 == 0 && kA % 1024 == 0, "1024-byte aligned stages");
  static_assert(kRW % kJ == 0 && kRW / kJ <= 8, "weight ring groups");
};

template <typename T, bool kInt8, int NSUB, int BM>
__global__ void __launch_bounds__(kThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                     const TcParams p, const __grid_constant__ OutMaps om) {
  using C = Cfg<kInt8, NSUB, BM>;
  constexpr int RW = C::kRW, RX = C::kRX;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  auto w_addr = [&](int s) { return base + C::kOffW + s * C::kW; };
  // Weight ring: WG groups of WJ k-tile slots; group g holds, per sub-tile,
  // WJ consecutive 8 KB k-tile blocks (one bulk copy each for the tiled
  // layout). Every ring index below divides by compile-time constants only:
  // the per-k-tile loops are latency chains, and a runtime division costs
  // more than the widening itself.
  constexpr int WJ = C::kJ;
  constexpr int WG = RW / WJ;
  auto x_addr = [&](int s) { return base + C::kOffX + s * C::kX; };
  const uint32_t bars = base + C::kOffBar;
  auto w_full = [&](int s) { return bars + 8 * s; };
  auto w_empty = [&](int s) { return bars + 8 * (8 + s); };
  auto x_full = [&](int s) { return bars + 8 * (16 + s); };
  auto x_empty = [&](int s) { return bars + 8 * (24 + s); };
  constexpr int AS = C::kATm;
  auto a_full = [&](int s) { return bars + 8 * (32 + s); };
  auto a_empty = [&](int s) { return bars + 8 * (36 + s); };
  const uint32_t acc_full = bars + 8 * 40;
  const uint32_t res_full = bars + 8 * 41;   // residual tiles landed (TMA output path)
  const uint32_t recv_full = bars + 8 * 42;  // split-K slices from the cluster peers landed
  unsigned char* misc = gbase + C::kOffBar + 8 * 44;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * C::kBN;
  const int m0 = blockIdx.y * BM;
  const int split = blockIdx.z;
  const int kt0 = split * p.k_tiles_per_split;
  const int kt1 = min(p.k_tiles, kt0 + p.k_tiles_per_split);
  const int nkt = kt1 - kt0;
  // K order: each CTA starts at a different whole weight group (rotation
  // among the full groups of its split; a partial last group stays last), so
  // the CTAs that share a token tile do not all request the same activation
  // k-tile at once. Sequence position i -> k-tile offset inside the split.
  const int nfull = nkt / WJ;
  const int rot = (p.stagger && nfull > 1) ? static_cast<int>((blockIdx.x * 5u + blockIdx.y * 3u) % nfull) : 0;
  auto kt_of = [&](int i) {
    if (i >= nfull * WJ) return i;
    const int g = i / WJ;
    int ag = g + rot;
    if (ag >= nfull) ag -= nfull;
    return ag * WJ + (i - g * WJ);
  };

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < WG; ++s) {
      mbar_init(w_full(s), 1);
      mbar_init(w_empty(s), kInt8 ? (kDeqWarps / 2) * WJ : 1);
    }
    for (int s = 0; s < RX; ++s) {
      mbar_init(x_full(s), 1);
      mbar_init(x_empty(s), 1);
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init(a_full(s), kDeqWarps / 2);
      mbar_init(a_empty(s), 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(res_full, 1);
    mbar_init(recv_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  PS_TC_TRACE(0, threadIdx.x == 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  PS_TC_TRACE(1, threadIdx.x == 0);
  // Programmatic dependent launch: the weight producer starts streaming the
  // (never written) weights while the previous kernel finishes; every other
  // role waits for it before reading activations / residuals or writing.
  pdl_trigger();
  if (warp != 0) pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------- weight producer --
    const int b0 = blockIdx.x * NSUB;
    const int nb = min(NSUB, p.n_blocks - b0);  // row blocks past the last are not loaded (outputs masked)
    for (int i = 0; i < nkt; i += WJ) {
      const int grp = i / WJ;
      const int s = grp % WG;
      if (grp >= WG && !warp_wait(w_empty(s), ((grp / WG) - 1) & 1, abort_flag, p.status)) break;
      PS_TC_TRACE(16 + (i & 255) * 8 + 0, lane == 0);
      if (lane == 0) {
        const int kt = kt0 + kt_of(i);
        const uint32_t dst = w_addr(s * WJ);
        if (kInt8) {
          const int nk = min(WJ, nkt - i);
          mbar_expect_tx(w_full(s), nb * nk * 8192);
          for (int sub = 0; sub < nb; ++sub) {
            if (p.wt) {  // tiled: nk consecutive 8 KB k-tile blocks of row block b0+sub are contiguous
              bulk_load(dst + sub * WJ * 8192, p.wt + (static_cast<long long>(b0 + sub) * p.k_tiles + kt) * 8192,
                        nk * 8192, w_full(s));
            } else {  // row-major: one 128-row x 64 box per k-tile
              for (int j = 0; j < nk; ++j)
                tma_load_2d(dst + (sub * WJ + j) * 8192, &wmap, w_full(s), (kt + j) * kBK, n0 + sub * 128);
            }
          }
        } else {
          mbar_expect_tx(w_full(s), C::kW);
          tma_load_2d(dst, &wmap, w_full(s), kt * kBK, n0);
        }
      }
      __syncwarp();
    }
  } else if (warp == 2) {
    // --------------------------------------------- activation producer --
    for (int i = 0; i < nkt; ++i) {
      const int s = i % RX;
      if (i >= RX && !warp_wait(x_empty(s), ((i / RX) - 1) & 1, abort_flag, p.status)) break;
      PS_TC_TRACE(16 + (i & 255) * 8 + 1, lane == 0);
      if (lane == 0) {
        mbar_expect_tx(x_full(s), C::kX);
        tma_load_2d(x_addr(s), &xmap, x_full(s), (kt0 + kt_of(i)) * kBK, m0);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer --
    constexpr uint32_t idesc = instr_desc(!std::is_same<T, __half>::value, 128, BM);
    bool ok = nkt > 0;
    for (int i = 0; i < nkt; ++i) {
      const int sx = i % RX;
      const int sa = kInt8 ? (i % AS) : (i % RW);
      ok = warp_wait(kInt8 ? a_full(sa) : w_full(sa), kInt8 ? ((i / AS) & 1) : ((i / RW) & 1), abort_flag,
                     p.status);
      PS_TC_TRACE(16 + (i & 255) * 8 + 6, lane == 0);
      if (ok) ok = warp_wait(x_full(sx), (i / RX) & 1, abort_flag, p.status);
      if (!ok) break;
      tc_fence_after();
      PS_TC_TRACE(16 + (i & 255) * 8 + 4, lane == 0);
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t bd = smem_desc_sw128(x_addr(sx) + kk * 32);
#pragma unroll
          for (int sub = 0; sub < NSUB; ++sub) {
            if constexpr (kInt8) {
              const uint32_t ta = tmem + C::kAccCols + sa * C::kACols + sub * (kBK / 2) + kk * 8;
              mma_ts(tmem + sub * BM, ta, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint64_t ad = smem_desc_sw128(w_addr(sa) + sub * (128 * 128) + kk * 32);
              mma_f16(tmem + sub * BM, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
            }
          }
        }
        mma_commit(kInt8 ? a_empty(sa) : w_empty(sa));
        mma_commit(x_empty(sx));
      }
      __syncwarp();
    }
    if (ok && lane == 0) mma_commit(acc_full);
    __syncwarp();
  } else {
    const int t = threadIdx.x - 96;  // 0 .. 32*kDeqWarps-1
    (void)t;
    // ------------------------------------- int8 -> bf16 widening into TMEM --
    // Warp (q = warp % 4, h = (warp - 3) / 4) owns TMEM lanes [32q, 32q+32)
    // (one weight row per lane) and every other k-tile (parity h): each
    // iteration widens the row's whole k-tile of every sub-tile, so the two
    // teams' per-k-tile round trips (wait, load, widen, TMEM store, arrive)
    // overlap instead of adding up.
    if (kInt8) {
      const int q = warp & 3;
      const int h = (warp - 3) >> 2;
      const int rin = q * 32 + lane;                        // row inside the 128-row block
      const int swz = p.wt ? ((rin >> 1) & 3) : 0;           // chunk slot swizzle of the tiled layout
      constexpr int kChunks = 4;                             // 16-byte chunks of one row per sub-tile
      const unsigned char* wring = gbase + C::kOffW + rin * 64;
      const uint32_t tlane = tmem + (static_cast<uint32_t>(q * 32) << 16) + C::kAccCols;
      for (int i = h; i < nkt; i += 2) {
        const int grp = i / WJ;
        const int jj = i - grp * WJ;
        const int sw = grp % WG;
        const int sa = i % AS;
        if (!warp_wait(w_full(sw), (grp / WG) & 1, abort_flag, p.status)) break;
        PS_TC_TRACE(16 + (i & 255) * 8 + 5, t == 0);
        // widen in registers first: only the TMEM store waits for the stage
        uint32_t words[NSUB][kChunks * 8];
#pragma unroll
        for (int sub = 0; sub < NSUB; ++sub) {
          const unsigned char* row = wring + (sw * WJ * NSUB + sub * WJ + jj) * 8192;
#pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            const uint4 in = *reinterpret_cast<const uint4*>(row + ((c ^ swz) << 4));
            uint4 lo, hi;
            if constexpr (std::is_same<T, __half>::value) widen16_f16(in, lo, hi);
            else widen16_bf16(in, lo, hi);
            uint32_t* w8 = words[sub] + c * 8;
            w8[0] = lo.x; w8[1] = lo.y; w8[2] = lo.z; w8[3] = lo.w;
            w8[4] = hi.x; w8[5] = hi.y; w8[6] = hi.z; w8[7] = hi.w;
          }
        }
        if (i >= AS && !warp_wait(a_empty(sa), ((i / AS) - 1) & 1, abort_flag, p.status)) break;
        tc_fence_after();
        PS_TC_TRACE(16 + (i & 255) * 8 + 2, t == 0);
#pragma unroll
        for (int sub = 0; sub < NSUB; ++sub) {
          const uint32_t ta = tlane + sa * C::kACols + sub * (kBK / 2);
          tmem_st16(ta, words[sub]);
          tmem_st16(ta + 16, words[sub] + 16);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(a_full(sa));
          mbar_arrive(w_empty(sw));
        }
        PS_TC_TRACE(16 + (i & 255) * 8 + 3, t == 0);
      }
    }
  }
  // -------------------------------------------------------------- epilogue --
  // Every warp of every CTA of the cluster takes the same barriers here; the
  // rings are idle once acc_full fired, so the epilogue's buffers alias them.
  //  * splits == 1, N % 8 == 0: per 128-row sub-tile the epilogue warps read
  //    the accumulators from TMEM (lane = weight row n, 32 tokens at a time),
  //    apply scale / bias / residual (the residual tile arrives by TMA into
  //    the output tile first), write dtype values into a token-major
  //    [BM][128] tile and one thread TMA-stores it (to y, or to every rank's
  //    slot when pushing).
  //  * splits > 1: the splits of a tile form a cluster. Each stages its fp32
  //    accumulators ([BM][128] per sub-tile), then bulk-copies token-row
  //    slice j to cluster CTA j, which sums the S slices in split order from
  //    its own shared memory and stores 8 outputs per thread.
  //  * splits == 1, N % 8 != 0: per-lane scalar stores (ragged widths).
  {
    bool ok = true;
    if (warp >= 3) {
      ok = nkt > 0 && warp_wait(acc_full, 0, abort_flag, p.status);
      tc_fence_after();
    }
    PS_TC_TRACE(2, threadIdx.x == 96);
    const T* bias = static_cast<const T*>(p.bias);
    const T* resid = static_cast<const T*>(p.resid);
    T* y = static_cast<T*>(p.y);
    const int S = p.splits;
    const int q = warp & 3;              // TMEM lane quarter (epilogue warps)
    const int h = (warp - 3) >> 2;       // alternating 32-token chunks
    if (S == 1) {
      const uint32_t out_sa = base + C::kOffStage;  // NSUB tiles of [BM][128] dtype
      T* out_tile = reinterpret_cast<T*>(gbase + C::kOffStage);
      const bool use_tma = p.tma_out != 0;
      if (use_tma && resid && threadIdx.x == 96) {
        mbar_expect_tx(res_full, NSUB * BM * 256);
        for (int sub = 0; sub < NSUB; ++sub) tma_load_2d(out_sa + sub * BM * 256, &om.res, res_full, n0 + sub * 128, m0);
      }
      if (warp >= 3) {
        const bool res_ok = !(use_tma && resid) || warp_wait(res_full, 0, abort_flag, p.status);
#pragma unroll 1
        for (int sub = 0; sub < NSUB; ++sub) {
          const int n = n0 + sub * 128 + q * 32 + lane;  // this lane's output column
          const float sc = (n < p.N && p.scale) ? p.scale[n] : 1.f;
          const float bs = (n < p.N && bias) ? to_f32(bias[n]) : 0.f;
          T* tile = out_tile + sub * BM * 128;
#pragma unroll 1
          for (int c = 32 * h; c < BM; c += 64) {
            float v[32];
            if (ok) tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + sub * BM + c, v);
            if (use_tma && p.swiglu) {
              // lanes 2k / 2k+1 hold gate / up of intermediate channel
              // (n0 + sub*128 + q*32)/2 + k: each rounded to dtype (the
              // linear's output), then silu(gate) * up in float32.
              T* tile2 = out_tile + sub * BM * 64;  // [BM][64] per sub-tile
              // The pair splits the 32 tokens: the even lane finishes tokens
              // 0..15, the odd lane 16..31 (one exchange per token pair).
              // Written as independent batches (round all, exchange all,
              // SiLU all, store all): one output's chain of ~15 dependent
              // steps is far longer than its instruction count.
              const bool odd = lane & 1;
              float keep[16], send[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                // both values rounded to the linear's dtype by one packed convert
                const float2 r = round2<T>(v[j] * sc + bs, v[j + 16] * sc + bs);
                keep[j] = odd ? r.y : r.x;
                send[j] = odd ? r.x : r.y;
              }
#pragma unroll
              for (int j = 0; j < 16; ++j) send[j] = __shfl_xor_sync(0xffffffffu, send[j], 1);
#pragma unroll
              for (int j = 0; j < 16; ++j) keep[j] = odd ? silu_mul_f32(send[j], keep[j]) : silu_mul_f32(keep[j], send[j]);
              T* col = tile2 + (c + (odd ? 16 : 0)) * 64 + q * 16 + (lane >> 1);
#pragma unroll
              for (int j = 0; j < 16; ++j) col[j * 64] = from_f32<T>(keep[j]);
            } else if (use_tma) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                float o = v[j] * sc + bs;
                T* e = tile + (c + j) * 128 + q * 32 + lane;
                if (resid && res_ok) o = to_f32(from_f32<T>(o)) + to_f32(*e);
                *e = from_f32<T>(o);
              }
            } else if (ok && n < p.N) {
#pragma unroll 4
              for (int j = 0; j < 32; ++j) {
                const int m = m0 + c + j;
                if (m < p.M) {
                  float o = v[j] * sc + bs;
                  if (resid) o = to_f32(from_f32<T>(o)) + to_f32(resid[static_cast<long long>(m) * p.N + n]);
                  y[static_cast<long long>(m) * p.N + n] = from_f32<T>(o);
                }
              }
            }
          }
          if (use_tma) {
            fence_proxy_async();
            epi_bar();
            if (threadIdx.x == 96) {
              if (p.swiglu) {
                tma_store_2d(&om.y, out_sa + sub * BM * 128, (n0 + sub * 128) / 2, m0);
              } else if (p.push.world > 0) {
                const int n = n0 + sub * 128;
                if (p.push.slice) {  // two-shot: the owner of these 128 columns only
                  const int d = n / p.push.slice;
                  if (n < p.N) tma_store_2d(&om.dst[d], out_sa + sub * BM * 256, n - d * p.push.slice, m0);
                } else {
                  for (int d = 0; d < p.push.world; ++d) tma_store_2d(&om.dst[d], out_sa + sub * BM * 256, n, m0);
                }
              } else {
                tma_store_2d(&om.y, out_sa + sub * BM * 256, n0 + sub * 128, m0);
              }
              bulk_commit();
            }
          }
        }
        if (use_tma && threadIdx.x == 96) {
          bulk_wait_all();  // stores done (pushed outputs complete before the arrival below)
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
      }
    } else {
      // ------------------------------------------------ split-K cluster --
      float* stage = reinterpret_cast<float*>(gbase + C::kOffStage);
      const uint32_t stage_sa = base + C::kOffStage;
      const uint32_t recv_sa = stage_sa + BM * 512;
      const int crank = static_cast<int>(cluster_ctarank());
      const int share = (BM + S - 1) / S;
      const int r0 = min(BM, crank * share);
      const int r1 = min(BM, r0 + share);
      const int my_rows = r1 - r0;
      const int ndst = p.push.world > 0 ? p.push.world : 1;
      // With a workspace the splits exchange their partial tiles through L2:
      // each stages its fp32 tile in shared memory and writes it to its
      // workspace slot with one bulk store; a GPU-scope fence and the cluster
      // barrier publish them, and each CTA sums its token-row slice over the
      // splits in split order (ld.cg, all splits' loads in flight at once).
      // Bulk copies between the CTAs' shared memories (the fallback without
      // a workspace) measured ~13 GB/s per SM on B200, several us per tile.
      const long long tile = static_cast<long long>(blockIdx.y) * gridDim.x + blockIdx.x;
      auto part = [&](int sr, int sub_) {
        return p.ws + ((tile * S + sr) * NSUB + sub_) * static_cast<long long>(BM) * 128;
      };
#pragma unroll 1
      for (int sub = 0; sub < NSUB; ++sub) {
        // thread t sums columns n8 = 8 * (t % 16) of the sub-tile, 22 rows per
        // pass; its scales and biases are requested before the exchange
        const int n8 = (threadIdx.x & 15) * 8;
        const int gn = n0 + sub * 128 + n8;
        const int cnt = min(8, p.N - gn);
        float sc[8], bs[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          sc[j] = (j < cnt && p.scale) ? p.scale[gn + j] : 1.f;
          bs[j] = (j < cnt && bias) ? to_f32(bias[gn + j]) : 0.f;
        }
        if (warp >= 3 && ok) {
#pragma unroll 1
          for (int c = 32 * h; c < BM; c += 64) {
            float v[32];
            tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + sub * BM + c, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) stage[(c + j) * 128 + q * 32 + lane] = v[j];
          }
        }
        if (p.ws) {
          fence_proxy_async();  // generic stage writes -> the bulk stores
          __syncthreads();
          // publish only the row slices the peers own (this CTA's own rows
          // stay in shared memory); slice j leaves from lane 0 of warp 3 + j
          if (lane == 0 && warp >= 3 && warp - 3 < S && warp - 3 != crank) {
            const int j0 = min(BM, (warp - 3) * share);
            const int rows = min(BM, j0 + share) - j0;
            if (rows > 0) {
              bulk_store(part(crank, sub) + j0 * 128, stage_sa + j0 * 512, rows * 512);
              bulk_commit();
              bulk_wait_all();
              asm volatile("fence.proxy.async.global;" ::: "memory");
            }
          }
          __threadfence();
          PS_TC_TRACE(5 + sub * 4, threadIdx.x == 96);
          cluster_sync();  // every split's partial tile is in L2
          PS_TC_TRACE(6 + sub * 4, threadIdx.x == 96);
        } else {
          fence_proxy_async();  // generic stage writes -> the bulk copies below
          if (threadIdx.x == 96) mbar_expect_tx(recv_full, (S - 1) * my_rows * 512);
          PS_TC_TRACE(5 + sub * 4, threadIdx.x == 96);
          cluster_sync();  // every split staged; every peer's rings idle
          PS_TC_TRACE(6 + sub * 4, threadIdx.x == 96);
          // the copy to peer j leaves from lane 0 of warp 3 + j: a thread issues
          // about one bulk copy per ~700 cycles, so one thread for all S - 1
          // copies would serialise them
          if (lane == 0 && warp >= 3 && warp - 3 < S && warp - 3 != crank) {
            const int j = warp - 3;
            const int j0 = min(BM, j * share);
            const int rows = min(BM, j0 + share) - j0;
            if (rows > 0) {
              const int slot = crank < j ? crank : crank - 1;  // my slot among j's S-1 senders
              bulk_s2s(mapa_shared(recv_sa + slot * share * 512, j), stage_sa + j0 * 512, rows * 512,
                       mapa_shared(recv_full, j));
            }
          }
        }
        const bool got = p.ws ? true : warp_wait(recv_full, sub & 1, abort_flag, p.status);
        if (got && gn < p.N) {
          const bool vec = (p.N % 8) == 0;
          // L2 path, full 16-byte groups: the residual and every split's
          // partial are requested before any is summed (each pass is one round
          // trip to L2 instead of S + 1).
          constexpr int kRowStep = kThreads / 16;
          // rows per pass sized to the split count (registers: R x SMAX x 32 B)
          auto l2_rows = [&](auto RT, auto ST) {
            constexpr int R = decltype(RT)::value;
            constexpr int SMAX = decltype(ST)::value;
#pragma unroll 1
            for (int m = r0 + (threadIdx.x >> 4); m < r1; m += R * kRowStep) {
              float4 pa[R][SMAX], pb[R][SMAX];
              uint4 rres[R];
              bool live[R];
#pragma unroll
              for (int u = 0; u < R; ++u) {
                const int mm = m + u * kRowStep;
                live[u] = mm < r1 && m0 + mm < p.M;
                rres[u] = make_uint4(0, 0, 0, 0);
                if (!live[u]) continue;
                if (resid) rres[u] = *reinterpret_cast<const uint4*>(resid + static_cast<long long>(m0 + mm) * p.N + gn);
#pragma unroll
                for (int sr = 0; sr < SMAX; ++sr) {
                  if (sr < S) {
                    const float4* src = sr == crank ? reinterpret_cast<const float4*>(stage + mm * 128 + n8)
                                                    : reinterpret_cast<const float4*>(part(sr, sub) + mm * 128 + n8);
                    pa[u][sr] = sr == crank ? src[0] : __ldcg(src);
                    pb[u][sr] = sr == crank ? src[1] : __ldcg(src + 1);
                  }
                }
              }
#pragma unroll
              for (int u = 0; u < R; ++u) {
                if (!live[u]) continue;
                const int gm = m0 + m + u * kRowStep;
                float acc[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
                for (int sr = 0; sr < SMAX; ++sr) {  // split order: identical sums on every run
                  if (sr < S) {
                    acc[0] += pa[u][sr].x; acc[1] += pa[u][sr].y; acc[2] += pa[u][sr].z; acc[3] += pa[u][sr].w;
                    acc[4] += pb[u][sr].x; acc[5] += pb[u][sr].y; acc[6] += pb[u][sr].z; acc[7] += pb[u][sr].w;
                  }
                }
                float rv[8];
                if (resid) unpack8<T>(rres[u], rv);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  acc[j] = acc[j] * sc[j] + bs[j];
                  if (resid) acc[j] = to_f32(from_f32<T>(acc[j])) + rv[j];
                }
                const uint4 pk = pack8<T>(acc);
                const long long off = static_cast<long long>(gm) * p.N + gn;
                if (p.push.world > 0 && p.push.slice) {  // two-shot: the owner of these columns only
                  const int d = gn / p.push.slice;
                  *reinterpret_cast<uint4*>(static_cast<T*>(p.push.dst[d]) + push_offset(p.push, gm, gn, p.N, d)) = pk;
                } else {
                  for (int d = 0; d < ndst; ++d)  // push: every rank's slot (peers over NVLink)
                    *reinterpret_cast<uint4*>((p.push.world > 0 ? static_cast<T*>(p.push.dst[d]) : y) + off) = pk;
                }
              }
            }
          };
          if (p.ws && vec) {
            if (S <= 2) l2_rows(std::integral_constant<int, 2>{}, std::integral_constant<int, 2>{});
            else l2_rows(std::integral_constant<int, 1>{}, std::integral_constant<int, 8>{});
          } else {
#pragma unroll 1
          for (int m = r0 + (threadIdx.x >> 4); m < r1; m += kThreads / 16) {
            const int gm = m0 + m;
            if (gm >= p.M) continue;
            float acc[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = 0.f;
            if (p.ws) {
              for (int sr = 0; sr < S; ++sr) {  // split order: identical sums on every run
                const float4* src = sr == crank ? reinterpret_cast<const float4*>(stage + m * 128 + n8)
                                                : reinterpret_cast<const float4*>(part(sr, sub) + m * 128 + n8);
                const float4 a = sr == crank ? src[0] : __ldcg(src);
                const float4 b = sr == crank ? src[1] : __ldcg(src + 1);
                acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
                acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
              }
            } else {
              for (int sr = 0; sr < S; ++sr) {  // split order: identical sums on every run
                const float* src = sr == crank ? stage + m * 128 + n8
                                               : reinterpret_cast<const float*>(gbase + C::kOffStage + BM * 512) +
                                                     ((sr < crank ? sr : sr - 1) * share + (m - r0)) * 128 + n8;
                const float4 a = reinterpret_cast<const float4*>(src)[0];
                const float4 b = reinterpret_cast<const float4*>(src)[1];
                acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
                acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
              }
            }
            const long long off = static_cast<long long>(gm) * p.N + gn;
            if (vec) {
              float rv[8];
              if (resid) unpack8<T>(*reinterpret_cast<const uint4*>(resid + off), rv);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                acc[j] = acc[j] * sc[j] + bs[j];
                if (resid) acc[j] = to_f32(from_f32<T>(acc[j])) + rv[j];
              }
              const uint4 pk = pack8<T>(acc);
              if (p.push.world > 0 && p.push.slice) {  // two-shot: the owner of these columns only
                const int d = gn / p.push.slice;
                *reinterpret_cast<uint4*>(static_cast<T*>(p.push.dst[d]) + push_offset(p.push, gm, gn, p.N, d)) = pk;
              } else {
                for (int d = 0; d < ndst; ++d)  // push: every rank's slot (peers over NVLink)
                  *reinterpret_cast<uint4*>((p.push.world > 0 ? static_cast<T*>(p.push.dst[d]) : y) + off) = pk;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                if (j < cnt) {
                  float v2 = acc[j] * sc[j] + bs[j];
                  if (resid) v2 = to_f32(from_f32<T>(v2)) + to_f32(resid[off + j]);
                  y[off + j] = from_f32<T>(v2);
                }
              }
            }
          }
          }
        }
        PS_TC_TRACE(7 + sub * 4, threadIdx.x == 96);
        // slices consumed: stage and receive buffers free again (the L2 path
        // writes each sub-tile's partials to slots of their own, so only this
        // CTA's stage must be released)
        if (p.ws) __syncthreads();
        else cluster_sync();
        PS_TC_TRACE(8 + sub * 4, threadIdx.x == 96);
      }
    }
  }
  PS_TC_TRACE(3, threadIdx.x == 96);
  tc_fence_before();
  __syncthreads();
  PS_TC_TRACE(4, threadIdx.x == 0);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
  }
  if (p.push.world > 0) push_arrive(p.push);
}

// Re-tile a row-major int8 weight [N][K] into 8 KB blocks [N/128][K/64][128][64]
// (zero padded), so one weight tile of the main loop is one contiguous copy.
// Inside a block, the 16-byte chunk c of row r sits in slot c ^ ((r >> 1) & 3),
// so the widening warps (one row per lane) read shared memory without bank
// conflicts.
__global__ void tile_int8_kernel(int8_t* __restrict__ dst, const int8_t* __restrict__ src, int N, int K, int kt) {
  const long long total = static_cast<long long>((N + 127) / 128) * kt * 8192 / 16;  // 16-byte units
  for (long long u = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; u < total;
       u += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long blk = u / 512;  // 8192 / 16
    const int within = static_cast<int>(u % 512);
    const int r = within >> 2, c16 = within & 3;
    const int b = static_cast<int>(blk / kt), k_tile = static_cast<int>(blk % kt);
    const int n = b * 128 + r, k = k_tile * 64 + c16 * 16;
    alignas(16) int8_t v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = (n < N && k + i < K) ? src[static_cast<long long>(n) * K + k + i] : 0;
    const long long slot = blk * 512 + r * 4 + (c16 ^ ((r >> 1) & 3));
    reinterpret_cast<uint4*>(dst)[slot] = *reinterpret_cast<const uint4*>(v);
  }
}

struct Plan {
  int nsub, bm, m_tiles, n_tiles, k_tiles, splits, per_split;
};

// PS_LINEAR_STAGGER=0 walks K in the same order in every CTA (tuning).
bool stagger_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("PS_LINEAR_STAGGER");
    return !(e && e[0] == '0');
  }();
  return v;
}

int snap_bm(int bm) { return bm <= 32 ? 32 : (bm <= 64 ? 64 : (bm <= 128 ? 128 : (bm <= 192 ? 192 : 256))); }

// Tile plan (rules measured on B200 with CUDA-graph timing over the
// Qwen2.5-3B projection shapes). Token tiles: one tile up to 256 tokens, else
// equal tiles. Prefill-sized token tiles (>= 128): wide outputs (N >= 8192)
// take 256-row weight slabs (two M=128 MMAs share each activation tile);
// long-K narrow outputs take 256-row slabs with K split so the grid is about
// one wave; short-K narrow outputs take 128-row slabs split in two.
// Decode-sized token tiles: 128-row slabs, or 256-row slabs when 128-row
// slabs would need a second, mostly empty wave; K split when the slabs alone
// leave most SMs idle. PS_LINEAR_TILE="nsub,bm,splits" overrides (tuning).
Plan plan(int M, int N, int K, bool int8) {
  Plan pl{};
  const int mt = (M + 255) / 256;
  pl.bm = snap_bm((((M + mt - 1) / mt) + 15) / 16 * 16);
  pl.k_tiles = (K + kBK - 1) / kBK;
  int m_tiles = (M + pl.bm - 1) / pl.bm;
  const int nt1 = (N + 127) / 128, nt2 = (N + 255) / 256;
  int splits = 1;
  if (pl.bm >= 128) {
    // Narrow outputs with few token tiles (M up to ~256) would leave most SMs
    // idle even after the K split: 128-token tiles double the tile count.
    const int m128 = (M + 127) / 128;
    if (N >= 8192) {
      pl.nsub = 2;
    } else if (K >= 8192) {
      pl.nsub = 2;
      if (pl.bm > 128 && nt2 * m_tiles * 8 < 100) {
        pl.bm = 128;
        m_tiles = m128;
      }
      splits = 148 / (nt2 * m_tiles);
      if (splits > 8) splits = 8;
    } else {
      pl.nsub = 1;
      splits = 2;
      if (pl.bm > 128 && nt1 * m_tiles * 2 < 74) {
        pl.bm = 128;
        m_tiles = m128;
        splits = 148 / (nt1 * m_tiles);
        if (splits > 4) splits = 4;
        if (splits < 1) splits = 1;
      } else if (pl.bm == 128) {
        // one token tile of 65..128 tokens: split K to about one wave
        // (M=128 q|k|v N=3584 K=5120: 25.6 -> 17.4 us; o_proj N=5120
        // K=2560: 16.2 -> 14.2 us)
        splits = 148 / (nt1 * m_tiles);
        if (splits > 8) splits = 8;
        if (splits < 2) splits = 2;
      }
    }
  } else {
    pl.nsub = (nt1 * m_tiles > 148 && nt2 * m_tiles <= 148) ? 2 : 1;
    const int tiles = m_tiles * (pl.nsub == 2 ? nt2 : nt1);
    if (tiles < 100) splits = 148 / tiles;
  }
  if (const char* env = std::getenv("PS_LINEAR_TILE")) {
    int a = 0, b = 0, c = 0;
    if (sscanf(env, "%d,%d,%d", &a, &b, &c) >= 2 && (a == 1 || a == 2)) {
      pl.nsub = a;
      pl.bm = snap_bm(b);
      splits = c > 0 ? c : 1;
    }
  }
  if (int8 && pl.nsub == 2 && pl.bm > 192) {  // TMEM: 2 x BM accumulators + 2 x 64 A columns <= 512
    const int mt2 = (M + 191) / 192;
    pl.bm = snap_bm((((M + mt2 - 1) / mt2) + 15) / 16 * 16);
    if (pl.bm > 192) pl.bm = 192;
  }
  pl.m_tiles = (M + pl.bm - 1) / pl.bm;
  pl.n_tiles = (N + 128 * pl.nsub - 1) / (128 * pl.nsub);
  const int max_split = pl.k_tiles / 4 > 0 ? pl.k_tiles / 4 : 1;  // >= 4 K tiles per split
  if (splits > max_split) splits = max_split;
  if (splits > 8) splits = 8;  // one portable cluster per output tile
  if (splits < 1) splits = 1;
  pl.per_split = (pl.k_tiles + splits - 1) / splits;
  pl.splits = (pl.k_tiles + pl.per_split - 1) / pl.per_split;
  return pl;
}

// Bytes of the split-K partial-tile exchange for `splits` splits.
size_t split_ws_bytes(const Plan& pl, int splits) {
  return splits > 1 ? static_cast<size_t>(pl.n_tiles) * pl.m_tiles * splits * pl.nsub * pl.bm * 128 * 4 : 0;
}

template <typename T, bool kInt8, int NSUB, int BM>
int launch_cfg(const CUtensorMap& wm, const CUtensorMap& xm, TcParams p, Plan pl, const OutMaps& om, cudaStream_t s,
               void* ws, size_t ws_bytes) {
  using C = Cfg<kInt8, NSUB, BM>;
  auto kern = linear_tc_kernel<T, kInt8, NSUB, BM>;
  static bool attr_set = false;  // one attribute call per instantiation
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes) != cudaSuccess) {
      ps_host::set_error("linear_tc: cannot reserve %d bytes of shared memory", C::kBytes);
      return PS_ERR_CUDA;
    }
    attr_set = true;
  }
  int splits = pl.splits;
  // split-K: all clusters must be resident at once: a cluster needs `splits`
  // SMs of one GPC, so large clusters can leave a second wave (queried once
  // per cluster size from the occupancy calculator).
  static int max_clusters[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
  const int tiles = pl.n_tiles * pl.m_tiles;
  while (splits > 1) {
    if (max_clusters[splits] == 0) {
      cudaLaunchConfig_t qc = {};
      qc.gridDim = dim3(1, 1, splits);
      qc.blockDim = dim3(kThreads);
      qc.dynamicSmemBytes = C::kBytes;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = 1;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = splits;
      qc.attrs = qa;
      qc.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &qc) != cudaSuccess || n < 1) {
        (void)cudaGetLastError();
        n = -1;
      }
      max_clusters[splits] = n;
    }
    if (max_clusters[splits] >= tiles) break;
    --splits;
  }
  // the partial tiles go through the caller's workspace when it is large
  // enough; otherwise through shared memory, where the fp32 stage plus S-1
  // received row slices must fit the rings
  p.ws = nullptr;
  if (splits > 1 && ws && ws_bytes >= split_ws_bytes(pl, splits) && ps_host::aligned(ws, 16)) {
    p.ws = static_cast<float*>(ws);
  } else {
    while (splits > 1 && static_cast<long long>(BM) * 512 + static_cast<long long>(splits - 1) *
                                                               ((BM + splits - 1) / splits) * 512 > C::kRings)
      --splits;
  }
  if (splits != pl.splits) {
    pl.per_split = (pl.k_tiles + splits - 1) / splits;
    pl.splits = (pl.k_tiles + pl.per_split - 1) / pl.per_split;
    p.k_tiles_per_split = pl.per_split;
    p.splits = pl.splits;
  }
  p.tma_out = (pl.splits == 1 && (p.N % 8) == 0) ? 1 : 0;  // SwiGLU implies N % 16 == 0
#ifdef PS_TRACE
  fprintf(stderr, "[linear_tc] M=%d N=%d K=%d nsub=%d bm=%d splits=%d tiles=%d max_clusters(splits)=%d\n", p.M, p.N,
          p.K, NSUB, BM, pl.splits, tiles, pl.splits > 1 ? max_clusters[pl.splits] : 0);
#endif
  // The split-K CTAs of one output tile form a (1, 1, splits) cluster and
  // reduce their partial tiles through distributed shared memory.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.n_tiles, pl.m_tiles, pl.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (ps_host::pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (pl.splits > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = pl.splits;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, wm, xm, p, om);
  if (e != cudaSuccess) {
    ps_host::set_error("linear_tc: launch failed: %s", cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  ps_host::count_launch();
  return ps_host::check_launch("linear_tc");
}

template <typename T, bool kInt8, int NSUB>
int launch_nsub(const CUtensorMap& wm, const CUtensorMap& xm, const TcParams& p, const Plan& pl, const OutMaps& om,
                cudaStream_t s, void* ws, size_t wsb) {
  switch (pl.bm) {
    case 32: return launch_cfg<T, kInt8, NSUB, 32>(wm, xm, p, pl, om, s, ws, wsb);
    case 64: return launch_cfg<T, kInt8, NSUB, 64>(wm, xm, p, pl, om, s, ws, wsb);
    case 128: return launch_cfg<T, kInt8, NSUB, 128>(wm, xm, p, pl, om, s, ws, wsb);
    case 192: return launch_cfg<T, kInt8, NSUB, 192>(wm, xm, p, pl, om, s, ws, wsb);
    default:
      // int8 with 256-row slabs caps the token tile at 192 (TMEM holds the
      // accumulators and two widened A stages); the planner never asks more.
      if constexpr (kInt8 && NSUB == 2) return launch_cfg<T, kInt8, NSUB, 192>(wm, xm, p, pl, om, s, ws, wsb);
      else return launch_cfg<T, kInt8, NSUB, 256>(wm, xm, p, pl, om, s, ws, wsb);
  }
}

template <typename T, bool kInt8>
int launch_t(const CUtensorMap& wm, const CUtensorMap& xm, const TcParams& p, const Plan& pl, const OutMaps& om,
             cudaStream_t s, void* ws, size_t wsb) {
  return pl.nsub == 2 ? launch_nsub<T, kInt8, 2>(wm, xm, p, pl, om, s, ws, wsb)
                      : launch_nsub<T, kInt8, 1>(wm, xm, p, pl, om, s, ws, wsb);
}

}  // namespace

#ifdef PS_TRACE
extern "C" PS_API int ps_debug_tc_trace(unsigned long long* host, int n) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, g_tc_trace, sizeof(unsigned long long) * n));
}
#endif

namespace ps_host {

// Split-K partial-tile exchange (an upper bound: the launch may use fewer
// splits). Without it the splits reduce through shared memory, slower.
size_t linear_tc_workspace(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  size_t b = 0;
  for (bool int8 : {true, false}) {
    const Plan pl = plan(M, N, K, int8);
    const size_t v = split_ws_bytes(pl, pl.splits);
    if (v > b) b = v;
  }
  return b;
}

size_t tiled_int8_bytes(int N, int K) {
  return static_cast<size_t>((N + 127) / 128) * ((K + kBK - 1) / kBK) * 8192;
}

int tile_int8(int8_t* dst, const int8_t* src, int N, int K, cudaStream_t s) {
  const int kt = (K + kBK - 1) / kBK;
  const long long units = static_cast<long long>((N + 127) / 128) * kt * 512;
  long long blocks = (units + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  tile_int8_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(dst, src, N, K, kt);
  count_launch();
  return check_launch("tile_int8_weight");
}

int linear_tc(void* y, const void* x, const void* w, int wdtype, const float* scale, const void* bias,
              const void* resid, int M, int N, int K, int dtype, void* workspace, size_t workspace_bytes,
              cudaStream_t s, const int8_t* w_tiled, const ps::PushTargets* push, bool swiglu) {
  if (dtype != PS_BF16 && dtype != PS_F16) return PS_ERR_UNSUPPORTED;
  // SwiGLU epilogue: TMA-stored [M][N/2] output, no residual, no push, no split
  if (swiglu && (resid || push || N % 16 != 0)) return PS_ERR_UNSUPPORTED;
  const bool int8 = wdtype == PS_I8;
  if (!int8 && wdtype != dtype) return PS_ERR_UNSUPPORTED;
  // TMA: global row strides must be multiples of 16 bytes; the epilogue's
  // vector loads of scale/bias/residual need 16-byte alignment.
  if (K % 16 != 0 || !aligned(x, 16) || !aligned(w, 16) || !aligned(y, 16) || !aligned(resid, 16) ||
      !aligned(bias, 16) || !aligned(scale, 16) || !aligned(w_tiled, 16))
    return PS_ERR_UNSUPPORTED;
  Plan pl = plan(M, N, K, int8);
  if (swiglu && pl.splits > 1) {  // the SwiGLU pairs are finished in the (unsplit) TMA epilogue
    pl.splits = 1;
    pl.per_split = pl.k_tiles;
  }
  TcParams p{};
  p.wt = int8 ? w_tiled : nullptr;
  p.n_blocks = (N + 127) / 128;
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
  p.swiglu = swiglu ? 1 : 0;
  p.stagger = stagger_enabled() ? 1 : 0;
  if (push) {
    // the push path stores whole 16-byte groups of outputs, residual-free
    if (resid || bias || N % 8 != 0) return PS_ERR_UNSUPPORTED;
    p.push = *push;
  }
  const CUtensorMapDataType xdt =
      dtype == PS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int bn = 128 * pl.nsub;
  CUtensorMap wm, xm;
  bool ok = make_map(&xm, x, xdt, 2, M, K, kBK, pl.bm, CU_TENSOR_MAP_SWIZZLE_128B);
  if (int8 && w_tiled) wm = xm;  // unused: the weight arrives by contiguous bulk copies
  else if (int8) ok = ok && make_map(&wm, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K, kBK, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
  else ok = ok && make_map(&wm, w, xdt, 2, N, K, kBK, bn, CU_TENSOR_MAP_SWIZZLE_128B);
  // Output maps (box 128 columns x BM tokens). Built whenever N % 8 == 0;
  // the kernel uses them only when the tile is not split.
  OutMaps om;
  std::memset(&om, 0, sizeof(om));
  if (ok && N % 8 == 0) {
    if (swiglu) {
      ok = ok && make_map(&om.y, y, xdt, 2, M, N / 2, 64, pl.bm, CU_TENSOR_MAP_SWIZZLE_NONE);
    } else if (push) {
      const int cols = push->slice ? push->slice : N;  // two-shot slots hold one column slice
      for (int d = 0; d < push->world; ++d)
        ok = ok && make_map(&om.dst[d], push->dst[d], xdt, 2, push->max_tokens, cols, 128, pl.bm,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
      ok = ok && make_map(&om.y, y, xdt, 2, M, N, 128, pl.bm, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    if (resid) ok = ok && make_map(&om.res, resid, xdt, 2, M, N, 128, pl.bm, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (!ok) {
    set_error("linear: cuTensorMapEncodeTiled failed (M=%d N=%d K=%d)", M, N, K);
    return PS_ERR_CUDA;
  }
  void* ws = workspace;
  const size_t wsb = workspace_bytes;
  if (dtype == PS_BF16)
    return int8 ? launch_t<__nv_bfloat16, true>(wm, xm, p, pl, om, s, ws, wsb)
                : launch_t<__nv_bfloat16, false>(wm, xm, p, pl, om, s, ws, wsb);
  return int8 ? launch_t<__half, true>(wm, xm, p, pl, om, s, ws, wsb) : launch_t<__half, false>(wm, xm, p, pl, om, s, ws, wsb);
}

}  // namespace ps_host
