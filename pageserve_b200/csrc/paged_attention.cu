// Paged decode / chunked-prefill attention over the block-scattered KV cache
// (engine/paged_attention.py:16-50, 82-99, 117-132 of the reference, with the
// gather of :82-99 fused away: blocks are read in place through the table).
//
// Work decomposition (one CTA = 4 warps):
//   * A CTA owns one (sequence, kv head) pair. Query rows are the pairs
//     (chunk token t, q head g of the GQA group) -> row t*G + g, so the whole
//     group shares one K/V stream from HBM.
//   * K/V tiles of 64 tokens for that kv head are staged in shared memory by
//     16-byte cp.async (zero-filled past the end), double buffered, XOR
//     swizzled so ldmatrix is conflict free.
//   * Scores and P.V run on tensor cores (mma.sync m16n8k16, bf16/f16 in,
//     fp32 accumulate); online softmax in the log2 domain with quad shuffles.
//   * DECODE (T*G <= 16 rows): the 4 warps split each tile's keys, merge
//     through shared memory, and the context is split across CTAs
//     (split-K); a combine kernel merges the splits' (o, lse) partials.
//   * PREFILL (T*G > 16 rows): each warp owns 16 rows; all warps share the
//     key tiles; the causal bound stops each CTA at its last row's position.
// The kernel is HBM bound: it reads each cached K/V row of the context once.
#include <cudaTypedefs.h>

#include <cfloat>
#include <cstdlib>
#include <climits>
#include <mutex>

#include "common.cuh"

namespace {

using namespace ps;

constexpr int kThreads = 128;
constexpr int kWarps = 4;
constexpr int kKT = 64;       // keys per shared-memory tile
constexpr int kStages = 3;
constexpr float kLog2e = 1.4426950408889634f;

struct AttnParams {
  void* out;
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const int32_t* tables;
  const int32_t* cu_q;
  const int32_t* start_pos;
  float* o_part;   // [B][splits][rows_max][D]
  float* lse_part; // [B][splits][rows_max]
  int* status;
  int max_blocks;
  int num_blocks;
  int block_size;
  int Hq;
  int Hkv;
  int G;
  int rows_max;     // max_q_len * Hq (partial row stride)
  int max_q_len;    // host bounds the grid and workspace were sized for
  int max_ctx;
  int num_splits;
  int split_tokens;
  float scale_log2;
  int num_seqs;
  int balanced;     // decode TMA kernel: 1-D grid of equal key chunks (chunk size chosen on the device)
  int* chunk_dev;   // balanced: the chunk size the attention kernel chose (read by the combine)
};

// Balanced decode split (device side): the smallest chunk size st (a
// multiple of 64, >= kMinChunk) for which the (sequence, kv head, chunk)
// items, Hkv * sum_b ceil(ctx_b / st), fit the grid (binary search over the
// true context lengths, kept in registers for up to 256 sequences); items
// are numbered sequence-major. Warp 0 finds item k's (b, h, c); b = -1 when
// k is past the last item.
constexpr int kMinChunk = 256;

PS_DEVICE int seq_ctx(const AttnParams& p, int b) {
  const int T_b = p.cu_q[b + 1] - p.cu_q[b];
  if (T_b <= 0) return 0;
  const int c = p.start_pos[b] + T_b;
  return c < 0 ? 0 : (c > p.max_ctx ? p.max_ctx : c);
}

PS_DEVICE void balanced_item(const AttnParams& p, int k, int lane, int* b_out, int* h_out, int* c_out,
                             int* st_out) {
  const int cap = (p.max_ctx + 63) / 64 * 64;
  long long st = cap;
  if (p.num_seqs <= 256) {
    int cr[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) cr[j] = lane + 32 * j < p.num_seqs ? seq_ctx(p, lane + 32 * j) : 0;
    int lo = kMinChunk / 64, hi = cap / 64;
    while (lo < hi) {
      const int mid = (lo + hi) / 2;
      const int cs = mid * 64;
      int n = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) n += (cr[j] + cs - 1) / cs;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
      if (static_cast<long long>(n) * p.Hkv <= gridDim.x) hi = mid;
      else lo = mid + 1;
    }
    st = static_cast<long long>(lo) * 64;
  }
  if (st > cap) st = cap;
  int found_b = -1, found_local = 0;
  long long running = 0;
  for (int base = 0; base < p.num_seqs; base += 32) {
    const int i = base + lane;
    const int ctx = i < p.num_seqs ? seq_ctx(p, i) : 0;
    const int n = p.Hkv * static_cast<int>((ctx + st - 1) / st);
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const long long lo = running + incl - n;
    const bool mine = n > 0 && k >= lo && k < running + incl;
    const unsigned hit = __ballot_sync(0xffffffffu, mine);
    if (hit) {
      const int src = __ffs(hit) - 1;
      found_b = __shfl_sync(0xffffffffu, i, src);
      found_local = __shfl_sync(0xffffffffu, static_cast<int>(k - lo), src);
      break;
    }
    running += __shfl_sync(0xffffffffu, incl, 31);
  }
  *b_out = found_b;
  *h_out = found_local % p.Hkv;
  *c_out = found_local / p.Hkv;
  *st_out = static_cast<int>(st);
}

template <int D>
struct Tile {
  static constexpr int kRowBytes = D * 2;
  static constexpr int kBytes = kKT * kRowBytes;  // one of K or V
};

PS_DEVICE uint32_t swz(int row, int chunk, int row_bytes) {
  return static_cast<uint32_t>(row * row_bytes + ((chunk ^ (row & 7)) << 4));
}

// Stage keys [t0, t0+64) of kv head h into K/V tile buffers.
template <typename T, int D>
PS_DEVICE void load_tile(const AttnParams& p, const int32_t* table, int h, int t0, int kv_end, uint32_t k_smem,
                         uint32_t v_smem) {
  constexpr int CPR = D / 8;            // 16-byte chunks per row
  constexpr int PER = kKT * CPR / kThreads;
  const T* kc = static_cast<const T*>(p.k_cache);
  const T* vc = static_cast<const T*>(p.v_cache);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int id = threadIdx.x + i * kThreads;
    const int r = id / CPR;
    const int c = id % CPR;
    const int tok = t0 + r;
    int bytes = 0;
    long long off = 0;
    if (tok < kv_end) {
      const int phys = table[tok / p.block_size];
      if (phys >= 0 && phys < p.num_blocks) {
        off = ((static_cast<long long>(phys) * p.block_size + tok % p.block_size) * p.Hkv + h) * D + c * 8;
        bytes = 16;
      } else {
        record_error(p.status, kErrBlockId);
      }
    }
    const uint32_t so = swz(r, c, D * 2);
    cp_async16(k_smem + so, kc + off, bytes);
    cp_async16(v_smem + so, vc + off, bytes);
  }
}

// Online-softmax state of one warp: 16 rows (this thread holds rows
// lane/4 and lane/4+8), D columns of O.
template <int D>
struct WarpState {
  float o[D / 8][4];
  float m[2];
  float l[2];
};

PS_DEVICE void fence_proxy_async_a() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory addressing of a K/V tile: row = key within the tile,
// chunk = 16-byte column chunk (8 elements).
template <int D>
struct CpAsyncLayout {  // [key][D] rows, chunk ^ (row & 7) swizzle (cp.async staging)
  static PS_DEVICE uint32_t addr(int row, int chunk) { return swz(row, chunk, D * 2); }
};
// D = 128 tiles of 16-key blocks, each block one 4 KB TMA box [16 keys][2 halves][64]
// (128B swizzle: the 16-byte chunk index is XORed with the 128-byte line index mod 8).
struct TmaLayout {
  static PS_DEVICE uint32_t addr(int row, int chunk) {
    const int line = (row & 15) * 2 + (chunk >> 3);
    return static_cast<uint32_t>((row >> 4) * 4096 + line * 128 + (((chunk & 7) ^ (line & 7)) << 4));
  }
};

// Process one 16-key slab at tile row `kr0` (key positions kp0..kp0+15).
// row_limit[i] = last key position row i may attend (causal), or -1.
template <typename T, int D, typename Layout = CpAsyncLayout<D>>
PS_DEVICE void process_slab(WarpState<D>& st, const uint32_t (*qa)[4], uint32_t k_smem, uint32_t v_smem, int kr0,
                            int kp0, const int row_limit[2], float scale_log2) {
  const int lane = threadIdx.x & 31;
  float s[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[n][e] = 0.f;
  // S = Q K^T over D.
  {
    const int mat = lane >> 3;
    const int krow = kr0 + ((mat >> 1) << 3) + (lane & 7);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t b[4];
      ldmatrix_x4(k_smem + Layout::addr(krow, 2 * ks + (mat & 1)), b[0], b[1], b[2], b[3]);
      mma_16816<T>(s[0], qa[ks], b);
      mma_16816<T>(s[1], qa[ks], b + 2);
    }
  }
  // scale, mask, running max
  float mt[2] = {-FLT_MAX, -FLT_MAX};
  bool any[2] = {false, false};
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int ri = e >> 1;
      const int kp = kp0 + n * 8 + 2 * (lane & 3) + (e & 1);
      if (kp <= row_limit[ri]) {
        s[n][e] *= scale_log2;
        mt[ri] = fmaxf(mt[ri], s[n][e]);
        any[ri] = true;
      } else {
        s[n][e] = -INFINITY;
      }
    }
  float corr[2];
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    mt[ri] = fmaxf(mt[ri], __shfl_xor_sync(0xffffffffu, mt[ri], 1));
    mt[ri] = fmaxf(mt[ri], __shfl_xor_sync(0xffffffffu, mt[ri], 2));
    const float mn = fmaxf(st.m[ri], mt[ri]);
    // m starts at -FLT_MAX (finite) so exp2 of a difference is never NaN;
    // a fully masked slab leaves the state unchanged (corr = 1).
    corr[ri] = exp2f(st.m[ri] - mn);
    st.m[ri] = mn;
    (void)any;
  }
  float ps[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int ri = e >> 1;
      ps[n][e] = exp2f(s[n][e] - st.m[ri]);  // exp2(-inf) = 0 for masked keys
    }
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    st.l[ri] = st.l[ri] * corr[ri] + ps[0][2 * ri] + ps[0][2 * ri + 1] + ps[1][2 * ri] + ps[1][2 * ri + 1];
  }
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) {
    st.o[dt][0] *= corr[0];
    st.o[dt][1] *= corr[0];
    st.o[dt][2] *= corr[1];
    st.o[dt][3] *= corr[1];
  }
  uint32_t pa[4];
  pa[0] = pack2<T>(ps[0][0], ps[0][1]);
  pa[1] = pack2<T>(ps[0][2], ps[0][3]);
  pa[2] = pack2<T>(ps[1][0], ps[1][1]);
  pa[3] = pack2<T>(ps[1][2], ps[1][3]);
  // O += P V
  {
    const int mat = lane >> 3;
    const int vrow = kr0 + ((mat & 1) << 3) + (lane & 7);
#pragma unroll
    for (int dp = 0; dp < D / 16; ++dp) {
      uint32_t b[4];
      ldmatrix_x4_trans(v_smem + Layout::addr(vrow, 2 * dp + (mat >> 1)), b[0], b[1], b[2], b[3]);
      mma_16816<T>(st.o[2 * dp], pa, b);
      mma_16816<T>(st.o[2 * dp + 1], pa, b + 2);
    }
  }
}

// Prefill step: 16 query rows against the whole 64-key tile at once (one
// online-softmax update and one rescale of O per 64 keys instead of four).
// masked = false when every key of the tile is visible to every valid row.
template <typename T, int D, typename Layout = CpAsyncLayout<D>>
PS_DEVICE void process_tile64(WarpState<D>& st, const uint32_t (*qa)[4], uint32_t k_smem, uint32_t v_smem, int kp0,
                              const int row_limit[2], float scale_log2, bool masked) {
  const int lane = threadIdx.x & 31;
  const int mat = lane >> 3;
  float s[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[n][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      const int krow = np * 16 + ((mat >> 1) << 3) + (lane & 7);
      ldmatrix_x4(k_smem + Layout::addr(krow, 2 * ks + (mat & 1)), b[0], b[1], b[2], b[3]);
      mma_16816<T>(s[2 * np], qa[ks], b);
      mma_16816<T>(s[2 * np + 1], qa[ks], b + 2);
    }
  }
  float mt[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int ri = e >> 1;
      const int kp = kp0 + n * 8 + 2 * (lane & 3) + (e & 1);
      if (!masked || kp <= row_limit[ri]) {
        s[n][e] *= scale_log2;
        mt[ri] = fmaxf(mt[ri], s[n][e]);
      } else {
        s[n][e] = -INFINITY;
      }
    }
  float corr[2];
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    mt[ri] = fmaxf(mt[ri], __shfl_xor_sync(0xffffffffu, mt[ri], 1));
    mt[ri] = fmaxf(mt[ri], __shfl_xor_sync(0xffffffffu, mt[ri], 2));
    const float mn = fmaxf(st.m[ri], mt[ri]);
    corr[ri] = exp2f(st.m[ri] - mn);
    st.m[ri] = mn;
  }
  float rs[2] = {0.f, 0.f};
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      s[n][e] = exp2f(s[n][e] - st.m[e >> 1]);
      rs[e >> 1] += s[n][e];
    }
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) st.l[ri] = st.l[ri] * corr[ri] + rs[ri];
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) {
    st.o[dt][0] *= corr[0];
    st.o[dt][1] *= corr[0];
    st.o[dt][2] *= corr[1];
    st.o[dt][3] *= corr[1];
  }
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t pa[4];
    pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
    pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
    pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
    pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
    const int vrow = kk * 16 + ((mat & 1) << 3) + (lane & 7);
#pragma unroll
    for (int dp = 0; dp < D / 16; ++dp) {
      uint32_t b[4];
      ldmatrix_x4_trans(v_smem + Layout::addr(vrow, 2 * dp + (mat >> 1)), b[0], b[1], b[2], b[3]);
      mma_16816<T>(st.o[2 * dp], pa, b);
      mma_16816<T>(st.o[2 * dp + 1], pa, b + 2);
    }
  }
}

// Query A-fragments for 16 rows starting at row r0 of this (seq, kv head).
template <typename T, int D>
PS_DEVICE void load_q(uint32_t (*qa)[4], const AttnParams& p, int q0, int h, int r0, int R) {
  const int lane = threadIdx.x & 31;
  const T* q = static_cast<const T*>(p.q);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = r0 + (lane >> 2) + half * 8;
    const bool ok = r < R;
    const int t = ok ? r / p.G : 0;
    const int g = ok ? r % p.G : 0;
    const uint32_t* src =
        reinterpret_cast<const uint32_t*>(q + (static_cast<long long>(q0 + t) * p.Hq + h * p.G + g) * D);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int d = ks * 16 + 2 * (lane & 3);
      qa[ks][half] = ok ? src[d / 2] : 0u;
      qa[ks][half + 2] = ok ? src[d / 2 + 4] : 0u;
    }
  }
}

template <typename T, int D, bool DECODE>
__global__ void __launch_bounds__(kThreads) paged_attention_kernel(const AttnParams p) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) unsigned char smem[];
  const int b = blockIdx.z;
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = p.cu_q[b];
  const int T_b = p.cu_q[b + 1] - q0;
  const int sp = p.start_pos[b];
  const int ctx = sp + T_b;
  const int R = T_b * p.G;
  const int32_t* table = p.tables + static_cast<long long>(b) * p.max_blocks;
  if (T_b <= 0) return;
  if (T_b > p.max_q_len || ctx > p.max_ctx || sp < 0 || ctx > p.max_blocks * p.block_size) {
    if (threadIdx.x == 0) record_error(p.status, kErrShape);
    return;
  }

  int kv_begin, kv_end, row0;
  if (DECODE) {
    kv_begin = blockIdx.x * p.split_tokens;
    if (kv_begin >= ctx) return;
    kv_end = min(ctx, kv_begin + p.split_tokens);
    row0 = 0;
    if (R > 16) {
      if (threadIdx.x == 0) record_error(p.status, kErrShape);
      return;
    }
  } else {
    // blockIdx.x = (row tile, key split); the last rows (longest causal key
    // ranges) come first so the tail of the grid is short.
    const int ntile = (gridDim.x + p.num_splits - 1) / p.num_splits;
    const int rt = ntile - 1 - static_cast<int>(blockIdx.x) / p.num_splits;
    const int split = static_cast<int>(blockIdx.x) % p.num_splits;
    row0 = rt * 64;
    if (row0 >= R) return;
    const int last_row = min(R, row0 + 64) - 1;
    kv_begin = split * p.split_tokens;
    kv_end = min(min(ctx, sp + last_row / p.G + 1), kv_begin + p.split_tokens);
    if (kv_begin >= kv_end) return;
  }
  const int warp_row0 = DECODE ? row0 : row0 + warp * 16;

  uint32_t qa[D / 16][4];
  load_q<T, D>(qa, p, q0, h, warp_row0, R);
  int row_limit[2];
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int r = warp_row0 + (lane >> 2) + hf * 8;
    row_limit[hf] = r < R ? min(sp + r / p.G, kv_end - 1) : -1;
  }

  WarpState<D> st;
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
    for (int e = 0; e < 4; ++e) st.o[dt][e] = 0.f;
  st.m[0] = st.m[1] = -FLT_MAX;
  st.l[0] = st.l[1] = 0.f;

  const uint32_t base = smem_u32(smem);
  const uint32_t stage_bytes = 2 * Tile<D>::kBytes;
  const int ntiles = (kv_end - kv_begin + kKT - 1) / kKT;
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < ntiles) load_tile<T, D>(p, table, h, kv_begin + s * kKT, kv_end, base + s * stage_bytes,
                                    base + s * stage_bytes + Tile<D>::kBytes);
    cp_async_commit();
  }
  const int warp_max_row_limit = max(row_limit[0], row_limit[1]);
  for (int j = 0; j < ntiles; ++j) {
    cp_async_wait<kStages - 2>();
    __syncthreads();
    {
      const int jn = j + kStages - 1;
      const uint32_t so = base + (jn % kStages) * stage_bytes;
      if (jn < ntiles) load_tile<T, D>(p, table, h, kv_begin + jn * kKT, kv_end, so, so + Tile<D>::kBytes);
      cp_async_commit();
    }
    const uint32_t ks = base + (j % kStages) * stage_bytes;
    const uint32_t vs = ks + Tile<D>::kBytes;
    const int t0 = kv_begin + j * kKT;
    if (DECODE) {
      const int kp0 = t0 + warp * 16;
      // quad-uniform skip is not warp-uniform; only skip when the whole warp is past its limit
      const int lim = __reduce_max_sync(0xffffffffu, warp_max_row_limit);
      if (kp0 <= lim) process_slab<T, D>(st, qa, ks, vs, warp * 16, kp0, row_limit, p.scale_log2);
    } else {
      const int lim = __reduce_max_sync(0xffffffffu, warp_max_row_limit);
      // every valid row sees the whole tile: no per-key masking needed
      const int vis = __reduce_min_sync(0xffffffffu, min(row_limit[0] < 0 ? INT_MAX : row_limit[0],
                                                         row_limit[1] < 0 ? INT_MAX : row_limit[1]));
      if (t0 <= lim) process_tile64<T, D>(st, qa, ks, vs, t0, row_limit, p.scale_log2, t0 + kKT - 1 > vis);
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // quad-reduce the row sums
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    st.l[ri] += __shfl_xor_sync(0xffffffffu, st.l[ri], 1);
    st.l[ri] += __shfl_xor_sync(0xffffffffu, st.l[ri], 2);
  }

  if (!DECODE) {
    T* out = static_cast<T*>(p.out);
    const int split = static_cast<int>(blockIdx.x) % p.num_splits;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = warp_row0 + (lane >> 2) + hf * 8;
      if (r >= R) continue;
      const float inv = st.l[hf] > 0.f ? 1.f / st.l[hf] : 0.f;
      const int t = r / p.G, g = r % p.G;
      if (p.num_splits == 1) {
        T* dst = out + (static_cast<long long>(q0 + t) * p.Hq + h * p.G + g) * D;
#pragma unroll
        for (int dt = 0; dt < D / 8; ++dt) {
          const int d = dt * 8 + 2 * (lane & 3);
          *reinterpret_cast<uint32_t*>(dst + d) = pack2<T>(st.o[dt][2 * hf] * inv, st.o[dt][2 * hf + 1] * inv);
        }
      } else {
        const long long prow = (static_cast<long long>(b) * p.num_splits + split) * p.rows_max + t * p.Hq + h * p.G + g;
        float* dst = p.o_part + prow * D;
#pragma unroll
        for (int dt = 0; dt < D / 8; ++dt) {
          const int d = dt * 8 + 2 * (lane & 3);
          *reinterpret_cast<float2*>(dst + d) = make_float2(st.o[dt][2 * hf] * inv, st.o[dt][2 * hf + 1] * inv);
        }
        if ((lane & 3) == 0) p.lse_part[prow] = st.l[hf] > 0.f ? st.m[hf] + log2f(st.l[hf]) : -FLT_MAX;
      }
    }
    return;
  }

  // DECODE: merge the 4 warps' partial states through shared memory.
  float* sm_o = reinterpret_cast<float*>(smem);            // [4][16][D]
  float* sm_m = sm_o + kWarps * 16 * D;                     // [4][16]
  float* sm_l = sm_m + kWarps * 16;                         // [4][16]
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int r = (lane >> 2) + hf * 8;
    float* orow = sm_o + (warp * 16 + r) * D;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      const int d = dt * 8 + 2 * (lane & 3);
      *reinterpret_cast<float2*>(orow + d) = make_float2(st.o[dt][2 * hf], st.o[dt][2 * hf + 1]);
    }
    if ((lane & 3) == 0) {
      sm_m[warp * 16 + r] = st.m[hf];
      sm_l[warp * 16 + r] = st.l[hf];
    }
  }
  __syncthreads();
  // 128 threads: row = tid / 8, 8 threads per row, D/8 dims each.
  {
    const int r = threadIdx.x >> 3;
    const int part = threadIdx.x & 7;
    if (r < R) {
      float mx = -FLT_MAX;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, sm_m[w * 16 + r]);
      float wgt[kWarps];
      float l = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        wgt[w] = exp2f(sm_m[w * 16 + r] - mx);
        l += sm_l[w * 16 + r] * wgt[w];
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      constexpr int DP = D / 8;
      float acc[DP];
#pragma unroll
      for (int i = 0; i < DP; ++i) acc[i] = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float* orow = sm_o + (w * 16 + r) * D + part * DP;
#pragma unroll
        for (int i = 0; i < DP; ++i) acc[i] += orow[i] * wgt[w];
      }
      const int t = r / p.G, g = r % p.G;
      if (p.num_splits == 1) {
        T* dst = static_cast<T*>(p.out) + (static_cast<long long>(q0 + t) * p.Hq + h * p.G + g) * D + part * DP;
#pragma unroll
        for (int i = 0; i < DP; i += 2) *reinterpret_cast<uint32_t*>(dst + i) = pack2<T>(acc[i] * inv, acc[i + 1] * inv);
      } else {
        const long long prow =
            (static_cast<long long>(b) * p.num_splits + blockIdx.x) * p.rows_max + t * p.Hq + h * p.G + g;
        float* dst = p.o_part + prow * D + part * DP;
#pragma unroll
        for (int i = 0; i < DP; i += 4)
          *reinterpret_cast<float4*>(dst + i) =
              make_float4(acc[i] * inv, acc[i + 1] * inv, acc[i + 2] * inv, acc[i + 3] * inv);
        if (part == 0) p.lse_part[prow] = l > 0.f ? mx + log2f(l) : -FLT_MAX;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA-fed decode kernel for the serving shape (head_dim 128, block size 16).
// CTA = (context split, kv head, sequence), 5 warps: warp 0 produces, warps
// 1..4 consume. The producer looks up each 16-key block of a 64-key tile in
// the block table and issues one 4-D TMA load per block for K and one for V
// (box: 64 dims x 2 halves x 1 head x 16 keys = 4 KB, 128B swizzle) into a
// 3-stage mbarrier ring; consumer warp w owns block w-1 of every tile (one
// 16-key mma.sync slab). A thread issues TMA loads at a bounded rate whatever
// their size, so whole-block boxes (rather than one per D half) keep the
// producer ahead of the HBM stream; the ring holds ~2 tiles per CTA (2 CTAs
// per SM) in flight.
constexpr int kTmaStages = 3;
constexpr int kTmaTile = 64;
constexpr int kTmaStageBytes = 2 * kTmaTile * 128 * 2;  // K + V, 32 KB
constexpr long long kAttnWaitCycles = 2000000000LL;

PS_DEVICE void mbar_init_a(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
PS_DEVICE void mbar_expect_tx_a(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
PS_DEVICE void mbar_arrive_a(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
PS_DEVICE bool mbar_try_wait_a(uint32_t bar, uint32_t parity) {
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
// Bounded warp-uniform wait (about a second): false on timeout or abort.
PS_DEVICE bool warp_wait_a(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  bool ok = true;
  const long long t0 = clock64();
  while (!mbar_try_wait_a(bar, parity)) {
    if (*abort_flag) {
      ok = false;
      break;
    }
    if (clock64() - t0 > kAttnWaitCycles) {
      *abort_flag = 1;
      record_error(status, kErrTimeout);
      ok = false;
      break;
    }
  }
  return __all_sync(0xffffffffu, ok);
}
PS_DEVICE void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
PS_DEVICE void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

template <typename T>
__global__ void __launch_bounds__(160) decode_tma_kernel(const __grid_constant__ CUtensorMap kmap,
                                                         const __grid_constant__ CUtensorMap vmap,
                                                         const AttnParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int D = 128;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + kTmaStages * kTmaStageBytes;
  auto full = [&](int s) { return bars + 8 * s; };
  auto empty = [&](int s) { return bars + 8 * (kTmaStages + s); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + kTmaStages * kTmaStageBytes + 8 * 2 * kTmaStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // which (sequence, kv head, key chunk) this CTA runs
  __shared__ int s_item[4];
  if (p.balanced) {
    if (warp == 0) {
      int ib, ih, ic, ist;
      balanced_item(p, blockIdx.x, lane, &ib, &ih, &ic, &ist);
      if (lane == 0) {
        s_item[0] = ib;
        s_item[1] = ih;
        s_item[2] = ic;
        s_item[3] = ist;
        if (blockIdx.x == 0) *p.chunk_dev = ist;
      }
    }
  } else if (threadIdx.x == 0) {
    s_item[0] = blockIdx.z;
    s_item[1] = blockIdx.y;
    s_item[2] = blockIdx.x;
    s_item[3] = p.split_tokens;
  }
  __syncthreads();
  const int b = s_item[0];
  const int h = s_item[1];
  const int chunk = s_item[2];
  const int chunk_keys = s_item[3];
  if (b < 0) return;  // past the last item
  const int q0 = p.cu_q[b];
  const int T_b = p.cu_q[b + 1] - q0;
  const int sp = p.start_pos[b];
  const int ctx = sp + T_b;
  const int R = T_b * p.G;
  const int32_t* table = p.tables + static_cast<long long>(b) * p.max_blocks;
  if (T_b <= 0) return;
  if (T_b > p.max_q_len || ctx > p.max_ctx || sp < 0 || ctx > p.max_blocks * p.block_size || R > 16 ||
      chunk >= p.num_splits) {
    if (threadIdx.x == 0) record_error(p.status, kErrShape);
    return;
  }
  const int kv_begin = chunk * chunk_keys;
  if (kv_begin >= ctx) return;
  const int kv_end = min(ctx, kv_begin + chunk_keys);
  const int ntiles = (kv_end - kv_begin + kTmaTile - 1) / kTmaTile;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kTmaStages; ++s) {
      mbar_init_a(full(s), 1);
      mbar_init_a(empty(s), 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  WarpState<D> st;
  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    // The block-table entries of this split are fetched 32 at a time, one per
    // lane, ahead of the TMA issue (a dependent table load per block would
    // serialise the ring behind global-memory latency).
    const int blk_last = (kv_end - 1) / 16;
    int tab = 0, tab_base = INT_MIN;
    for (int i = 0; i < ntiles; ++i) {
      const int s = i % kTmaStages;
      if (i >= kTmaStages && !warp_wait_a(empty(s), ((i / kTmaStages) - 1) & 1, abort_flag, p.status)) break;
      const int t0 = kv_begin + i * kTmaTile;
      const int blk0 = t0 / 16;
      if (blk0 + 3 > tab_base + 31) {
        tab_base = blk0;
        tab = blk0 + lane <= blk_last ? table[blk0 + lane] : 0;
      }
      int physj[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) physj[j] = __shfl_sync(0xffffffffu, tab, blk0 - tab_base + j);
      if (lane == 0) {
        const int nblk = min(4, (kv_end - t0 + 15) / 16);
        mbar_expect_tx_a(full(s), nblk * 4 * 2048);
        const uint32_t kst = base + s * kTmaStageBytes;
        const uint32_t vst = kst + kTmaStageBytes / 2;
        for (int j = 0; j < nblk; ++j) {
          int phys = physj[j];
          if (phys < 0 || phys >= p.num_blocks) {
            record_error(p.status, kErrBlockId);
            phys = 0;  // keep the transaction count; the output is flagged invalid
          }
          const int row = phys * 16;
          // one 4 KB box per block and tensor (both D halves of kv head h)
          tma_load_4d(kst + j * 4096, &kmap, full(s), 0, 0, h, row);
          tma_load_4d(vst + j * 4096, &vmap, full(s), 0, 0, h, row);
        }
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ consumers --
    const int cw = warp - 1;  // which 16-key block of each tile
    uint32_t qa[D / 16][4];
    load_q<T, D>(qa, p, q0, h, 0, R);
    int row_limit[2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = (lane >> 2) + hf * 8;
      row_limit[hf] = r < R ? min(sp + r / p.G, kv_end - 1) : -1;
    }
    const int lim = __reduce_max_sync(0xffffffffu, max(row_limit[0], row_limit[1]));
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
      for (int e = 0; e < 4; ++e) st.o[dt][e] = 0.f;
    st.m[0] = st.m[1] = -FLT_MAX;
    st.l[0] = st.l[1] = 0.f;
    for (int i = 0; i < ntiles; ++i) {
      const int s = i % kTmaStages;
      if (!warp_wait_a(full(s), (i / kTmaStages) & 1, abort_flag, p.status)) break;
      const uint32_t kst = base + s * kTmaStageBytes;
      const uint32_t vst = kst + kTmaStageBytes / 2;
      const int kp0 = kv_begin + i * kTmaTile + cw * 16;
      if (kp0 < kv_end && kp0 <= lim) {
        const int valid = kv_end - kp0;
        if (valid < 16) {
          // zero the V rows past the context so 0-probability keys add 0
          unsigned char* vb = gbase + (vst - base) + cw * 4096;
          for (int u = lane; u < (16 - valid) * 16; u += 32) {
            const int row = valid + u / 16, part = u % 16;
            *reinterpret_cast<uint4*>(vb + row * 256 + part * 16) = make_uint4(0, 0, 0, 0);  // whole rows
          }
          __syncwarp();
        }
        process_slab<T, D, TmaLayout>(st, qa, kst, vst, cw * 16, kp0, row_limit, p.scale_log2);
        if (valid < 16) fence_proxy_async_a();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_a(empty(s));
    }
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      st.l[ri] += __shfl_xor_sync(0xffffffffu, st.l[ri], 1);
      st.l[ri] += __shfl_xor_sync(0xffffffffu, st.l[ri], 2);
    }
  }
  __syncthreads();  // every TMA consumed: the stage memory is free for the merge

  // Merge the 4 consumer warps' states (same as the cp.async decode kernel).
  float* sm_o = reinterpret_cast<float*>(gbase);  // [4][16][D]
  float* sm_m = sm_o + 4 * 16 * D;
  float* sm_l = sm_m + 4 * 16;
  if (warp > 0) {
    const int cw = warp - 1;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = (lane >> 2) + hf * 8;
      float* orow = sm_o + (cw * 16 + r) * D;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        const int d = dt * 8 + 2 * (lane & 3);
        *reinterpret_cast<float2*>(orow + d) = make_float2(st.o[dt][2 * hf], st.o[dt][2 * hf + 1]);
      }
      if ((lane & 3) == 0) {
        sm_m[cw * 16 + r] = st.m[hf];
        sm_l[cw * 16 + r] = st.l[hf];
      }
    }
  }
  __syncthreads();
  if (warp > 0) {
    const int ct = threadIdx.x - 32;
    const int r = ct >> 3;
    const int part = ct & 7;
    if (r < R) {
      float mx = -FLT_MAX;
#pragma unroll
      for (int w = 0; w < 4; ++w) mx = fmaxf(mx, sm_m[w * 16 + r]);
      float wgt[4];
      float l = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        wgt[w] = exp2f(sm_m[w * 16 + r] - mx);
        l += sm_l[w * 16 + r] * wgt[w];
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      constexpr int DP = D / 8;
      float acc[DP];
#pragma unroll
      for (int i2 = 0; i2 < DP; ++i2) acc[i2] = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float* orow = sm_o + (w * 16 + r) * D + part * DP;
#pragma unroll
        for (int i2 = 0; i2 < DP; ++i2) acc[i2] += orow[i2] * wgt[w];
      }
      const int t = r / p.G, g = r % p.G;
      if (p.num_splits == 1) {
        T* dst = static_cast<T*>(p.out) + (static_cast<long long>(q0 + t) * p.Hq + h * p.G + g) * D + part * DP;
#pragma unroll
        for (int i2 = 0; i2 < DP; i2 += 2)
          *reinterpret_cast<uint32_t*>(dst + i2) = pack2<T>(acc[i2] * inv, acc[i2 + 1] * inv);
      } else {
        const long long prow =
            (static_cast<long long>(b) * p.num_splits + chunk) * p.rows_max + t * p.Hq + h * p.G + g;
        float* dst = p.o_part + prow * D + part * DP;
#pragma unroll
        for (int i2 = 0; i2 < DP; i2 += 4)
          *reinterpret_cast<float4*>(dst + i2) =
              make_float4(acc[i2] * inv, acc[i2 + 1] * inv, acc[i2 + 2] * inv, acc[i2 + 3] * inv);
        if (part == 0) p.lse_part[prow] = l > 0.f ? mx + log2f(l) : -FLT_MAX;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Prefill / chunked-prefill attention on tcgen05 (D = 128, block 16).
// One CTA = one kv head x 128 query rows (128/G tokens x the G heads of the
// group, row r = token*G + g) x all of their causal key range, in 128-key
// tiles. Roles (192 threads):
//   warp 0    TMA producer: the Q tile once (3-D box 64 x G x 128/G per D
//             half), then per key tile 8 blocks x 2 halves of K and of V
//             (3-D boxes 64 x 1 x 16 from the paged cache, 128B swizzle)
//             into a 2-stage ring; block-table entries prefetched per lane
//   warp 1    TMEM allocator + MMA issuer: S_j = Q K_j^T into one of two
//             TMEM S buffers (M=128, N=128, K=16 x 8, both operands K-major
//             in shared memory), then O += P_{j-1} V_{j-1} (A = P from TMEM,
//             B = V read MN-major from its [key][D] tile)
//   warps 2-5 softmax, one query row per thread (TMEM lane quarter w%4):
//             S from TMEM, causal mask, online max/sum in the log2 domain,
//             O rescaled in TMEM when the max moves, P written to TMEM as
//             bf16/f16 (the PV MMA's A operand); at the end O / l to global
// TMEM: S0 | S1 | O (128 columns each) | P (64 columns). Every wait is
// bounded (kErrTimeout, then the roles drain and TMEM is freed).
constexpr int kPtKeys = 128;                      // keys per tile
constexpr int kPtQBytes = 128 * 128 * 2;          // Q tile: 2 halves x 16 KB
constexpr int kPtKVBytes = kPtKeys * 128 * 2;     // K (or V) tile: 2 halves x 16 KB
constexpr int kPtStages = 2;
constexpr int kPtThreads = 192;

PS_DEVICE void tc_fence_before_a() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PS_DEVICE void tc_fence_after_a() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
PS_DEVICE uint64_t desc_sw128_a(uint32_t addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;  // 8-row group stride
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;           // 128B swizzle
  return d;
}
// kind::f16 instruction descriptor, f32 accumulate; b_mn: B is MN-major.
__host__ __device__ constexpr uint32_t idesc_a(bool bf16, int m, int n, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}
PS_DEVICE void mma_ss_a(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
PS_DEVICE void mma_ts_a(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
PS_DEVICE void mma_commit_a(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
PS_DEVICE void tmem_ld32_a(uint32_t addr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
PS_DEVICE void tmem_st16_a(uint32_t addr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          addr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
PS_DEVICE void tmem_st32f_a(uint32_t addr, const float* f) {
  uint32_t v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(f[i]);
  tmem_st16_a(addr, v);
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(f[16 + i]);
  tmem_st16_a(addr + 16, v);
}
PS_DEVICE void tmem_wait_st_a() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 2^x by the MUFU approximation (relative error ~2^-22; 2^-inf = 0): the
// probabilities are rounded to 16 bits right after.
PS_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__global__ void __launch_bounds__(kPtThreads, 1) prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                   const __grid_constant__ CUtensorMap kmap,
                                                                   const __grid_constant__ CUtensorMap vmap,
                                                                   const AttnParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  const uint32_t q_sa = base;
  auto k_sa = [&](int s) { return base + kPtQBytes + s * 2 * kPtKVBytes; };
  auto v_sa = [&](int s) { return k_sa(s) + kPtKVBytes; };
  const uint32_t bars = base + kPtQBytes + kPtStages * 2 * kPtKVBytes;
  auto kv_full = [&](int s) { return bars + 8 * s; };
  auto kv_empty = [&](int s) { return bars + 8 * (2 + s); };
  auto s_full = [&](int b) { return bars + 8 * (4 + b); };
  auto s_free = [&](int b) { return bars + 8 * (6 + b); };
  const uint32_t q_full = bars + 8 * 8;
  const uint32_t p_full = bars + 8 * 9;
  const uint32_t pv_done = bars + 8 * 10;
  unsigned char* misc = gbase + kPtQBytes + kPtStages * 2 * kPtKVBytes + 8 * 12;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y;
  const int q0 = p.cu_q[b];
  const int T_b = p.cu_q[b + 1] - q0;
  const int sp = p.start_pos[b];
  const int ctx = sp + T_b;
  const int G = p.G;
  const int TQ = 128 / G;  // tokens per tile
  const int ntile_rows = (T_b + TQ - 1) / TQ;
  const int rt = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);  // longest key ranges first
  if (T_b <= 0 || rt >= ntile_rows) return;
  if (T_b > p.max_q_len || ctx > p.max_ctx || sp < 0 || ctx > p.max_blocks * p.block_size) {
    if (threadIdx.x == 0) record_error(p.status, kErrShape);
    return;
  }
  const int tq0 = rt * TQ;
  const int kv_end = min(ctx, sp + min(T_b, tq0 + TQ));  // keys the tile's last row sees
  const int ntiles = (kv_end + kPtKeys - 1) / kPtKeys;
  const int32_t* table = p.tables + static_cast<long long>(b) * p.max_blocks;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kPtStages; ++s) {
      mbar_init_a(kv_full(s), 1);
      mbar_init_a(kv_empty(s), 1);
    }
    for (int bb = 0; bb < 2; ++bb) {
      mbar_init_a(s_full(bb), 1);
      mbar_init_a(s_free(bb), 4);
    }
    mbar_init_a(q_full, 1);
    mbar_init_a(p_full, 4);
    mbar_init_a(pv_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before_a();
  __syncthreads();
  tc_fence_after_a();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s0 = tmem, t_o = tmem + 256, t_p = tmem + 384;

  if (warp == 0) {
    // ---------------------------------------------------------- producer --
    if (lane == 0) {
      mbar_expect_tx_a(q_full, kPtQBytes);
      for (int half = 0; half < 2; ++half)
        tma_load_3d(q_sa + half * (kPtQBytes / 2), &qmap, q_full, half * 64, h * G, q0 + tq0);
    }
    __syncwarp();
    const int last_blk = (kv_end - 1) / 16;  // later tile blocks reload it (finite data, masked keys)
    for (int j = 0; j < ntiles; ++j) {
      const int s = j % kPtStages;
      if (j >= kPtStages && !warp_wait_a(kv_empty(s), ((j / kPtStages) - 1) & 1, abort_flag, p.status)) break;
      int blk = j * 8 + (lane & 7);
      if (blk > last_blk) blk = last_blk;
      int phys = table[blk];
      if (phys < 0 || phys >= p.num_blocks) {
        record_error(p.status, kErrBlockId);
        phys = 0;
      }
      int physj[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) physj[i] = __shfl_sync(0xffffffffu, phys, i);
      if (lane == 0) {
        mbar_expect_tx_a(kv_full(s), 2 * kPtKVBytes);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int row = physj[i] * 16;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            tma_load_3d(k_sa(s) + half * (kPtKVBytes / 2) + i * 2048, &kmap, kv_full(s), half * 64, h, row);
            tma_load_3d(v_sa(s) + half * (kPtKVBytes / 2) + i * 2048, &vmap, kv_full(s), half * 64, h, row);
          }
        }
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA --
    constexpr uint32_t id_qk = idesc_a(kBf16, 128, 128, false);
    constexpr uint32_t id_pv = idesc_a(kBf16, 128, 128, true);
    bool ok = warp_wait_a(q_full, 0, abort_flag, p.status);
    for (int j = 0; ok && j <= ntiles; ++j) {
      if (j < ntiles) {
        const int s = j % kPtStages, sb = j & 1;
        ok = warp_wait_a(kv_full(s), (j / kPtStages) & 1, abort_flag, p.status);
        if (ok && j >= 2) ok = warp_wait_a(s_free(sb), ((j >> 1) - 1) & 1, abort_flag, p.status);
        if (!ok) break;
        tc_fence_after_a();
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {  // D = 128 in 8 steps of 16 (64 per 128B-swizzled half)
            const uint32_t off = (kk >> 2) * (kPtQBytes / 2) + (kk & 3) * 32;
            mma_ss_a(t_s0 + sb * 128, desc_sw128_a(q_sa + off, 0), desc_sw128_a(k_sa(s) + off, 0), id_qk,
                     kk > 0 ? 1u : 0u);
          }
          mma_commit_a(s_full(sb));
        }
        __syncwarp();
      }
      if (j >= 1) {
        // O += P_{j-1} V_{j-1}: V tile [key][D] read MN-major (D halves 16 KB apart)
        const int s = (j - 1) % kPtStages;
        ok = warp_wait_a(p_full, (j - 1) & 1, abort_flag, p.status);
        if (!ok) break;
        tc_fence_after_a();
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // 128 keys in 8 steps of 16
            mma_ts_a(t_o, t_p + kk * 8, desc_sw128_a(v_sa(s) + kk * 16 * 128, kPtKVBytes / 2), id_pv,
                     (j > 1 || kk > 0) ? 1u : 0u);
          mma_commit_a(kv_empty(s));
          mma_commit_a(pv_done);
        }
        __syncwarp();
      }
    }
  } else {
    // ----------------------------------------------------------- softmax --
    // One pass over S per tile (128 scores in registers). The running max
    // used for P and O ("m_ref") only moves when a row's max grows by more
    // than 8 (log2 domain), so O is rescaled in TMEM rarely; P <= 2^8 stays
    // well inside the 16-bit range and l uses the same reference.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // this thread's query row (TMEM lane)
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int tok = tq0 + r / G;
    const int g = r % G;
    const int qpos = sp + tok;           // causal limit: keys <= qpos
    const bool row_ok = tok < T_b;
    float m_ref = -FLT_MAX, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      ok = warp_wait_a(s_full(sb), (j >> 1) & 1, abort_flag, p.status);
      if (!ok) break;
      tc_fence_after_a();
      const int key0 = j * kPtKeys;
      float sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32_a(t_s0 + sb * 128 + c * 32 + lane_off, sv + 32 * c);
      // keys past a row's causal limit or the context get -inf (whole-warp fast path when none does)
      const bool full = __all_sync(0xffffffffu, key0 + kPtKeys - 1 <= qpos && key0 + kPtKeys <= kv_end);
      float mx = -FLT_MAX;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        float x = sv[i] * p.scale_log2;
        if (!full && (key0 + i > qpos || key0 + i >= kv_end)) x = -INFINITY;  // 2^(-inf - m) = 0 for any m
        sv[i] = x;
        mx = fmaxf(mx, x);
      }
      float alpha = 1.f;
      bool moved = false;
      if (mx > m_ref + 8.f) {
        const float m_new = mx;
        alpha = (m_ref == -FLT_MAX) ? 0.f : ex2_approx(m_ref - m_new);
        m_ref = m_new;
        moved = true;
      }
      // O must hold P_{j-1} V_{j-1} before it is rescaled and P overwritten
      if (j >= 1) {
        ok = warp_wait_a(pv_done, (j - 1) & 1, abort_flag, p.status);
        if (!ok) break;
        tc_fence_after_a();
        if (__any_sync(0xffffffffu, moved)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_ld32_a(t_o + c * 32 + lane_off, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= alpha;
            tmem_st32f_a(t_o + c * 32 + lane_off, v);
          }
        }
      }
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = ex2_approx(sv[32 * c + i] - m_ref);      // -inf -> 0
          const float p1 = ex2_approx(sv[32 * c + i + 1] - m_ref);
          sum += p0 + p1;
          pk[i / 2] = pack2<T>(p0, p1);
        }
        tmem_st16_a(t_p + c * 16 + lane_off, pk);
      }
      tmem_wait_st_a();
      tc_fence_before_a();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_a(s_free(sb));
        mbar_arrive_a(p_full);
      }
      l = l * alpha + sum;
    }
    // epilogue: O / l
    if (ok) ok = warp_wait_a(pv_done, (ntiles - 1) & 1, abort_flag, p.status);
    if (ok) {
      tc_fence_after_a();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* dst = static_cast<T*>(p.out) + (static_cast<long long>(q0 + tok) * p.Hq + h * G + g) * 128;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32_a(t_o + c * 32 + lane_off, v);
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = v[i + e] * inv;
            *reinterpret_cast<uint4*>(dst + c * 32 + i) = pack8<T>(o);
          }
        }
      }
    }
  }
  tc_fence_before_a();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_a();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// Merge split partials: one warp per (sequence, chunk token, q head) row.
template <typename T, int D>
__global__ void combine_kernel(const AttnParams p) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.y;
  const int q0 = p.cu_q[b];
  const int T_b = p.cu_q[b + 1] - q0;
  const int ctx = p.start_pos[b] + T_b;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (T_b > p.max_q_len || ctx > p.max_ctx) return;  // the attention kernel recorded the error
  if (row >= T_b * p.Hq) return;
  // splits that saw this row's keys: positions 0 .. start_pos + t (causal)
  const int last_key = p.start_pos[b] + row / p.Hq;
  const int st = p.balanced ? *p.chunk_dev : p.split_tokens;
  const int nsplit = min(p.num_splits, last_key / st + 1);
  (void)ctx;
  const long long base = static_cast<long long>(b) * p.num_splits * p.rows_max + row;
  float mx = -FLT_MAX;
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, p.lse_part[base + static_cast<long long>(s) * p.rows_max]);
  constexpr int DPL = D / 32;
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
  float wsum = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const long long pr = base + static_cast<long long>(s) * p.rows_max;
    const float w = exp2f(p.lse_part[pr] - mx);
    wsum += w;
    const float* o = p.o_part + pr * D + lane * DPL;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] += w * o[i];
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  const int t = row / p.Hq, hq = row % p.Hq;
  T* dst = static_cast<T*>(p.out) + (static_cast<long long>(q0 + t) * p.Hq + hq) * D + lane * DPL;
#pragma unroll
  for (int i = 0; i < DPL; i += 2) *reinterpret_cast<uint32_t*>(dst + i) = pack2<T>(acc[i] * inv, acc[i + 1] * inv);
}

// Split heuristic shared by the workspace query and the launch: split the
// context when (sequences x kv heads) CTAs cannot fill the 148 SMs a few
// times over.
void plan_splits(int num_seqs, int max_q_len, int max_ctx, int Hq, int Hkv, int D, int* num_splits,
                 int* split_tokens, size_t max_ws = ~static_cast<size_t>(0)) {
  const int G = Hq / Hkv;
  *num_splits = 1;
  *split_tokens = max_ctx > 0 ? max_ctx : 1;
  if (max_q_len * G > 16) {
    // Prefill tiles (64 query rows) over the causal key range: split the key
    // range into 128-key pieces when the tiles alone give under ~3 CTAs per
    // SM (one warp per SM sub-partition leaves every mma.sync stall exposed),
    // as long as the (o, lse) partials fit the workspace cap.
    const long long base = static_cast<long long>((max_q_len * G + 63) / 64) * Hkv * num_seqs;
    long long target = 3LL * 148;
    if (const char* env = std::getenv("PS_ATTN_PREFILL_CTAS")) target = std::atoll(env) > 0 ? std::atoll(env) : target;  // tuning
    int splits = static_cast<int>((target + base - 1) / base);
    const int max_by_len = (max_ctx + 127) / 128;
    if (splits > max_by_len) splits = max_by_len;
    while (splits > 1 &&
           static_cast<size_t>(num_seqs) * splits * max_q_len * Hq * (D + 1) * sizeof(float) + 256 > max_ws)
      --splits;
    if (splits <= 1) return;
    int st = (max_ctx + splits - 1) / splits;
    st = (st + kKT - 1) / kKT * kKT;
    *split_tokens = st;
    *num_splits = (max_ctx + st - 1) / st;
    return;
  }
  if (D == 128) {
    // the TMA decode kernel picks its chunk (>= kMinChunk keys) on the device
    // from the actual context lengths; size partials for the smallest chunk
    const int chunks = (max_ctx + kMinChunk - 1) / kMinChunk;
    if (chunks > 1) {
      *num_splits = chunks;
      *split_tokens = kMinChunk;
    }
    return;
  }
  const long long ctas = static_cast<long long>(num_seqs) * Hkv;
  // head_dim 128 runs the TMA kernel (2 CTAs per SM with a deep ring): about
  // 1.5 waves of long splits; the cp.async kernel wants many short ones.
  long long target = D == 128 ? 148LL * 2 * 3 / 2 : 148LL * 3 * 4;
  if (const char* env = std::getenv("PS_ATTN_DECODE_CTAS")) target = std::atoll(env) > 0 ? std::atoll(env) : target;  // tuning
  int splits = static_cast<int>((target + ctas - 1) / ctas);
  const int max_by_len = (max_ctx + 255) / 256;  // at least 256 keys per split
  if (splits > max_by_len) splits = max_by_len;
  if (splits < 1) splits = 1;
  int st = (max_ctx + splits - 1) / splits;
  st = (st + kKT - 1) / kKT * kKT;
  *split_tokens = st;
  *num_splits = (max_ctx + st - 1) / st;
}

size_t workspace_bytes_for(int num_seqs, int max_q_len, int max_ctx, int Hq, int Hkv, int D) {
  int ns, st;
  plan_splits(num_seqs, max_q_len, max_ctx, Hq, Hkv, D, &ns, &st);
  if (ns <= 1) return 0;
  const size_t rows = static_cast<size_t>(num_seqs) * ns * max_q_len * Hq;
  return rows * D * sizeof(float) + rows * sizeof(float) + 256 + 16;
}

PFN_cuTensorMapEncodeTiled_v12000 attn_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// One layer's cache as a 3-D tensor [num_blocks*16 keys][Hkv][128] with a
// 64 x 1 x 16 box (one half of one head's 16-key block), 128B swizzle.
// The KV cache as a 4-D tensor {64 dims, 2 halves, Hkv, NB*16 rows}: one box
// {64, 2, 1, 16} = 4 KB loads a whole 16-key block of one kv head (both D
// halves, 128B swizzle per 128-byte line) in a single TMA.
bool make_kv_map4(CUtensorMap* map, const void* cache, bool bf16, int num_blocks, int Hkv) {
  auto fn = attn_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {64, 2, static_cast<cuuint64_t>(Hkv), static_cast<cuuint64_t>(num_blocks) * 16};
  cuuint64_t strides[3] = {64 * 2, 128 * 2, static_cast<cuuint64_t>(Hkv) * 128 * 2};
  cuuint32_t box[4] = {64, 2, 1, 16};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
            const_cast<void*>(cache), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_kv_map(CUtensorMap* map, const void* cache, bool bf16, int num_blocks, int Hkv) {
  auto fn = attn_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(Hkv), static_cast<cuuint64_t>(num_blocks) * 16};
  cuuint64_t strides[2] = {128 * 2, static_cast<cuuint64_t>(Hkv) * 128 * 2};
  cuuint32_t box[3] = {64, 1, 16};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
            const_cast<void*>(cache), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
int launch_decode_tma(AttnParams& p, int num_seqs, int max_q_len, cudaStream_t s) {
  CUtensorMap km, vm;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  if (!make_kv_map4(&km, p.k_cache, bf16, p.num_blocks, p.Hkv) ||
      !make_kv_map4(&vm, p.v_cache, bf16, p.num_blocks, p.Hkv)) {
    ps_host::set_error("paged_attention: cuTensorMapEncodeTiled failed for the KV cache");
    return PS_ERR_CUDA;
  }
  const int smem = kTmaStages * kTmaStageBytes + 1024 + 256;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(decode_tma_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      ps_host::set_error("paged_attention: cannot reserve %d bytes of shared memory", smem);
      return PS_ERR_CUDA;
    }
    attr = true;
  }
  // With a split: a 1-D grid of two CTAs per SM (at least one per sequence x
  // kv head) over equal key chunks, so the KV stream is spread evenly
  // whatever the mix of context lengths.
  p.balanced = p.num_splits > 1 ? 1 : 0;
  const long long pairs = static_cast<long long>(num_seqs) * p.Hkv;
  long long slots = 2 * 148;
  if (const char* env = std::getenv("PS_ATTN_DECODE_GRID")) slots = std::atoll(env) > 0 ? std::atoll(env) : slots;  // tuning
  dim3 grid = p.balanced ? dim3(static_cast<unsigned>(pairs > slots ? pairs : slots))
                         : dim3(p.num_splits, p.Hkv, num_seqs);
  ps_host::launch(decode_tma_kernel<T>, grid, 160, smem, s, km, vm, p);
  ps_host::count_launch();
  int rc = ps_host::check_launch("paged_attention(decode, tma)");
  if (rc != PS_OK || p.num_splits == 1) return rc;
  const int rows = max_q_len * p.Hq;
  dim3 cgrid((rows + 3) / 4, num_seqs);
  ps_host::launch(combine_kernel<T, 128>, cgrid, 128, 0, s, p);
  ps_host::count_launch();
  return ps_host::check_launch("paged_attention(combine)");
}

// The q tensor [total_q][Hq][128] as a 3-D TMA tensor, box 64 x G x 128/G
// (one 128-row query tile per D half), 128B swizzle.
bool make_q_map(CUtensorMap* map, const void* q, bool bf16, int total_q, int Hq, int G) {
  auto fn = attn_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(Hq), static_cast<cuuint64_t>(total_q)};
  cuuint64_t strides[2] = {128 * 2, static_cast<cuuint64_t>(Hq) * 128 * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(G), static_cast<cuuint32_t>(128 / G)};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(q),
            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool prefill_tc_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("PS_ATTN_PREFILL_TC");
    return !(e && e[0] == '0');
  }();
  return v;
}

template <typename T>
int launch_prefill_tc(AttnParams& p, int num_seqs, int max_q_len, int total_q, cudaStream_t s) {
  CUtensorMap qm, km, vm;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  if (!make_q_map(&qm, p.q, bf16, total_q, p.Hq, p.G) || !make_kv_map(&km, p.k_cache, bf16, p.num_blocks, p.Hkv) ||
      !make_kv_map(&vm, p.v_cache, bf16, p.num_blocks, p.Hkv)) {
    ps_host::set_error("paged_attention: cuTensorMapEncodeTiled failed (prefill)");
    return PS_ERR_CUDA;
  }
  const int smem = kPtQBytes + kPtStages * 2 * kPtKVBytes + 1024 + 1024;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(prefill_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      ps_host::set_error("paged_attention: cannot reserve %d bytes of shared memory", smem);
      return PS_ERR_CUDA;
    }
    attr = true;
  }
  const int tq = 128 / p.G;
  dim3 grid((max_q_len + tq - 1) / tq, p.Hkv, num_seqs);
  ps_host::launch(prefill_tc_kernel<T>, grid, kPtThreads, smem, s, qm, km, vm, p);
  ps_host::count_launch();
  return ps_host::check_launch("paged_attention(prefill, tcgen05)");
}

template <typename T, int D>
int launch(AttnParams& p, int num_seqs, int max_q_len, int max_ctx, cudaStream_t s, int total_q) {
  const bool decode = max_q_len * p.G <= 16;
  if constexpr (D == 128) {
    // the serving layout: TMA needs 16-key blocks and 16-byte aligned rows
    const bool tma_ok = p.block_size == 16 && static_cast<long long>(p.num_blocks) * 16 < (1LL << 31) &&
                        ps_host::aligned(p.k_cache, 16) && ps_host::aligned(p.v_cache, 16);
    if (decode && tma_ok) return launch_decode_tma<T>(p, num_seqs, max_q_len, s);
    if (!decode && tma_ok && prefill_tc_enabled() && 128 % p.G == 0 && ps_host::aligned(p.q, 16) &&
        ps_host::aligned(p.out, 16))
      return launch_prefill_tc<T>(p, num_seqs, max_q_len, total_q, s);
  }
  const int stage_smem = kStages * 2 * Tile<D>::kBytes;
  const int merge_smem = kWarps * 16 * D * 4 + 2 * kWarps * 16 * 4;
  const int smem = stage_smem > merge_smem ? stage_smem : merge_smem;
  if (decode) {
    auto kern = paged_attention_kernel<T, D, true>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 grid(p.num_splits, p.Hkv, num_seqs);
    ps_host::launch(kern, grid, kThreads, smem, s, p);
    ps_host::count_launch();
    int rc = ps_host::check_launch("paged_attention(decode)");
    if (rc != PS_OK || p.num_splits == 1) return rc;
    const int rows = max_q_len * p.Hq;
    dim3 cgrid((rows + 3) / 4, num_seqs);
    ps_host::launch(combine_kernel<T, D>, cgrid, 128, 0, s, p);
    ps_host::count_launch();
    return ps_host::check_launch("paged_attention(combine)");
  }
  auto kern = paged_attention_kernel<T, D, false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid(((max_q_len * p.G + 63) / 64) * p.num_splits, p.Hkv, num_seqs);
  ps_host::launch(kern, grid, kThreads, smem, s, p);
  ps_host::count_launch();
  int rc = ps_host::check_launch("paged_attention(prefill)");
  if (rc != PS_OK || p.num_splits == 1) return rc;
  const int rows = max_q_len * p.Hq;
  dim3 cgrid((rows + 3) / 4, num_seqs);
  ps_host::launch(combine_kernel<T, D>, cgrid, 128, 0, s, p);
  ps_host::count_launch();
  return ps_host::check_launch("paged_attention(prefill combine)");
}

}  // namespace

extern "C" {

size_t ps_paged_attention_workspace_size(int num_seqs, int max_q_len, int max_ctx, int Hq, int Hkv, int D) {
  if (num_seqs <= 0 || max_q_len <= 0 || Hkv <= 0 || Hq % Hkv != 0) return 0;
  return workspace_bytes_for(num_seqs, max_q_len, max_ctx, Hq, Hkv, D);
}

int ps_paged_attention(void* out, const void* q, const void* k_cache, const void* v_cache, const int32_t* tables,
                       int max_blocks, const int32_t* cu_q, const int32_t* start_pos, int num_seqs, int total_q,
                       int max_q_len, int max_ctx, int num_blocks, int block_size, int Hq, int Hkv, int D,
                       int dtype, void* workspace, size_t workspace_bytes, ps_stream_t stream) {
  if (num_seqs <= 0 || total_q < 0 || max_q_len <= 0 || max_ctx < max_q_len || block_size <= 0 ||
      num_blocks <= 0 || max_blocks <= 0 || Hq <= 0 || Hkv <= 0) {
    ps_host::set_error("paged_attention: invalid sizes (seqs %d, max_q %d, max_ctx %d)", num_seqs, max_q_len,
                       max_ctx);
    return PS_ERR_INVALID;
  }
  if (Hq % Hkv != 0) {
    ps_host::set_error("paged_attention: %d q heads not divisible by %d kv heads", Hq, Hkv);
    return PS_ERR_INVALID;
  }
  if (max_ctx > max_blocks * block_size) {
    ps_host::set_error("paged_attention: context %d needs %d table entries, table has %d", max_ctx,
                       (max_ctx + block_size - 1) / block_size, max_blocks);
    return PS_ERR_INDEX;
  }
  if (!out || !q || !k_cache || !v_cache || !tables || !cu_q || !start_pos) {
    ps_host::set_error("paged_attention: null pointer");
    return PS_ERR_INVALID;
  }
  if (!ps_host::aligned(k_cache, 16) || !ps_host::aligned(v_cache, 16) || !ps_host::aligned(q, 4) ||
      !ps_host::aligned(out, 4) || !ps_host::aligned(workspace, 16)) {
    ps_host::set_error("paged_attention: caches need 16-byte, q/out 4-byte alignment");
    return PS_ERR_INVALID;
  }
  if (total_q == 0) return PS_OK;
  AttnParams p{};
  p.out = out;
  p.q = q;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.tables = tables;
  p.cu_q = cu_q;
  p.start_pos = start_pos;
  p.status = ps_host::status_word(PS_TU_ATTN);
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = Hq / Hkv;
  p.rows_max = max_q_len * Hq;
  p.max_q_len = max_q_len;
  p.max_ctx = max_ctx;
  p.scale_log2 = (1.0f / sqrtf(static_cast<float>(D))) * kLog2e;
  plan_splits(num_seqs, max_q_len, max_ctx, Hq, Hkv, D, &p.num_splits, &p.split_tokens);
  if (p.num_splits > 1) {
    const size_t need = workspace_bytes_for(num_seqs, max_q_len, max_ctx, Hq, Hkv, D);
    if (!workspace || workspace_bytes < need) {
      ps_host::set_error("paged_attention: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
      return PS_ERR_INVALID;
    }
    const size_t rows = static_cast<size_t>(num_seqs) * p.num_splits * p.rows_max;
    uintptr_t w = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~static_cast<uintptr_t>(255);
    p.o_part = reinterpret_cast<float*>(w);
    p.lse_part = p.o_part + rows * D;
    p.chunk_dev = reinterpret_cast<int*>(p.lse_part + rows);
  }
  p.num_seqs = num_seqs;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PS_BF16) {
    if (D == 128) return launch<__nv_bfloat16, 128>(p, num_seqs, max_q_len, max_ctx, s, total_q);
    if (D == 64) return launch<__nv_bfloat16, 64>(p, num_seqs, max_q_len, max_ctx, s, total_q);
  } else if (dtype == PS_F16) {
    if (D == 128) return launch<__half, 128>(p, num_seqs, max_q_len, max_ctx, s, total_q);
    if (D == 64) return launch<__half, 64>(p, num_seqs, max_q_len, max_ctx, s, total_q);
  } else {
    ps_host::set_error("paged_attention: dtype must be bf16 or f16");
    return PS_ERR_UNSUPPORTED;
  }
  ps_host::set_error("paged_attention: head_dim %d unsupported (64, 128)", D);
  return PS_ERR_UNSUPPORTED;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// ps_paged_attention needs a caller-provided workspace for its split-context
// partials and lazily cudaMalloc's a per-device status word. Some callers can
// do neither: a plugin hosted by another serving engine whose device memory
// is owned entirely by that engine's pool allocator, or a latency-critical
// path that may not call cudaMalloc (it can synchronise the device). This
// variant takes the same inputs and outputs but keeps its scratch in the
// file-scope array below, sized PS_ATTN_NOALLOC_SCRATCH_BYTES; every GPU that
// loads this library reserves it until the process exits.
//
// Its first call on a device looks up the array's device address with
// cudaGetSymbolAddress (the host-side name of a __device__ array is not a
// device address) and caches it per device for the life of the process; make
// that first call before any stream capture, and reload the library after a
// cudaDeviceReset, which may move the array. Decode batches whose partials do
// not fit are rejected; prefill batches split into as many key pieces as fit
// (plan_splits' max_ws). All calls
// on a device share the array: calls that overlap on the GPU (different
// streams, or threads racing) corrupt each other's partials. Nothing in the
// array must start at zero: every split writes its partial output and
// log-sum-exp before the combine kernel reads them, so a previous call's
// contents are never read. Device-side range errors (a block id outside the
// pool) skip the access as in ps_paged_attention, and the kernels' bounded
// waits still end, but neither is recorded, since this variant owns no status
// word.
namespace {

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[PS_ATTN_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    ps_host::set_error("paged_attention_noalloc: no current device (%s)", cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      ps_host::set_error("paged_attention_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return PS_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return PS_OK;
}

}  // namespace

extern "C" int ps_paged_attention_noalloc(void* out, const void* q, const void* k_cache, const void* v_cache,
                                          const int32_t* tables, int max_blocks, const int32_t* cu_q,
                                          const int32_t* start_pos, int num_seqs, int total_q, int max_q_len,
                                          int max_ctx, int num_blocks, int block_size, int Hq, int Hkv, int D,
                                          int dtype, ps_stream_t stream) {
  if (num_seqs <= 0 || total_q < 0 || max_q_len <= 0 || max_ctx < max_q_len || block_size <= 0 ||
      num_blocks <= 0 || max_blocks <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0) {
    ps_host::set_error("paged_attention_noalloc: invalid sizes (seqs %d, max_q %d, max_ctx %d)", num_seqs,
                       max_q_len, max_ctx);
    return PS_ERR_INVALID;
  }
  if (max_ctx > max_blocks * block_size) {
    ps_host::set_error("paged_attention_noalloc: context %d needs %d table entries, table has %d", max_ctx,
                       (max_ctx + block_size - 1) / block_size, max_blocks);
    return PS_ERR_INDEX;
  }
  if (!out || !q || !k_cache || !v_cache || !tables || !cu_q || !start_pos) {
    ps_host::set_error("paged_attention_noalloc: null pointer");
    return PS_ERR_INVALID;
  }
  if (!ps_host::aligned(k_cache, 16) || !ps_host::aligned(v_cache, 16) || !ps_host::aligned(q, 4) ||
      !ps_host::aligned(out, 4)) {
    ps_host::set_error("paged_attention_noalloc: caches need 16-byte, q/out 4-byte alignment");
    return PS_ERR_INVALID;
  }
  const bool prefill = max_q_len * (Hq / Hkv) > 16;  // prefill splits shrink to fit the static scratch
  const size_t need = prefill ? 0 : workspace_bytes_for(num_seqs, max_q_len, max_ctx, Hq, Hkv, D);
  if (need > PS_ATTN_NOALLOC_SCRATCH_BYTES) {
    ps_host::set_error(
        "paged_attention_noalloc: this batch needs %zu bytes of split scratch, above the static limit of %zu "
        "bytes (use ps_paged_attention with a workspace)",
        need, static_cast<size_t>(PS_ATTN_NOALLOC_SCRATCH_BYTES));
    return PS_ERR_INVALID;
  }
  if (total_q == 0) return PS_OK;
  AttnParams p{};
  p.out = out;
  p.q = q;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.tables = tables;
  p.cu_q = cu_q;
  p.start_pos = start_pos;
  p.status = nullptr;
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = Hq / Hkv;
  p.rows_max = max_q_len * Hq;
  p.max_q_len = max_q_len;
  p.max_ctx = max_ctx;
  p.scale_log2 = (1.0f / sqrtf(static_cast<float>(D))) * kLog2e;
  plan_splits(num_seqs, max_q_len, max_ctx, Hq, Hkv, D, &p.num_splits, &p.split_tokens,
              PS_ATTN_NOALLOC_SCRATCH_BYTES);
  if (p.num_splits > 1) {
    void* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != PS_OK) return rc;
    const size_t rows = static_cast<size_t>(num_seqs) * p.num_splits * p.rows_max;
    p.o_part = static_cast<float*>(scratch);  // the array is 256-byte aligned
    p.lse_part = p.o_part + rows * D;
    p.chunk_dev = reinterpret_cast<int*>(p.lse_part + rows);
  }
  p.num_seqs = num_seqs;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PS_BF16) {
    if (D == 128) return launch<__nv_bfloat16, 128>(p, num_seqs, max_q_len, max_ctx, s, total_q);
    if (D == 64) return launch<__nv_bfloat16, 64>(p, num_seqs, max_q_len, max_ctx, s, total_q);
  } else if (dtype == PS_F16) {
    if (D == 128) return launch<__half, 128>(p, num_seqs, max_q_len, max_ctx, s, total_q);
    if (D == 64) return launch<__half, 64>(p, num_seqs, max_q_len, max_ctx, s, total_q);
  } else {
    ps_host::set_error("paged_attention_noalloc: dtype must be bf16 or f16");
    return PS_ERR_UNSUPPORTED;
  }
  ps_host::set_error("paged_attention_noalloc: head_dim %d unsupported (64, 128)", D);
  return PS_ERR_UNSUPPORTED;
}
