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
#include <cfloat>
#include <mutex>

#include "common.cuh"

namespace {

using namespace ps;

constexpr int kThreads = 128;
constexpr int kWarps = 4;
constexpr int kKT = 64;       // keys per shared-memory tile
constexpr int kStages = 2;
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
};

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

// Process one 16-key slab at tile row `kr0` (key positions kp0..kp0+15).
// row_limit[i] = last key position row i may attend (causal), or -1.
template <typename T, int D>
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
      ldmatrix_x4(k_smem + swz(krow, 2 * ks + (mat & 1), D * 2), b[0], b[1], b[2], b[3]);
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
      ldmatrix_x4_trans(v_smem + swz(vrow, 2 * dp + (mat >> 1), D * 2), b[0], b[1], b[2], b[3]);
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
    row0 = blockIdx.x * 64;
    if (row0 >= R) return;
    const int last_row = min(R, row0 + 64) - 1;
    kv_begin = 0;
    kv_end = min(ctx, sp + last_row / p.G + 1);
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
#pragma unroll
      for (int sl = 0; sl < kKT / 16; ++sl) {
        const int kp0 = t0 + sl * 16;
        if (kp0 <= lim) process_slab<T, D>(st, qa, ks, vs, sl * 16, kp0, row_limit, p.scale_log2);
      }
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
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = warp_row0 + (lane >> 2) + hf * 8;
      if (r >= R) continue;
      const float inv = st.l[hf] > 0.f ? 1.f / st.l[hf] : 0.f;
      T* dst = out + (static_cast<long long>(q0 + r / p.G) * p.Hq + h * p.G + r % p.G) * D;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        const int d = dt * 8 + 2 * (lane & 3);
        *reinterpret_cast<uint32_t*>(dst + d) = pack2<T>(st.o[dt][2 * hf] * inv, st.o[dt][2 * hf + 1] * inv);
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

// Merge split partials: one warp per (sequence, chunk token, q head) row.
template <typename T, int D>
__global__ void combine_kernel(const AttnParams p) {
  const int b = blockIdx.y;
  const int q0 = p.cu_q[b];
  const int T_b = p.cu_q[b + 1] - q0;
  const int ctx = p.start_pos[b] + T_b;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (T_b > p.max_q_len || ctx > p.max_ctx) return;  // the attention kernel recorded the error
  if (row >= T_b * p.Hq) return;
  const int nsplit = min(p.num_splits, (ctx + p.split_tokens - 1) / p.split_tokens);
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
void plan_splits(int num_seqs, int max_q_len, int max_ctx, int Hq, int Hkv, int* num_splits, int* split_tokens) {
  const int G = Hq / Hkv;
  *num_splits = 1;
  *split_tokens = max_ctx > 0 ? max_ctx : 1;
  if (max_q_len * G > 16) return;  // prefill kernel: no split
  const long long ctas = static_cast<long long>(num_seqs) * Hkv;
  const long long target = 148LL * 3 * 4;
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
  plan_splits(num_seqs, max_q_len, max_ctx, Hq, Hkv, &ns, &st);
  if (ns <= 1) return 0;
  const size_t rows = static_cast<size_t>(num_seqs) * ns * max_q_len * Hq;
  return rows * D * sizeof(float) + rows * sizeof(float) + 256;
}

template <typename T, int D>
int launch(AttnParams& p, int num_seqs, int max_q_len, int max_ctx, cudaStream_t s) {
  const bool decode = max_q_len * p.G <= 16;
  const int stage_smem = kStages * 2 * Tile<D>::kBytes;
  const int merge_smem = kWarps * 16 * D * 4 + 2 * kWarps * 16 * 4;
  const int smem = stage_smem > merge_smem ? stage_smem : merge_smem;
  if (decode) {
    auto kern = paged_attention_kernel<T, D, true>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 grid(p.num_splits, p.Hkv, num_seqs);
    kern<<<grid, kThreads, smem, s>>>(p);
    ps_host::count_launch();
    int rc = ps_host::check_launch("paged_attention(decode)");
    if (rc != PS_OK || p.num_splits == 1) return rc;
    const int rows = max_q_len * p.Hq;
    dim3 cgrid((rows + 3) / 4, num_seqs);
    combine_kernel<T, D><<<cgrid, 128, 0, s>>>(p);
    ps_host::count_launch();
    return ps_host::check_launch("paged_attention(combine)");
  }
  auto kern = paged_attention_kernel<T, D, false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((max_q_len * p.G + 63) / 64, p.Hkv, num_seqs);
  kern<<<grid, kThreads, smem, s>>>(p);
  ps_host::count_launch();
  return ps_host::check_launch("paged_attention(prefill)");
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
  plan_splits(num_seqs, max_q_len, max_ctx, Hq, Hkv, &p.num_splits, &p.split_tokens);
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
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PS_BF16) {
    if (D == 128) return launch<__nv_bfloat16, 128>(p, num_seqs, max_q_len, max_ctx, s);
    if (D == 64) return launch<__nv_bfloat16, 64>(p, num_seqs, max_q_len, max_ctx, s);
  } else if (dtype == PS_F16) {
    if (D == 128) return launch<__half, 128>(p, num_seqs, max_q_len, max_ctx, s);
    if (D == 64) return launch<__half, 64>(p, num_seqs, max_q_len, max_ctx, s);
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
// device address); make that first call before any stream capture. All calls
// on a device share the array: calls that overlap on the GPU (different
// streams, or threads racing) corrupt each other's partials. Nothing in the
// array must start at zero: every split writes its partial output and
// log-sum-exp before the combine kernel reads them, so a previous call's
// contents are never read. Device-side range errors (a block id outside the
// pool) skip the access as in ps_paged_attention but are not recorded, since
// this variant owns no status word.
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
  const size_t need = workspace_bytes_for(num_seqs, max_q_len, max_ctx, Hq, Hkv, D);
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
  plan_splits(num_seqs, max_q_len, max_ctx, Hq, Hkv, &p.num_splits, &p.split_tokens);
  if (p.num_splits > 1) {
    void* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != PS_OK) return rc;
    const size_t rows = static_cast<size_t>(num_seqs) * p.num_splits * p.rows_max;
    p.o_part = static_cast<float*>(scratch);  // the array is 256-byte aligned
    p.lse_part = p.o_part + rows * D;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PS_BF16) {
    if (D == 128) return launch<__nv_bfloat16, 128>(p, num_seqs, max_q_len, max_ctx, s);
    if (D == 64) return launch<__nv_bfloat16, 64>(p, num_seqs, max_q_len, max_ctx, s);
  } else if (dtype == PS_F16) {
    if (D == 128) return launch<__half, 128>(p, num_seqs, max_q_len, max_ctx, s);
    if (D == 64) return launch<__half, 64>(p, num_seqs, max_q_len, max_ctx, s);
  } else {
    ps_host::set_error("paged_attention_noalloc: dtype must be bf16 or f16");
    return PS_ERR_UNSUPPORTED;
  }
  ps_host::set_error("paged_attention_noalloc: head_dim %d unsupported (64, 128)", D);
  return PS_ERR_UNSUPPORTED;
}
