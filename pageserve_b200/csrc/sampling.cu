// On-device token selection after the lm_head: top-k of each logits row and
// sampling from the top-k (the reference picks the next token on the host,
// one sequence at a time: int(logits[-1].argmax()), server.py:47-51 and
// engine/runner.py:79-83; greedy argmax is ps_argmax in norm_misc.cu).
//
// top-k: one CTA per row. A radix select over order-preserving 32-bit keys of
// the float values (4 passes of 8 bits, a 256-bin shared-memory histogram per
// pass, each pass counting only keys that match the digits fixed so far)
// finds the k-th largest key T; the elements above T and the lowest-index
// elements equal to T (ties broken by index, as argmax breaks them) are
// gathered and sorted by (value descending, index ascending) with a bitonic
// sort in shared memory. HBM-bound: 5 reads of the row.
#include "common.cuh"

namespace {

using namespace ps;

constexpr int kTopkThreads = 1024;
constexpr int kTopkMax = 1024;

// Order-preserving map float -> uint32 (larger float, larger key; NaN above +inf).
PS_DEVICE uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
PS_DEVICE float kfloat(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

template <typename T>
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(float* __restrict__ vals, int32_t* __restrict__ idx,
                                                            const T* __restrict__ logits, int V, int ld, int k) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_need;
  __shared__ int s_count;
  __shared__ uint32_t ckey[kTopkMax];
  __shared__ int cidx[kTopkMax];
  __shared__ int wsum[kTopkThreads / 32];
  const T* lr = logits + static_cast<long long>(blockIdx.x) * ld;
  const int tid = threadIdx.x;
  uint32_t prefix = 0, mask = 0;
  int need = k;  // rank of the k-th largest among the keys matching the prefix
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < V; i += kTopkThreads) {
      const uint32_t key = fkey(to_f32(lr[i]));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      int above = 0, d = 255;
      for (; d > 0; --d) {  // the digit whose bucket holds the need-th largest
        if (above + static_cast<int>(hist[d]) >= need) break;
        above += hist[d];
      }
      s_prefix = prefix | (static_cast<uint32_t>(d) << shift);
      s_need = need - above;
    }
    __syncthreads();
    prefix = s_prefix;
    need = s_need;
    mask |= 255u << shift;
  }
  // prefix is the k-th largest key; `need` of the elements equal to it are
  // taken (the lowest indices), all k - need elements above it.
  const uint32_t kth = prefix;
  if (tid == 0) s_count = 0;
  for (int i = tid; i < kTopkMax; i += kTopkThreads) {
    ckey[i] = 0u;
    cidx[i] = 0x7fffffff;
  }
  __syncthreads();
  for (int i = tid; i < V; i += kTopkThreads) {
    const uint32_t key = fkey(to_f32(lr[i]));
    if (key > kth) {
      const int at = atomicAdd(&s_count, 1);
      ckey[at] = key;
      cidx[at] = i;
    }
  }
  __syncthreads();
  const int n_gt = s_count;  // == k - need
  // ties in index order: a block-wide running count over chunks of the row
  int taken = 0;
  const int lane = tid & 31, warp = tid >> 5;
  for (int base = 0; base < V && taken < need; base += kTopkThreads) {
    const int i = base + tid;
    const bool eq = i < V && fkey(to_f32(lr[i])) == kth;
    const unsigned bal = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < kTopkThreads / 32; ++w) {
      before += w < warp ? wsum[w] : 0;
      total += wsum[w];
    }
    const int rank = taken + before + __popc(bal & ((1u << lane) - 1u));
    if (eq && rank < need) {
      ckey[n_gt + rank] = kth;
      cidx[n_gt + rank] = i;
    }
    taken += total;
    __syncthreads();
  }
  __syncthreads();
  // bitonic sort of the padded candidates: value descending, index ascending
  int n2 = 1;
  while (n2 < k) n2 <<= 1;
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n2; i += kTopkThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;  // this pair sorts "first-before-second"
          const bool first_before =
              ckey[i] > ckey[j] || (ckey[i] == ckey[j] && cidx[i] < cidx[j]);
          if (first_before != up) {
            const uint32_t tk = ckey[i];
            ckey[i] = ckey[j];
            ckey[j] = tk;
            const int ti = cidx[i];
            cidx[i] = cidx[j];
            cidx[j] = ti;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int j = tid; j < k; j += kTopkThreads) {
    vals[static_cast<long long>(blockIdx.x) * k + j] = kfloat(ckey[j]);
    idx[static_cast<long long>(blockIdx.x) * k + j] = cidx[j];
  }
}

// One warp per row: p_j = exp((v_j - v_0) / temperature) over the row's sorted
// top-k values, token = idx[first j with cumsum(p) > u * sum(p)] (inverse CDF
// with the row's uniform u in [0, 1)). Sums in index order (deterministic).
__global__ void sample_topk_kernel(int32_t* __restrict__ out, const float* __restrict__ vals,
                                   const int32_t* __restrict__ idx, const float* __restrict__ uniforms, int M, int k,
                                   float inv_temp) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float* v = vals + static_cast<long long>(row) * k;
  const float v0 = v[0];
  float total = 0.f;
  for (int j = 0; j < k; ++j) total += __expf((v[j] - v0) * inv_temp);
  const float target = uniforms[row] * total;
  float acc = 0.f;
  int pick = k - 1;
  for (int j = 0; j < k; ++j) {
    acc += __expf((v[j] - v0) * inv_temp);
    if (acc > target) {
      pick = j;
      break;
    }
  }
  if (lane == 0) out[row] = idx[static_cast<long long>(row) * k + pick];
}

}  // namespace

extern "C" {

int ps_topk(float* vals, int32_t* idx, const void* logits, int M, int V, int ld, int k, int dtype,
            ps_stream_t stream) {
  if (M < 0 || V <= 0 || ld < V || k < 1 || k > kTopkMax || k > V || (M > 0 && (!vals || !idx || !logits))) {
    ps_host::set_error("topk: invalid arguments (M=%d V=%d ld=%d k=%d; 1 <= k <= min(V, %d))", M, V, ld, k,
                       kTopkMax);
    return PS_ERR_INVALID;
  }
  if (M == 0) return PS_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PS_F32: ps_host::launch(topk_kernel<float>, M, kTopkThreads, 0, s, vals, idx, static_cast<const float*>(logits), V, ld, k); break;
    case PS_BF16: ps_host::launch(topk_kernel<__nv_bfloat16>, M, kTopkThreads, 0, s, vals, idx, static_cast<const __nv_bfloat16*>(logits), V, ld, k); break;
    case PS_F16: ps_host::launch(topk_kernel<__half>, M, kTopkThreads, 0, s, vals, idx, static_cast<const __half*>(logits), V, ld, k); break;
    default: ps_host::set_error("topk: unsupported dtype"); return PS_ERR_UNSUPPORTED;
  }
  ps_host::count_launch();
  return ps_host::check_launch("topk");
}

int ps_sample_topk(int32_t* out, const float* vals, const int32_t* idx, const float* uniforms, int M, int k,
                   float temperature, ps_stream_t stream) {
  if (M < 0 || k < 1 || !(temperature > 0.f) || (M > 0 && (!out || !vals || !idx || !uniforms))) {
    ps_host::set_error("sample_topk: invalid arguments (M=%d k=%d temperature=%g)", M, k, temperature);
    return PS_ERR_INVALID;
  }
  if (M == 0) return PS_OK;
  const int rows_per_cta = 4;
  ps_host::launch(sample_topk_kernel, (M + rows_per_cta - 1) / rows_per_cta, 32 * rows_per_cta, 0,
                  reinterpret_cast<cudaStream_t>(stream), out, vals, idx, uniforms, M, k, 1.0f / temperature);
  ps_host::count_launch();
  return ps_host::check_launch("sample_topk");
}

}  // extern "C"
