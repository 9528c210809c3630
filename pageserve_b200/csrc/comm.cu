// Tensor-parallel all-reduce fused around the row-parallel linears
// (engine/tensor_parallel.py:34-48 of the reference: partial = x_shard @ W.T,
// dist.all_reduce(partial, SUM)), over peer memory instead of a collective.
//
// Every rank owns one receive buffer, mapped into its peers through CUDA IPC:
//   [control words][2 sets][W slots][max_tokens][H] bf16/f16
// The row-parallel GEMM's final writer (its epilogue, or its split-K
// reduction) stores each output tile straight into slot[my_rank] of every
// rank's buffer (16-byte stores, to peers over NVLink), so the exchange
// overlaps the GEMM tile by tile (comm.cuh: push_arrive). The consumer — the
// next RMSNorm — waits until its flag shows all W ranks, sums the W slots,
// adds the residual, normalises, and re-arms the set once all its CTAs have
// read the slots.
//
// Why two sets suffice: a rank writes set s again only after its consumer of
// the other set has seen every peer's partial of that set, and each peer
// produced that partial after its own consumer of set s had finished (stream
// order), i.e. after reading and re-arming set s.
//
// Waits give up after a few seconds of clock64 cycles, record kErrTimeout in
// the status word and go on (results are then invalid, the GPU never spins
// unbounded). No multicast: plain loads and stores, peer stores and
// system-scope atomics only.
#include <cstring>

#include "comm.cuh"

namespace {

using namespace ps;

constexpr long long kCommWaitCycles = 6000000000LL;  // ~3 s at 1.97 GHz

PS_DEVICE unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

PS_DEVICE unsigned* ctrl_flag(void* buf, int set) { return reinterpret_cast<unsigned*>(buf) + set; }
PS_DEVICE unsigned* ctrl_consumed(void* buf, int set) { return reinterpret_cast<unsigned*>(buf) + 16 + set; }
// Set by the first wait that times out: later waits on this buffer return at
// once, so a lost peer costs one timeout, not one per layer. Cleared only by
// re-zeroing the buffer.
PS_DEVICE volatile unsigned* ctrl_broken(void* buf) { return reinterpret_cast<volatile unsigned*>(buf) + 48; }

// One CTA per token row. NORM: x += s (in place), y = rmsnorm(x) * w;
// otherwise y = s. s = T(sum over ranks, float32, rank order) — the same on
// every rank, so all ranks keep bit-identical residual streams.
template <typename T, int MAXV, bool NORM>
__global__ void __launch_bounds__(256) allreduce_rmsnorm_kernel(T* __restrict__ y, T* __restrict__ x,
                                                                const T* __restrict__ w, float eps, int M, int H,
                                                                void* buf, int W, int set, long long slot_elems,
                                                                long long slots_off, int* status) {
  pdl_wait();
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T);
  __shared__ float red[8];
  unsigned* flag = ctrl_flag(buf, set);
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    volatile unsigned* broken = ctrl_broken(buf);
    while (ld_acquire_sys(flag) < static_cast<unsigned>(W)) {
      if (*broken) {
        record_error(status, kErrTimeout);
        break;
      }
      if (clock64() - t0 > kCommWaitCycles) {
        *broken = 1u;
        record_error(status, kErrTimeout);
        break;
      }
    }
  }
  __syncthreads();
  const T* slots = reinterpret_cast<const T*>(static_cast<const unsigned char*>(buf) + slots_off) +
                   static_cast<long long>(set) * W * slot_elems;
  const int row = blockIdx.x;
  const long long roff = static_cast<long long>(row) * H;
  const int nvec = H / VEC;
  float v[MAXV][VEC];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int c = threadIdx.x + j * 256;
    if (c < nvec) {
      float acc[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
      for (int r = 0; r < W; ++r) {
        // written by other GPUs during this kernel's wait: L2 loads, no L1
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(slots + r * slot_elems + roff) + c);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] += to_f32(e[i]);
      }
      if constexpr (NORM) {
        uint4 xu = reinterpret_cast<const uint4*>(x + roff)[c];
        T* xe = reinterpret_cast<T*>(&xu);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          xe[i] = from_f32<T>(to_f32(xe[i]) + to_f32(from_f32<T>(acc[i])));
          v[j][i] = to_f32(xe[i]);
          ss += v[j][i] * v[j][i];
        }
        reinterpret_cast<uint4*>(x + roff)[c] = xu;
      } else {
        reinterpret_cast<uint4*>(y + roff)[c] = pack8<T>(acc);
      }
    }
  }
  if constexpr (NORM) {
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
      t = warp_sum(t);
      if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / static_cast<float>(H) + eps);
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int c = threadIdx.x + j * 256;
      if (c < nvec) {
        float wv[VEC], o[VEC];
        unpack8<T>(reinterpret_cast<const uint4*>(w)[c], wv);
#pragma unroll
        for (int i = 0; i < VEC; ++i) o[i] = v[j][i] * inv * wv[i];
        reinterpret_cast<uint4*>(y + roff)[c] = pack8<T>(o);
      }
    }
  }
  // re-arm: the last CTA to finish reading clears the flag and the counter
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* consumed = ctrl_consumed(buf, set);
    __threadfence();
    const unsigned prev = atomicAdd(consumed, 1u);
    if (prev == static_cast<unsigned>(M) - 1) {
      atomicExch(consumed, 0u);
      atomicExch(flag, 0u);
      __threadfence_system();
    }
  }
}

struct RankBufs {
  void* b[kMaxWorld];  // every rank's receive buffer, as mapped in this process
};

PS_DEVICE bool wait_count(const unsigned* p, unsigned target, void* buf, int* status) {
  const long long t0 = clock64();
  volatile unsigned* broken = ctrl_broken(buf);
  while (ld_acquire_sys(p) < target) {
    if (*broken) {
      record_error(status, kErrTimeout);
      return false;
    }
    if (clock64() - t0 > kCommWaitCycles) {
      *broken = 1u;
      record_error(status, kErrTimeout);
      return false;
    }
  }
  return true;
}

// Two-shot consumer: the rest of the all-reduce after a scattering
// row-parallel linear, plus the residual add and RMSNorm (engine/
// tensor_parallel.py:47, engine/model.py:184-190). Rank `rank` owns the
// columns [rank * S, (rank + 1) * S), S = H / W; CTA b owns rows
// [b * R, (b + 1) * R).
// Phase 1: wait until the set's flag shows W scatters; for the CTA's rows and
//   the owned columns, x = T(x_old + T(sum of the W slots, rank order));
//   store x into xg[set] of EVERY rank (the all-gather, 16-byte stores, peers
//   over NVLink), then count the row block on every rank. The last CTA to
//   finish re-arms the set's flag.
// Phase 2: wait until this rank's count of the row block shows W, re-arm it,
//   and normalise whole rows read from xg[set]: y = rmsnorm(x) * w (y = x
//   without a weight).
// `phases` is 3 for real ranks; one process emulating several ranks on one
// GPU runs phase 1 of every rank before phase 2 of any (nothing then waits
// on a later launch). x_old (row stride H) is the residual stream the
// previous reduction gathered (xg of the other set), or the embedding output.
template <typename T>
__global__ void __launch_bounds__(256) tp_reduce_rmsnorm_kernel(T* __restrict__ y, const T* __restrict__ x_old,
                                                                const T* __restrict__ w, float eps, int M, int H,
                                                                RankBufs bufs, int W, int rank, int set,
                                                                int max_tokens, int R, int phases,
                                                                long long xg_off, long long slots_off, int* status) {
  pdl_wait();
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T);
  void* own = bufs.b[rank];
  const int S = H / W;
  const int m0 = blockIdx.x * R;
  const int rows = min(R, M - m0);
  unsigned* gcount = reinterpret_cast<unsigned*>(static_cast<unsigned char*>(own) + kGatherCountOff) +
                     set * kGatherBlocks + blockIdx.x;
  const long long xg_set = static_cast<long long>(set) * max_tokens * H;  // elements
  if (phases & 1) {
    unsigned* flag = ctrl_flag(own, set);
    __shared__ int ok;
    if (threadIdx.x == 0) ok = wait_count(flag, static_cast<unsigned>(W), own, status) ? 1 : 0;
    __syncthreads();
    const T* slots = reinterpret_cast<const T*>(static_cast<const unsigned char*>(own) + slots_off) +
                     static_cast<long long>(set) * W * max_tokens * S;
    const int vpr = S / VEC;  // 16-byte vectors per row of the slice
    for (int i = threadIdx.x; i < rows * vpr && ok; i += blockDim.x) {
      const int m = m0 + i / vpr;
      const int c = (i % vpr) * VEC;  // column within the slice
      float acc[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
      for (int r = 0; r < W; ++r) {  // rank order: the same sum on every run
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(slots + (static_cast<long long>(r) * max_tokens + m) * S + c));
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] += to_f32(e[k]);
      }
      const long long col = static_cast<long long>(rank) * S + c;
      if (x_old) {
        float xo[VEC];
        unpack8<T>(*reinterpret_cast<const uint4*>(x_old + static_cast<long long>(m) * H + col), xo);
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] = xo[k] + to_f32(from_f32<T>(acc[k]));
      }
      const uint4 pk = pack8<T>(acc);
      const long long off = xg_set + static_cast<long long>(m) * H + col;
      for (int r = 0; r < W; ++r) {
        T* xg = reinterpret_cast<T*>(static_cast<unsigned char*>(bufs.b[r]) + xg_off);
        *reinterpret_cast<uint4*>(xg + off) = pk;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();  // this CTA's stores (ordered by the barrier) before the counts
      for (int r = 0; r < W; ++r) {
        unsigned* g = reinterpret_cast<unsigned*>(static_cast<unsigned char*>(bufs.b[r]) + kGatherCountOff) +
                      set * kGatherBlocks + blockIdx.x;
        red_release_sys_add(g, 1u);
      }
      // re-arm the flag once every CTA has seen it
      unsigned* consumed = ctrl_consumed(own, set);
      const unsigned prev = atomicAdd(consumed, 1u);
      if (prev == gridDim.x - 1) {
        atomicExch(consumed, 0u);
        atomicExch(flag, 0u);
        __threadfence_system();
      }
    }
  }
  if (phases & 2) {
    __shared__ int ok2;
    if (threadIdx.x == 0) {
      ok2 = wait_count(gcount, static_cast<unsigned>(W), own, status) ? 1 : 0;
      if (ok2) atomicExch(gcount, 0u);  // only this CTA reads this count; every rank's W adds have landed
    }
    __syncthreads();
    if (!ok2) return;
    const T* xg = reinterpret_cast<const T*>(static_cast<const unsigned char*>(own) + xg_off) + xg_set;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nvec = H / VEC;
    for (int r = warp; r < rows; r += blockDim.x / 32) {
      const long long ro = static_cast<long long>(m0 + r) * H;
      float ss = 0.f;
      for (int c = lane; c < nvec; c += 32) {  // pass 1: sum of squares (written by peers: L2 loads)
        float v[VEC];
        unpack8<T>(__ldcg(reinterpret_cast<const uint4*>(xg + ro) + c), v);
#pragma unroll
        for (int k = 0; k < VEC; ++k) ss += v[k] * v[k];
      }
      ss = warp_sum(ss);
      const float inv = w ? rsqrtf(ss / static_cast<float>(H) + eps) : 1.f;
      for (int c = lane; c < nvec; c += 32) {
        float v[VEC], wv[VEC];
        unpack8<T>(__ldcg(reinterpret_cast<const uint4*>(xg + ro) + c), v);
        if (w) {
          unpack8<T>(reinterpret_cast<const uint4*>(w)[c], wv);
#pragma unroll
          for (int k = 0; k < VEC; ++k) v[k] = v[k] * inv * wv[k];
        }
        reinterpret_cast<uint4*>(y + ro)[c] = pack8<T>(v);
      }
    }
  }
}

int elem_bytes(int dtype) { return dtype == PS_BF16 || dtype == PS_F16 ? 2 : 0; }

}  // namespace

namespace ps_host {

int push_targets(ps::PushTargets* pt, void* const* rank_bufs, int world, int rank, int set, int max_tokens, int n,
                 int esize, bool scatter) {
  if (!rank_bufs || world < 1 || world > ps::kMaxWorld || rank < 0 || rank >= world || (set != 0 && set != 1) ||
      max_tokens < 1 || n < 1 || esize < 1) {
    set_error("linear_push: invalid world/rank/set/max_tokens");
    return PS_ERR_INVALID;
  }
  if (scatter && (n % world != 0 || (n / world) % 128 != 0)) {
    set_error("linear_push: two-shot needs N (%d) split into %d slices of whole 128-column tiles", n, world);
    return PS_ERR_UNSUPPORTED;
  }
  std::memset(pt, 0, sizeof(*pt));
  pt->world = world;
  pt->slice = scatter ? n / world : 0;
  const ps::CommLayout lay = ps::comm_layout(world, max_tokens, n, esize);
  const long long slot_bytes = static_cast<long long>(max_tokens) * (scatter ? n / world : n) * esize;
  for (int r = 0; r < world; ++r) {
    unsigned char* b = static_cast<unsigned char*>(rank_bufs[r]);
    if (!b || !aligned(b, 256)) {
      set_error("linear_push: receive buffer of rank %d is null or not 256-byte aligned", r);
      return PS_ERR_INVALID;
    }
    pt->dst[r] = b + lay.slots + (static_cast<long long>(set) * world + rank) * slot_bytes;
    pt->flag[r] = reinterpret_cast<unsigned*>(b) + set;
  }
  pt->arrivals = reinterpret_cast<unsigned*>(rank_bufs[rank]) + 32 + set;
  pt->max_tokens = max_tokens;
  return PS_OK;
}

}  // namespace ps_host

extern "C" {

PS_API size_t ps_comm_buffer_bytes(int world, int max_tokens, int hidden, int dtype) {
  const int es = elem_bytes(dtype);
  if (world < 1 || world > ps::kMaxWorld || max_tokens < 1 || hidden < 1 || es == 0) return 0;
  return static_cast<size_t>(ps::comm_layout(world, max_tokens, hidden, es).total);
}

PS_API int ps_comm_alloc(void** buf, size_t bytes) {
  if (!buf || bytes == 0) {
    ps_host::set_error("comm_alloc: invalid arguments");
    return PS_ERR_INVALID;
  }
  *buf = nullptr;
  cudaError_t e = cudaMalloc(buf, bytes);
  if (e == cudaSuccess) e = cudaMemset(*buf, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    ps_host::set_error("comm_alloc: %s", cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  return PS_OK;
}

PS_API int ps_comm_reset(void* buf, ps_stream_t stream) {
  if (!buf) {
    ps_host::set_error("comm_reset: null buffer");
    return PS_ERR_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(buf, 0, PS_COMM_CTRL_BYTES, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    ps_host::set_error("comm_reset: %s", cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  return PS_OK;
}

PS_API int ps_comm_free(void* buf) {
  const cudaError_t e = cudaFree(buf);
  if (e != cudaSuccess) {
    ps_host::set_error("comm_free: %s", cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  return PS_OK;
}

PS_API int ps_ipc_get_handle(void* buf, void* handle_out) {
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handles");
  if (!buf || !handle_out) {
    ps_host::set_error("ipc_get_handle: null pointer");
    return PS_ERR_INVALID;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, buf);
  if (e != cudaSuccess) {
    ps_host::set_error("ipc_get_handle: %s", cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  std::memcpy(handle_out, &h, sizeof(h));
  return PS_OK;
}

PS_API int ps_ipc_open_handle(const void* handle, void** peer_buf) {
  if (!handle || !peer_buf) {
    ps_host::set_error("ipc_open_handle: null pointer");
    return PS_ERR_INVALID;
  }
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *peer_buf = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    ps_host::set_error("ipc_open_handle: %s", cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  return PS_OK;
}

PS_API int ps_ipc_close(void* peer_buf) {
  const cudaError_t e = cudaIpcCloseMemHandle(peer_buf);
  if (e != cudaSuccess) {
    ps_host::set_error("ipc_close: %s", cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  return PS_OK;
}

PS_API int ps_allreduce_rmsnorm(void* y, void* x, const void* weight, float eps, int M, int H, int dtype, void* buf,
                                int world, int set, int max_tokens, ps_stream_t stream) {
  const bool norm = weight != nullptr;
  if (M <= 0 || H <= 0 || H % 8 != 0 || M > max_tokens || world < 1 || world > ps::kMaxWorld ||
      (set != 0 && set != 1) || !y || !buf || (norm && !x)) {
    ps_host::set_error("allreduce_rmsnorm: invalid arguments (M=%d H=%d world=%d set=%d max_tokens=%d)", M, H,
                       world, set, max_tokens);
    return PS_ERR_INVALID;
  }
  if (!ps_host::aligned(y, 16) || !ps_host::aligned(x, 16) || !ps_host::aligned(weight, 16) ||
      !ps_host::aligned(buf, 256)) {
    ps_host::set_error("allreduce_rmsnorm: tensors must be 16-byte aligned (buffer 256-byte)");
    return PS_ERR_INVALID;
  }
  const int per = (H / 8 + 255) / 256;
  if (per > 4) {
    ps_host::set_error("allreduce_rmsnorm: hidden size %d too large", H);
    return PS_ERR_UNSUPPORTED;
  }
  const long long slot = static_cast<long long>(max_tokens) * H;
  const long long slots_off = ps::comm_layout(world, max_tokens, H, 2).slots;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* st = ps_host::status_word(PS_TU_COMM);
#define PS_ARN(T, MV, NORM)                                                                                   \
  ps_host::launch(allreduce_rmsnorm_kernel<T, MV, NORM>, M, 256, 0, s, static_cast<T*>(y), static_cast<T*>(x),            \
                                                          static_cast<const T*>(weight), eps, M, H, buf, world, \
                                                          set, slot, slots_off, st)
#define PS_ARN_N(T, MV) \
  if (norm) PS_ARN(T, MV, true); else PS_ARN(T, MV, false)
#define PS_ARN_T(T)                   \
  if (per <= 1) { PS_ARN_N(T, 1); }   \
  else if (per <= 2) { PS_ARN_N(T, 2); } \
  else { PS_ARN_N(T, 4); }
  if (dtype == PS_BF16) {
    PS_ARN_T(__nv_bfloat16);
  } else if (dtype == PS_F16) {
    PS_ARN_T(__half);
  } else {
    ps_host::set_error("allreduce_rmsnorm: dtype must be bf16 or f16");
    return PS_ERR_UNSUPPORTED;
  }
#undef PS_ARN_T
#undef PS_ARN_N
#undef PS_ARN
  ps_host::count_launch();
  return ps_host::check_launch("allreduce_rmsnorm");
}

PS_API int ps_tp_reduce_rmsnorm(void* y, const void* x_old, const void* weight, float eps, int M, int H, int dtype,
                                void* const* rank_bufs, int world, int rank, int set, int max_tokens, int phases,
                                ps_stream_t stream) {
  if (M <= 0 || H <= 0 || world < 1 || world > ps::kMaxWorld || rank < 0 || rank >= world || M > max_tokens ||
      (set != 0 && set != 1) || phases < 1 || phases > 3 || !y || !rank_bufs) {
    ps_host::set_error("tp_reduce_rmsnorm: invalid arguments (M=%d H=%d world=%d rank=%d set=%d max_tokens=%d)", M,
                       H, world, rank, set, max_tokens);
    return PS_ERR_INVALID;
  }
  if (H % world != 0 || (H / world) % 8 != 0) {
    ps_host::set_error("tp_reduce_rmsnorm: hidden %d must split into %d slices of whole 16-byte vectors", H, world);
    return PS_ERR_UNSUPPORTED;
  }
  if (!ps_host::aligned(y, 16) || !ps_host::aligned(x_old, 16) || !ps_host::aligned(weight, 16)) {
    ps_host::set_error("tp_reduce_rmsnorm: tensors must be 16-byte aligned");
    return PS_ERR_INVALID;
  }
  RankBufs rb;
  std::memset(&rb, 0, sizeof(rb));
  for (int r = 0; r < world; ++r) {
    if (!rank_bufs[r] || !ps_host::aligned(rank_bufs[r], 256)) {
      ps_host::set_error("tp_reduce_rmsnorm: receive buffer of rank %d is null or not 256-byte aligned", r);
      return PS_ERR_INVALID;
    }
    rb.b[r] = rank_bufs[r];
  }
  const ps::CommLayout lay = ps::comm_layout(world, max_tokens, H, 2);
  // rows per CTA: about one CTA per SM, at most kGatherBlocks CTAs (the counters)
  int R = (M + 147) / 148;
  if (R < 1) R = 1;
  const int grid = (M + R - 1) / R;
  if (grid > ps::kGatherBlocks) {
    ps_host::set_error("tp_reduce_rmsnorm: %d row blocks exceed %d", grid, ps::kGatherBlocks);
    return PS_ERR_UNSUPPORTED;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* st = ps_host::status_word(PS_TU_COMM);
  if (dtype == PS_BF16) {
    using T = __nv_bfloat16;
    ps_host::launch(tp_reduce_rmsnorm_kernel<T>, grid, 256, 0, s, static_cast<T*>(y), static_cast<const T*>(x_old),
                    static_cast<const T*>(weight), eps, M, H, rb, world, rank, set, max_tokens, R, phases, lay.xg,
                    lay.slots, st);
  } else if (dtype == PS_F16) {
    using T = __half;
    ps_host::launch(tp_reduce_rmsnorm_kernel<T>, grid, 256, 0, s, static_cast<T*>(y), static_cast<const T*>(x_old),
                    static_cast<const T*>(weight), eps, M, H, rb, world, rank, set, max_tokens, R, phases, lay.xg,
                    lay.slots, st);
  } else {
    ps_host::set_error("tp_reduce_rmsnorm: dtype must be bf16 or f16");
    return PS_ERR_UNSUPPORTED;
  }
  ps_host::count_launch();
  return ps_host::check_launch("tp_reduce_rmsnorm");
}

PS_API size_t ps_comm_gathered_offset(int world, int max_tokens, int hidden, int dtype, int set) {
  const int es = elem_bytes(dtype);
  if (world < 1 || world > ps::kMaxWorld || max_tokens < 1 || hidden < 1 || es == 0 || (set != 0 && set != 1))
    return 0;
  const ps::CommLayout lay = ps::comm_layout(world, max_tokens, hidden, es);
  return static_cast<size_t>(lay.xg + static_cast<long long>(set) * max_tokens * hidden * es);
}

}  // extern "C"
