// Peer-memory push of a row-parallel linear's output (the producer half of
// the fused tensor-parallel all-reduce; the consumer is in comm.cu).
#pragma once
#include "common.cuh"

namespace ps {

constexpr int kMaxWorld = 8;

// Where the writing grid stores its (tokens, N) output when pushing: the
// same values go to every rank's receive slot of this rank.
struct PushTargets {
  int world;                  // 0: no push (plain output)
  void* dst[kMaxWorld];       // rank r's slot for this rank's partial, [max_tokens][N], row stride N
  unsigned* flag[kMaxWorld];  // rank r's arrival flag of this set
  unsigned* arrivals;         // this rank's CTA arrival counter of this set
  int max_tokens;             // rows of each slot
};

PS_DEVICE void red_release_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Every thread of every CTA of the writing grid calls this once, after its
// last store. The CTA barrier orders all its threads' stores before thread
// 0's system-scope fence (the fence is cumulative over what the barrier made
// visible to thread 0), whose counter increment publishes them; the last CTA
// to arrive re-arms the local counter and adds one to every rank's flag, so
// a rank's flag reaches `world` once all ranks' outputs are in its slots.
PS_DEVICE void push_arrive(const PushTargets& pt) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned total = gridDim.x * gridDim.y * gridDim.z;
    const unsigned prev = atomicAdd(pt.arrivals, 1u);
    if (prev == total - 1) {
      atomicExch(pt.arrivals, 0u);
      __threadfence_system();
      for (int r = 0; r < pt.world; ++r) red_release_sys_add(pt.flag[r], 1u);
    }
  }
}

}  // namespace ps

namespace ps_host {
// Fills `pt` for rank `rank` writing set `set` of (max_tokens, n) slots into
// the receive buffers rank_bufs[0..world) (ps_comm_buffer layout).
int push_targets(ps::PushTargets* pt, void* const* rank_bufs, int world, int rank, int set, int max_tokens, int n,
                 int elem_bytes);
}  // namespace ps_host
