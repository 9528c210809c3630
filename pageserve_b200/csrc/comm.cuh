// Peer-memory push of a row-parallel linear's output (the producer half of
// the fused tensor-parallel all-reduce; the consumer is in comm.cu).
#pragma once
#include "common.cuh"

namespace ps {

constexpr int kMaxWorld = 8;

// Byte offsets inside one rank's receive buffer (every rank uses the same
// world / max_tokens / hidden / element size, so the layout is the same on
// every rank):
//   [0, PS_COMM_CTRL_BYTES)  u32 control words: flags and counters per set
//                            (words 0..63), and from byte 1024 the two-shot
//                            gather stage's per row-block arrival counters,
//                            u32 [2 sets][kGatherBlocks]
//   xg                       [2 sets][max_tokens][hidden]: the gathered
//                            residual stream of the two-shot reduction
//   slots                    [2 sets][world][max_tokens][hidden] (one-shot),
//                            or [2 sets][world][max_tokens][hidden / world]
//                            (two-shot: only this rank's column slice)
constexpr int kGatherBlocks = 256;  // row blocks (CTAs) of one two-shot reduction, at most
constexpr int kGatherCountOff = 1024;

struct CommLayout {
  long long gcount, xg, slots, total;
};

PS_HOST_DEVICE long long comm_round256(long long v) { return (v + 255) / 256 * 256; }

PS_HOST_DEVICE CommLayout comm_layout(int world, int max_tokens, int hidden, int esize) {
  CommLayout l;
  l.gcount = kGatherCountOff;
  l.xg = PS_COMM_CTRL_BYTES;
  l.slots = l.xg + comm_round256(2LL * max_tokens * hidden * esize);
  l.total = l.slots + 2LL * world * max_tokens * hidden * esize;
  return l;
}

// Where the writing grid stores its (tokens, N) output when pushing.
// One-shot (slice == 0): the same values go to every rank's slot of this
// rank. Two-shot (slice = N / world): columns [d * slice, (d + 1) * slice)
// go to rank d only, into its [max_tokens][slice] slot of this rank
// (the reduce-scatter half of the all-reduce).
struct PushTargets {
  int world;                  // 0: no push (plain output)
  void* dst[kMaxWorld];       // rank r's slot for this rank's partial (row stride N, or slice when scattering)
  unsigned* flag[kMaxWorld];  // rank r's arrival flag of this set
  unsigned* arrivals;         // this rank's CTA arrival counter of this set
  int max_tokens;             // rows of each slot
  int slice;                  // two-shot: output columns per rank (0 = one-shot)
};

// Destination of output element (m, n) in rank d's slot (d = n / slice when
// scattering, else every d).
PS_DEVICE long long push_offset(const PushTargets& pt, int m, int n, int N, int d) {
  return pt.slice ? static_cast<long long>(m) * pt.slice + (n - d * pt.slice) : static_cast<long long>(m) * N + n;
}

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
// the receive buffers rank_bufs[0..world) (comm_layout). scatter: two-shot
// (n must split into world slices of whole 128-column tiles).
int push_targets(ps::PushTargets* pt, void* const* rank_bufs, int world, int rank, int set, int max_tokens, int n,
                 int elem_bytes, bool scatter = false);
}  // namespace ps_host
