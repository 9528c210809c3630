// Shared device helpers for the pageserve_b200 kernels (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pageserve_b200.h"

#define PS_DEVICE __device__ __forceinline__
#define PS_HOST_DEVICE __host__ __device__ __forceinline__

namespace ps {

// ------------------------------------------------------------ status word --
// Each translation unit owns one device status word. Kernels never trap: an
// out-of-range block id, slot or token id is recorded here (first error
// wins) and the access is skipped. The host reads and clears it through
// ps_device_status().
enum DeviceError : int {
  kErrNone = 0,
  kErrBlockId = 1,      // block-table entry outside [0, num_blocks)
  kErrSlot = 2,         // slot outside the cache
  kErrTokenId = 3,      // embedding id outside [0, vocab)
  kErrTimeout = 4,      // a bounded spin-wait gave up
  kErrShape = 5,        // per-sequence metadata inconsistent with launch bounds
};

// ----------------------------------------------------------------- types --
template <typename T> struct Vec8;  // 16 bytes of T

PS_DEVICE float to_f32(float x) { return x; }
PS_DEVICE float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
PS_DEVICE float to_f32(__half x) { return __half2float(x); }

template <typename T> PS_DEVICE T from_f32(float x);
template <> PS_DEVICE float from_f32<float>(float x) { return x; }
template <> PS_DEVICE __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> PS_DEVICE __half from_f32<__half>(float x) { return __float2half_rn(x); }

// 8 packed 16-bit values <-> 8 floats.
template <typename T>
PS_DEVICE void unpack8(const uint4& u, float* f) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32(h[i]);
}
template <typename T>
PS_DEVICE uint4 pack8(const float* f) {
  uint4 u;
  T* h = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = from_f32<T>(f[i]);
  return u;
}

// --------------------------------------------------------------- cp.async --
PS_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte async copy global->shared; src_bytes = 0 zero-fills the destination.
PS_DEVICE void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
PS_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
PS_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ------------------------------------------------------ ldmatrix / mma.sync --
PS_DEVICE void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
PS_DEVICE void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D(16x8 f32) += A(16x16) * B(16x8), A/B bf16 or f16.
template <typename T>
PS_DEVICE void mma_16816(float* d, const uint32_t* a, const uint32_t* b);
template <>
PS_DEVICE void mma_16816<__nv_bfloat16>(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <>
PS_DEVICE void mma_16816<__half>(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Two floats -> one packed 16-bit pair (lo in bits 0..15).
template <typename T> PS_DEVICE uint32_t pack2(float lo, float hi);
template <>
PS_DEVICE uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
PS_DEVICE uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// --------------------------------------------------------- warp reductions --
PS_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
PS_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// silu(g) * u in float32 (F.silu(gate) * up, engine/model.py:190), shared by
// the standalone kernel and the gate|up linear's epilogue so both give the
// same values: g / (1 + e^-g) with the fast exponential and divide (relative
// error ~1e-6, far below the bf16/f16 output rounding; 0 for g -> -inf).
// Round two floats to T (round to nearest even) and back with one packed
// convert: (float(T(a)), float(T(b))).
template <typename T> PS_DEVICE float2 round2(float a, float b);
template <> PS_DEVICE float2 round2<__nv_bfloat16>(float a, float b) {
  return __bfloat1622float2(__floats2bfloat162_rn(a, b));
}
template <> PS_DEVICE float2 round2<__half>(float a, float b) { return __half22float2(__floats2half2_rn(a, b)); }
template <> PS_DEVICE float2 round2<float>(float a, float b) { return make_float2(a, b); }

PS_DEVICE float silu_mul_f32(float g, float u) { return __fdividef(g, 1.f + __expf(-g)) * u; }

// Programmatic dependent launch (kernels launched through ps_host::launch):
// the next kernel in the stream may start while this one finishes. A kernel
// calls pdl_wait() before it reads anything an earlier kernel writes and
// before any global write (it returns once the previous grid has completed
// and its writes are visible), and pdl_trigger() to let the next kernel begin
// launching. Without the launch attribute both are no-ops.
PS_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
PS_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

PS_DEVICE void record_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

}  // namespace ps

// Host-side helpers shared by the .cu files.
namespace ps_host {
bool pdl_enabled();  // programmatic dependent launch on (PS_PDL=0 turns it off)
// Launch `kern` with the programmatic-dependent-launch attribute; `kern` must
// call ps::pdl_wait() before touching memory earlier kernels write.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}
void set_error(const char* fmt, ...);
int check_launch(const char* what);
void count_launch(int n = 1);
int* status_word(int tu);  // device status word of translation unit `tu`
// true for NULL or a pointer aligned to `bytes` (vector loads need it)
inline bool aligned(const void* p, uintptr_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }
}  // namespace ps_host

// Translation-unit ids for the device status words.
enum PsUnit { PS_TU_KV = 0, PS_TU_ATTN = 1, PS_TU_GEMV = 2, PS_TU_GEMM = 3, PS_TU_MISC = 4, PS_TU_COMM = 5, PS_TU_COUNT = 6 };
