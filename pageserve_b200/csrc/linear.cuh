// Internal dispatch between the linear kernels.
#pragma once
#include "comm.cuh"

namespace ps_host {
// CUDA-core weight-streaming kernel (any M; chosen for small M).
int linear_simt(void* y, const void* x, const void* w, int wdtype, const float* scale, const void* bias,
                const void* resid, int M, int N, int K, int dtype, cudaStream_t s);
// tcgen05 tensor-core kernel (bf16/f16 activations). Returns PS_ERR_UNSUPPORTED
// when the shape has no tensor-core configuration.
int linear_tc(void* y, const void* x, const void* w, int wdtype, const float* scale, const void* bias,
              const void* resid, int M, int N, int K, int dtype, void* workspace, size_t workspace_bytes,
              cudaStream_t s, const int8_t* w_tiled = nullptr, const ps::PushTargets* push = nullptr,
              bool swiglu = false);
// int8 weight re-tiled into 8 KB blocks [N/128][K/64][128][64] for linear_tc.
size_t tiled_int8_bytes(int N, int K);
int tile_int8(int8_t* dst, const int8_t* src, int N, int K, cudaStream_t s);
size_t linear_tc_workspace(int M, int N, int K);
// mma.sync weight-streaming linear for int8 weights and M <= kMmaMaxM (row-major
// or pre-tiled q); PS_ERR_UNSUPPORTED outside its domain.
constexpr int kMmaMaxM = 32;  // largest M the kernel supports
constexpr int kMmaDefaultMaxM = 16;  // default dispatch bound (the tcgen05 kernel wins above)
int linear_mma(void* y, const void* x, const int8_t* q, bool tiled, const float* scale, const void* bias,
               const void* resid, int M, int N, int K, int dtype, bool swiglu, cudaStream_t s,
               const ps::PushTargets* push = nullptr);
// Largest M the mma.sync linear serves (PS_MMA_MAX_M overrides; 0 disables).
int mma_max_m();
}  // namespace ps_host
