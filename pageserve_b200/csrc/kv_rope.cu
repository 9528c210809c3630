// KV-slot writes, slot mapping and RoPE (engine/paged_attention.py:62-79,
// engine/model.py:37-54, 168-178 of the reference).
//
// All of these are HBM-bound byte movers: one pass over their inputs, 16-byte
// vector accesses where the row width allows, no shared memory.
#include "common.cuh"

namespace {

using namespace ps;

// ---------------------------------------------------------------- write_kv --
// One thread per 16-byte (or Unit-sized) chunk of one token's K or V row.
template <typename Unit>
__global__ void write_kv_kernel(char* __restrict__ k_cache, char* __restrict__ v_cache,
                                const int32_t* __restrict__ table, int num_blocks, int block_size,
                                int row_units, int start_pos, int num_tokens, const char* __restrict__ k,
                                const char* __restrict__ v, int* status) {
  const long long work = static_cast<long long>(num_tokens) * row_units * 2;
  for (long long w = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; w < work;
       w += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int which = static_cast<int>(w / (static_cast<long long>(num_tokens) * row_units));  // 0 = K, 1 = V
    const long long r = w - static_cast<long long>(which) * num_tokens * row_units;
    const int t = static_cast<int>(r / row_units);
    const int u = static_cast<int>(r - static_cast<long long>(t) * row_units);
    const int pos = start_pos + t;
    const int phys = table[pos / block_size];
    if (phys < 0 || phys >= num_blocks) {
      record_error(status, kErrBlockId);
      continue;
    }
    const long long slot = static_cast<long long>(phys) * block_size + pos % block_size;
    const Unit* src = reinterpret_cast<const Unit*>(which ? v : k) + static_cast<long long>(t) * row_units + u;
    Unit* dst = reinterpret_cast<Unit*>(which ? v_cache : k_cache) + slot * row_units + u;
    *dst = *src;
  }
}

// ------------------------------------------------------------ slot mapping --
__global__ void slot_mapping_kernel(int32_t* __restrict__ positions, int32_t* __restrict__ slots,
                                    const int32_t* __restrict__ tables, int max_blocks,
                                    const int32_t* __restrict__ cu_q, const int32_t* __restrict__ start_pos,
                                    int num_seqs, int total_tokens, int num_blocks, int block_size, int* status) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= total_tokens) return;
  // sequence of token t: last b with cu_q[b] <= t
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_q[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int pos = start_pos[b] + (t - cu_q[b]);
  positions[t] = pos;
  const int bi = pos / block_size;
  int slot = -1;
  if (pos < 0 || bi >= max_blocks) {
    record_error(status, kErrShape);
  } else {
    const int phys = tables[static_cast<long long>(b) * max_blocks + bi];
    if (phys < 0 || phys >= num_blocks) record_error(status, kErrBlockId);
    else slot = phys * block_size + pos % block_size;
  }
  slots[t] = slot;
}

// ------------------------------------------------------ fused rope + write --
// Work item = (token, head, chunk of 8 rotation pairs). Heads [0, Hq) are q,
// [Hq, Hq+Hkv) k, [Hq+Hkv, Hq+2Hkv) v. q/k are rotated in float32 with the
// float32 cos/sin table; v is copied.
template <typename T>
__global__ void rope_qkv_kernel(T* __restrict__ q_out, T* __restrict__ k_cache, T* __restrict__ v_cache,
                                const T* __restrict__ qkv, const int32_t* __restrict__ positions,
                                const int32_t* __restrict__ slots, const float* __restrict__ cos_tab,
                                const float* __restrict__ sin_tab, int max_pos, int num_tokens, int Hq, int Hkv,
                                int D, int num_slots, int* status) {
  pdl_wait();
  pdl_trigger();
  const int half = D / 2;
  const int chunks = half / 8;
  const int heads = Hq + 2 * Hkv;
  const long long work = static_cast<long long>(num_tokens) * heads * chunks;
  for (long long w = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; w < work;
       w += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(w % chunks);
    const int h = static_cast<int>((w / chunks) % heads);
    const int t = static_cast<int>(w / (static_cast<long long>(chunks) * heads));
    const T* src = qkv + static_cast<long long>(t) * heads * D + static_cast<long long>(h) * D;
    const uint4 lo_u = *reinterpret_cast<const uint4*>(src + c * 8);
    const uint4 hi_u = *reinterpret_cast<const uint4*>(src + half + c * 8);
    uint4 out_lo = lo_u, out_hi = hi_u;
    if (h < Hq + Hkv) {
      int pos = positions[t];
      if (pos < 0 || pos >= max_pos) {
        record_error(status, kErrShape);
        pos = pos < 0 ? 0 : max_pos - 1;
      }
      float x1[8], x2[8], y1[8], y2[8];
      unpack8<T>(lo_u, x1);
      unpack8<T>(hi_u, x2);
      const float4* cp = reinterpret_cast<const float4*>(cos_tab + static_cast<long long>(pos) * half + c * 8);
      const float4* sp = reinterpret_cast<const float4*>(sin_tab + static_cast<long long>(pos) * half + c * 8);
      const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
      const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // rotate_half(x) = cat(-x2, x1); cos/sin are duplicated halves.
        y1[i] = x1[i] * cs[i] - x2[i] * sn[i];
        y2[i] = x2[i] * cs[i] + x1[i] * sn[i];
      }
      out_lo = pack8<T>(y1);
      out_hi = pack8<T>(y2);
    }
    if (h < Hq) {
      T* dst = q_out + (static_cast<long long>(t) * Hq + h) * D;
      *reinterpret_cast<uint4*>(dst + c * 8) = out_lo;
      *reinterpret_cast<uint4*>(dst + half + c * 8) = out_hi;
    } else {
      const int slot = slots[t];
      if (slot < 0) continue;
      if (slot >= num_slots) {
        record_error(status, kErrSlot);
        continue;
      }
      const bool is_k = h < Hq + Hkv;
      const int kh = is_k ? h - Hq : h - Hq - Hkv;
      T* dst = (is_k ? k_cache : v_cache) + (static_cast<long long>(slot) * Hkv + kh) * D;
      *reinterpret_cast<uint4*>(dst + c * 8) = out_lo;
      *reinterpret_cast<uint4*>(dst + half + c * 8) = out_hi;
    }
  }
}

// ------------------------------------------------------ reference apply_rope --
template <typename T>
__global__ void apply_rope_kernel(T* __restrict__ out, const T* __restrict__ x, const T* __restrict__ cosv,
                                  const T* __restrict__ sinv, int num_tokens, int H, int D) {
  const int half = D / 2;
  const long long work = static_cast<long long>(num_tokens) * H * half;
  for (long long w = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; w < work;
       w += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(w % half);
    const long long th = w / half;
    const int t = static_cast<int>(th / H);
    const T* xr = x + th * D;
    const float a = to_f32(xr[i]), b = to_f32(xr[i + half]);
    const T* cr = cosv + static_cast<long long>(t) * D;
    const T* sr = sinv + static_cast<long long>(t) * D;
    out[th * D + i] = from_f32<T>(a * to_f32(cr[i]) - b * to_f32(sr[i]));
    out[th * D + i + half] = from_f32<T>(b * to_f32(cr[i + half]) + a * to_f32(sr[i + half]));
  }
}

int grid_for(long long work, int threads) {
  long long g = (work + threads - 1) / threads;
  const long long cap = 148LL * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

int elem_size(int dtype) {
  switch (dtype) {
    case PS_F32: return 4;
    case PS_BF16: case PS_F16: return 2;
    case PS_I8: return 1;
  }
  return 0;
}

// ------------------------------------------------------------- copy_blocks --
// Copy-on-write of KV blocks: for every (src, dst) pair and every layer, the
// whole block (block_size x Hkv x D) of K and V is copied. One CTA-stride loop
// over (pair, layer, K/V, 16-byte unit). Ids outside [0, num_blocks) skip the
// pair and are recorded.
__global__ void copy_blocks_kernel(uint4* __restrict__ k_cache, uint4* __restrict__ v_cache,
                                   const int32_t* __restrict__ pairs, int n_pairs, int num_layers,
                                   long long layer_units, long long block_units, int num_blocks, int* status) {
  const long long per_pair = 2LL * num_layers * block_units;
  const long long work = per_pair * n_pairs;
  for (long long w = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; w < work;
       w += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(w / per_pair);
    long long r = w - static_cast<long long>(p) * per_pair;
    const int which = static_cast<int>(r / (num_layers * block_units));  // 0 = K, 1 = V
    r -= static_cast<long long>(which) * num_layers * block_units;
    const int layer = static_cast<int>(r / block_units);
    const long long u = r - static_cast<long long>(layer) * block_units;
    const int src = pairs[2 * p], dst = pairs[2 * p + 1];
    if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) {
      record_error(status, kErrBlockId);
      continue;
    }
    uint4* c = which ? v_cache : k_cache;
    const long long base = static_cast<long long>(layer) * layer_units;
    c[base + static_cast<long long>(dst) * block_units + u] = c[base + static_cast<long long>(src) * block_units + u];
  }
}

}  // namespace

extern "C" {

int ps_copy_kv_blocks(void* k_cache, void* v_cache, const int32_t* pairs, int n_pairs, int num_layers, int num_blocks,
                      int block_size, int num_kv_heads, int head_dim, int dtype, ps_stream_t stream) {
  const int es = elem_size(dtype);
  if (!es || dtype == PS_I8) {
    ps_host::set_error("copy_kv_blocks: unsupported dtype %d", dtype);
    return PS_ERR_UNSUPPORTED;
  }
  if (n_pairs < 0 || num_layers <= 0 || num_blocks <= 0 || block_size <= 0 || num_kv_heads <= 0 || head_dim <= 0) {
    ps_host::set_error("copy_kv_blocks: invalid sizes");
    return PS_ERR_INVALID;
  }
  if (n_pairs == 0) return PS_OK;
  if (!k_cache || !v_cache || !pairs) {
    ps_host::set_error("copy_kv_blocks: null pointer");
    return PS_ERR_INVALID;
  }
  const long long block_bytes = static_cast<long long>(block_size) * num_kv_heads * head_dim * es;
  if (block_bytes % 16 != 0 || !ps_host::aligned(k_cache, 16) || !ps_host::aligned(v_cache, 16)) {
    ps_host::set_error("copy_kv_blocks: blocks must be whole 16-byte units and the caches 16-byte aligned");
    return PS_ERR_INVALID;
  }
  const long long block_units = block_bytes / 16;
  const long long layer_units = block_units * num_blocks;
  const int threads = 256;
  copy_blocks_kernel<<<grid_for(2LL * n_pairs * num_layers * block_units, threads), threads, 0,
                       reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(k_cache), static_cast<uint4*>(v_cache), pairs, n_pairs, num_layers, layer_units,
      block_units, num_blocks, ps_host::status_word(PS_TU_KV));
  ps_host::count_launch();
  return ps_host::check_launch("copy_kv_blocks");
}

int ps_write_kv(void* k_cache, void* v_cache, const int32_t* table, int table_len, int num_blocks,
                int block_size, int num_kv_heads, int head_dim, int dtype, int start_pos, int num_tokens,
                const void* k, const void* v, ps_stream_t stream) {
  const int es = elem_size(dtype);
  if (!es || dtype == PS_I8) {
    ps_host::set_error("write_kv: unsupported dtype %d", dtype);
    return PS_ERR_UNSUPPORTED;
  }
  if (num_tokens < 0 || start_pos < 0 || block_size <= 0 || num_kv_heads <= 0 || head_dim <= 0) {
    ps_host::set_error("write_kv: invalid sizes");
    return PS_ERR_INVALID;
  }
  if (num_tokens == 0) return PS_OK;
  if ((start_pos + num_tokens - 1) / block_size >= table_len) {
    ps_host::set_error("write_kv: block_table has %d entries, position %d needs entry %d", table_len,
                       start_pos + num_tokens - 1, (start_pos + num_tokens - 1) / block_size);
    return PS_ERR_INDEX;
  }
  if (!k_cache || !v_cache || !table || !k || !v) {
    ps_host::set_error("write_kv: null pointer");
    return PS_ERR_INVALID;
  }
  const long long row_bytes = static_cast<long long>(num_kv_heads) * head_dim * es;
  const uintptr_t align = reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
                          reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v);
  int* status = ps_host::status_word(PS_TU_KV);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int threads = 256;
  if (row_bytes % 16 == 0 && align % 16 == 0) {
    const int units = static_cast<int>(row_bytes / 16);
    write_kv_kernel<uint4><<<grid_for(2LL * num_tokens * units, threads), threads, 0, s>>>(
        static_cast<char*>(k_cache), static_cast<char*>(v_cache), table, num_blocks, block_size, units, start_pos,
        num_tokens, static_cast<const char*>(k), static_cast<const char*>(v), status);
  } else if (row_bytes % 4 == 0 && align % 4 == 0) {
    const int units = static_cast<int>(row_bytes / 4);
    write_kv_kernel<uint32_t><<<grid_for(2LL * num_tokens * units, threads), threads, 0, s>>>(
        static_cast<char*>(k_cache), static_cast<char*>(v_cache), table, num_blocks, block_size, units, start_pos,
        num_tokens, static_cast<const char*>(k), static_cast<const char*>(v), status);
  } else {
    const int units = static_cast<int>(row_bytes / 2);
    write_kv_kernel<uint16_t><<<grid_for(2LL * num_tokens * units, threads), threads, 0, s>>>(
        static_cast<char*>(k_cache), static_cast<char*>(v_cache), table, num_blocks, block_size, units, start_pos,
        num_tokens, static_cast<const char*>(k), static_cast<const char*>(v), status);
  }
  ps_host::count_launch();
  return ps_host::check_launch("write_kv");
}

int ps_build_slot_mapping(int32_t* positions, int32_t* slots, const int32_t* tables, int max_blocks,
                          const int32_t* cu_q, const int32_t* start_pos, int num_seqs, int total_tokens,
                          int num_blocks, int block_size, ps_stream_t stream) {
  if (num_seqs <= 0 || total_tokens < 0 || max_blocks <= 0 || block_size <= 0) {
    ps_host::set_error("build_slot_mapping: invalid sizes");
    return PS_ERR_INVALID;
  }
  if (total_tokens == 0) return PS_OK;
  const int threads = 256;
  ps_host::launch(slot_mapping_kernel, (total_tokens + threads - 1) / threads, threads, 0,
                        reinterpret_cast<cudaStream_t>(stream), positions, slots, tables, max_blocks, cu_q,
                                                                  start_pos, num_seqs, total_tokens, num_blocks,
                                                                  block_size, ps_host::status_word(PS_TU_KV));
  ps_host::count_launch();
  return ps_host::check_launch("build_slot_mapping");
}

int ps_rope_qkv_write_kv(void* q_out, void* k_cache, void* v_cache, const void* qkv, const int32_t* positions,
                         const int32_t* slots, const float* rope_cos, const float* rope_sin, int max_pos, int T,
                         int Hq, int Hkv, int D, int num_slots, int dtype, ps_stream_t stream) {
  if (D % 16 != 0 || Hq <= 0 || Hkv <= 0 || T < 0) {
    ps_host::set_error("rope_qkv_write_kv: head_dim must be a multiple of 16 (got %d)", D);
    return PS_ERR_UNSUPPORTED;
  }
  if (T == 0) return PS_OK;
  if (!ps_host::aligned(q_out, 16) || !ps_host::aligned(k_cache, 16) || !ps_host::aligned(v_cache, 16) ||
      !ps_host::aligned(qkv, 16) || !ps_host::aligned(rope_cos, 16) || !ps_host::aligned(rope_sin, 16)) {
    ps_host::set_error("rope_qkv_write_kv: tensors must be 16-byte aligned");
    return PS_ERR_INVALID;
  }
  const long long work = static_cast<long long>(T) * (Hq + 2 * Hkv) * (D / 16);
  const int threads = 128;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* status = ps_host::status_word(PS_TU_KV);
  if (dtype == PS_BF16) {
    ps_host::launch(rope_qkv_kernel<__nv_bfloat16>, grid_for(work, threads), threads, 0, s, 
        static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cache),
        static_cast<__nv_bfloat16*>(v_cache), static_cast<const __nv_bfloat16*>(qkv), positions, slots, rope_cos,
        rope_sin, max_pos, T, Hq, Hkv, D, num_slots, status);
  } else if (dtype == PS_F16) {
    ps_host::launch(rope_qkv_kernel<__half>, grid_for(work, threads), threads, 0, s, 
        static_cast<__half*>(q_out), static_cast<__half*>(k_cache), static_cast<__half*>(v_cache),
        static_cast<const __half*>(qkv), positions, slots, rope_cos, rope_sin, max_pos, T, Hq, Hkv, D, num_slots,
        status);
  } else {
    ps_host::set_error("rope_qkv_write_kv: dtype must be bf16 or f16");
    return PS_ERR_UNSUPPORTED;
  }
  ps_host::count_launch();
  return ps_host::check_launch("rope_qkv_write_kv");
}

int ps_apply_rope(void* out, const void* x, const void* cosv, const void* sinv, int T, int H, int D, int dtype,
                  ps_stream_t stream) {
  if (D % 2 != 0 || T < 0 || H <= 0) {
    ps_host::set_error("apply_rope: invalid sizes");
    return PS_ERR_INVALID;
  }
  if (T == 0) return PS_OK;
  const long long work = static_cast<long long>(T) * H * (D / 2);
  const int threads = 256;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PS_F32:
      apply_rope_kernel<float><<<grid_for(work, threads), threads, 0, s>>>(
          static_cast<float*>(out), static_cast<const float*>(x), static_cast<const float*>(cosv),
          static_cast<const float*>(sinv), T, H, D);
      break;
    case PS_BF16:
      apply_rope_kernel<__nv_bfloat16><<<grid_for(work, threads), threads, 0, s>>>(
          static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(x),
          static_cast<const __nv_bfloat16*>(cosv), static_cast<const __nv_bfloat16*>(sinv), T, H, D);
      break;
    case PS_F16:
      apply_rope_kernel<__half><<<grid_for(work, threads), threads, 0, s>>>(
          static_cast<__half*>(out), static_cast<const __half*>(x), static_cast<const __half*>(cosv),
          static_cast<const __half*>(sinv), T, H, D);
      break;
    default:
      ps_host::set_error("apply_rope: unsupported dtype");
      return PS_ERR_UNSUPPORTED;
  }
  ps_host::count_launch();
  return ps_host::check_launch("apply_rope");
}

}  // extern "C"
