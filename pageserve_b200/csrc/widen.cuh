// Exact int8 -> bf16 / f16 widening of 16 bytes into 8 packed pairs
// (out word 2j = bytes 4j, 4j+1; word 2j+1 = bytes 4j+2, 4j+3), shared by
// the tensor-core linears.
#pragma once
#include "common.cuh"

namespace ps {

// 16 signed bytes -> 16 bf16 (exact). For byte b = s*128 + u (two's
// complement, u = low 7 bits): value = (128 + u) - (128 + 128*s); both
// terms are exact bf16 built by byte permutes, one packed subtract per pair.
PS_DEVICE void widen16_bf16(const uint4& in, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {in.x, in.y, in.z, in.w};
  uint32_t out[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t low7 = w[j] & 0x7F7F7F7Fu;
    const uint32_t sign = w[j] & 0x80808080u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t sel = h ? 0x4342u : 0x4140u;  // bytes (2h, 2h+1) -> two bf16 {0x43 : byte}
      const uint32_t a = __byte_perm(low7, 0x43434343u, sel);
      const uint32_t b = __byte_perm(sign, 0x43434343u, sel);
      uint32_t r;
      asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
      out[j * 2 + h] = r;
    }
  }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
}
PS_DEVICE void widen16_f16(const uint4& in, uint4& lo, uint4& hi) {
  // f16: 0x64:byte = 1024 + byte; flip the sign bit first, subtract 1024 + 128.
  const uint32_t w[4] = {in.x ^ 0x80808080u, in.y ^ 0x80808080u, in.z ^ 0x80808080u, in.w ^ 0x80808080u};
  uint32_t out[8];
  const uint32_t bias = 0x64806480u;  // 1152.0 in both halves
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t a = __byte_perm(w[j], 0x64646464u, h ? 0x4342u : 0x4140u);
      uint32_t r;
      asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(bias));
      out[j * 2 + h] = r;
    }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
}

}  // namespace ps
