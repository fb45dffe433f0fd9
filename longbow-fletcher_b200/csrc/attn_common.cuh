// Device helpers of the tcgen05 attention kernel (attention_tc.cu):
// the exp2 / packed-fp32 arithmetic of the softmax rows, TMEM row loads and the MN-major
// operand descriptor.
#pragma once
#include "tc_common.cuh"

namespace fl {
namespace tca {

using namespace tc;

// 2^x on the SFU (one instruction; -inf -> 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 256-bit global store (sm_100), not allocated in L1.  dst must be 32-byte aligned.
__device__ __forceinline__ void st_global_256(void* dst, const uint32_t (&u)[8]) {
  asm volatile("st.global.L1::no_allocate.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(u[0]),
               "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7])
               : "memory");
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// Keys at and past `valid` lie outside the sequence.
template <int N>
__device__ __forceinline__ void mask_tail(float (&sv)[N], int valid) {
#pragma unroll
  for (int i = 0; i < N; i++)
    if (i >= valid) sv[i] = -INFINITY;
}
// Row max as a short tree of 3-input max instructions.
template <int N>
__device__ __forceinline__ float row_max(const float (&sv)[N]) {
  float mp[8];
#pragma unroll
  for (int k = 0; k < 8; k++) mp[k] = fmaxf(sv[k], sv[8 + k]);
#pragma unroll
  for (int c = 16; c + 16 <= N; c += 16)
#pragma unroll
    for (int k = 0; k < 8; k++) mp[k] = max3(mp[k], sv[c + k], sv[c + 8 + k]);
  return max3(max3(mp[0], mp[1], mp[2]), max3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
}

// Largest P (checked through the row sum, which bounds it) between reference-max updates: 2^64 for bf16 (fp32 O and row sums stay far from
// overflow), 2^15 for fp16 (its largest finite value is 65504).
template <typename T>
__device__ __forceinline__ float kPMax() {
  return std::is_same<T, __nv_bfloat16>::value ? 18446744073709551616.0f : 32768.0f;
}

// P = 2^(S * scale * log2 e - ms) for an N-key row: 16-bit pairs in pk, fp32 sum in `sum`.
template <typename T, int N>
__device__ __forceinline__ void exp_row(float (&sv)[N], float sl2, float ms, uint32_t (&pk)[N / 2], float& sum) {
  float ra[4][2] = {};  // four independent packed partial sums
#pragma unroll
  for (int i = 0; i < N; i += 2) {
    fma2(sv[i], sv[i + 1], sv[i], sv[i + 1], sl2, sl2, -ms, -ms);
    sv[i] = ex2(sv[i]);
    sv[i + 1] = ex2(sv[i + 1]);
    add2(ra[(i >> 1) & 3][0], ra[(i >> 1) & 3][1], sv[i], sv[i + 1]);
    pk[i >> 1] = pack2<T>(sv[i], sv[i + 1]);
  }
  sum = ((ra[0][0] + ra[0][1]) + (ra[1][0] + ra[1][1])) + ((ra[2][0] + ra[2][1]) + (ra[3][0] + ra[3][1]));
}

// A row of N fp32 S columns (N = 64 or 128) with one wait.
template <int N>
__device__ __forceinline__ void tmem_ld_row(uint32_t taddr, float (&v)[N]) {
  if constexpr (N == 64) {
    tmem_ld64(taddr, v);
  } else {
    static_assert(N == 128, "row width");
    float (&a)[64] = *reinterpret_cast<float(*)[64]>(&v[0]);
    float (&b)[64] = *reinterpret_cast<float(*)[64]>(&v[64]);
    tmem_ld64x2(taddr, taddr + 64, a, b);
  }
}
// P row (N/2 packed columns).
template <int N>
__device__ __forceinline__ void tmem_st_p(uint32_t taddr, const uint32_t (&pk)[N / 2]) {
#pragma unroll
  for (int c = 0; c < N / 64; c++) tmem_st32(taddr + 32 * c, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32 * c]));
}

// MN-major, 128-byte-swizzled operand: 64 contiguous MN elements per 128-byte row, 8-row K
// groups 1024 bytes apart (SBO); a single MN atom, so LBO is not used.
__device__ __forceinline__ uint64_t sw128_desc_mn(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}


}  // namespace tca
}  // namespace fl
