// Shared definitions of libcuda_fletcher: context, buffers, error plumbing, dtype helpers.
#pragma once
#include <utility>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "../../include/fletcher_cuda.h"

namespace fl {

// Device-side error codes written to Ctx::d_err by kernels whose bounded waits expire.
enum DeviceErr : int32_t { kDevOk = 0, kDevWaitTimeout = 1 };

struct Ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  int64_t allocated = 0;
  int32_t* d_err = nullptr;  // device flag, set by kernels on a bounded-wait timeout
  int64_t launches = 0;      // kernels launched on this context (counted by FL_LAUNCH)
  float* splitk = nullptr;   // split-K workspace of small-M GEMMs, lent by the running model
  int64_t splitk_bytes = 0;
  int32_t half_mode = FLETCHER_HALF_REFERENCE;  // fp32 <-> fp16 conversion of host-facing copies
  // Pinned staging ring for small per-call host arrays (lengths, indices): a slot is reused
  // once the copy that last read it has completed (its event), so calls never block on the
  // stream the way a synchronous upload would.
  static constexpr int kStageSlots = 8;
  uint8_t* h_stage[kStageSlots] = {};
  int64_t h_stage_cap[kStageSlots] = {};
  cudaEvent_t stage_ev[kStageSlots] = {};
  int stage_next = 0;
  std::string last_error;
};

struct Buf {
  Ctx* ctx = nullptr;
  void* ptr = nullptr;
  int64_t bytes = 0;
  int64_t rows = 0, cols = 0;
  int32_t dtype = FLETCHER_F32;
  // Write counter: bumped by every ABI call that may change the contents (see touch()).
  uint64_t version = 0;
  // Cuda_Linear_Fused's derived copies of a 16-bit weight / bias, valid while `version` equals
  // the recorded one and the layout key (SwiGLU interleave, tile width) matches.
  void* packed = nullptr;
  int64_t packed_bytes = 0;
  int packed_key = -1;
  uint64_t packed_ver = 0;
  float* bias32 = nullptr;
  int64_t bias32_bytes = 0;
  int bias32_key = -1;
  uint64_t bias32_ver = 0;
};

// Marks a buffer as written (invalidates Cuda_Linear_Fused's cached layouts of it).
inline void touch(Buf* b) {
  if (b) b->version++;
}

// Copies `bytes` of host memory to device memory `d` in stream order through the context's
// pinned staging ring; the host array may be reused as soon as this returns.
int32_t stage_to_device(Ctx* c, void* d, const void* h, int64_t bytes);
void free_staging(Ctx* c);

inline int64_t dtype_size(int32_t dt) { return dt == FLETCHER_F32 ? 4 : 2; }

int32_t set_error(Ctx* c, int32_t code, const char* fmt, ...);

// Binds the context's device for the duration of an ABI call.
struct DeviceGuard {
  explicit DeviceGuard(const Ctx* c) { cudaSetDevice(c->device); }
};

#define FL_CUDA(ctx, call)                                                                  \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess)                                                                  \
      return ::fl::set_error((ctx), FLETCHER_ERR_CUDA, "%s failed: %s (%s:%d)", #call,      \
                             cudaGetErrorString(e_), __FILE__, __LINE__);                   \
  } while (0)

#define FL_CHECK(ctx, cond, ...)                                                            \
  do {                                                                                      \
    if (!(cond)) return ::fl::set_error((ctx), FLETCHER_ERR_INVALID, __VA_ARGS__);          \
  } while (0)

#define FL_LAUNCH(ctx)                                                                      \
  do {                                                                                      \
    (ctx)->launches++;                                                                      \
    cudaError_t e_ = cudaGetLastError();                                                    \
    if (e_ != cudaSuccess)                                                                  \
      return ::fl::set_error((ctx), FLETCHER_ERR_CUDA, "kernel launch failed: %s (%s:%d)",  \
                             cudaGetErrorString(e_), __FILE__, __LINE__);                   \
  } while (0)

// Programmatic dependent launch (sm_90+): a kernel launched with launch_pdl may begin while the
// previous kernel on the stream is finishing, so its setup (barrier init, TMEM allocation,
// tensor-map prefetch) overlaps that kernel's tail.  It must call pdl_wait() before it touches
// global memory that an earlier kernel writes or reads; the wait returns once that kernel has
// completed and its writes are visible.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Allocation from the stream-ordered pool; zero-filled.
int32_t dev_alloc(Ctx* c, void** p, int64_t bytes);
void dev_free(Ctx* c, void* p, int64_t bytes);

// ---------------------------------------------------------------- device helpers
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// The reference's host-side fp16 conversion (internal/device/utils.go:13-72), which its fp16 CUDA
// backend applies to every CopyFromFloat32 / Set / ToHost (cuda_linux.go:128,148,163): NaN ->
// 0x7E00; +-Inf kept; finite values clamped to +-65504; |x| below the smallest normal (2^-14)
// flushed to a signed zero; otherwise the mantissa is truncated (not rounded) to 10 bits.
__device__ __forceinline__ uint16_t half_bits_ref(float f) {
  if (f != f) return 0x7E00;
  if (isinf(f)) return f > 0.0f ? 0x7C00 : 0xFC00;
  f = fminf(fmaxf(f, -65504.0f), 65504.0f);
  const float a = fabsf(f);
  if (a < 6.103515625e-05f && a > 0.0f) return f < 0.0f ? 0x8000 : 0x0000;
  const uint32_t bits = __float_as_uint(f);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const int e = (int)((bits >> 23) & 0xFF) - 127 + 15;
  const uint32_t frac = (bits >> 13) & 0x3FFu;
  if (e >= 0x1F) return (uint16_t)(sign | 0x7BFFu);
  if (e <= 0) return (uint16_t)sign;
  return (uint16_t)(sign | ((uint32_t)e << 10) | frac);
}
// Float16ToFloat32 (utils.go:75-91): zero and every subnormal read as +0; Inf/NaN keep their
// payload; normals widen exactly.
__device__ __forceinline__ float half_bits_to_f32_ref(uint16_t h) {
  const uint32_t sign = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, frac = h & 0x3FFu;
  if (e == 0) return 0.0f;
  if (e == 31) return __uint_as_float((sign << 31) | (0xFFu << 23) | (frac << 13));
  return __uint_as_float((sign << 31) | ((e - 15 + 127) << 23) | (frac << 13));
}
// Host-facing conversions: fp16 follows the context's mode (the reference's bytes, or IEEE
// round-to-nearest-even); bf16 and fp32 are unaffected.
template <typename T> __device__ __forceinline__ T from_f_host(float v, bool ref) { return from_f<T>(v); }
template <> __device__ __forceinline__ __half from_f_host<__half>(float v, bool ref) {
  return ref ? __ushort_as_half(half_bits_ref(v)) : __float2half_rn(v);
}
template <typename T> __device__ __forceinline__ float to_f_host(T v, bool ref) { return to_f<T>(v); }
template <> __device__ __forceinline__ float to_f_host<__half>(__half v, bool ref) {
  return ref ? half_bits_to_f32_ref(__half_as_ushort(v)) : __half2float(v);
}

// The reference's fast-math helpers (internal/simd/simd.go), written with explicitly
// rounded float operations so that the compiler cannot contract them into FMAs: the
// results then match the Go code (which does not fuse on amd64) operation for operation.
// ExpFast, simd.go:7-46.
__device__ __forceinline__ float exp_fast(float x) {
  if (x > 88.0f) return 1e38f;
  if (x < -88.0f) return 0.0f;
  float t = __fmul_rn(x, 1.442695f);
  int k = (int)t;  // truncation toward zero, as Go's int(t)
  if (t < 0.0f) k--;
  float f = __fsub_rn(t, (float)k);
  float p = __fadd_rn(1.0f, __fmul_rn(f, __fadd_rn(0.6931472f, __fmul_rn(f, __fadd_rn(0.2402265f, __fmul_rn(f, 0.0555041f))))));
  // 2^k exactly; k is in [-128, 127] here, so 2^k may be subnormal.
  float two_k = k >= -126 ? __int_as_float((k + 127) << 23) : __int_as_float(1 << (k + 149));
  return __fmul_rn(p, two_k);
}
// TanhFast, simd.go:49-63.
__device__ __forceinline__ float tanh_fast(float x) {
  if (x > 4.0f) return 1.0f;
  if (x < -4.0f) return -1.0f;
  float x2 = __fmul_rn(x, x);
  return __fdiv_rn(__fmul_rn(x, __fadd_rn(27.0f, x2)), __fadd_rn(27.0f, __fmul_rn(9.0f, x2)));
}
// GeluFast, simd.go:66-75: 0.5*x*(1 + TanhFast(0.7978846*(x + 0.044715*x^3))).
__device__ __forceinline__ float gelu_fast(float x) {
  float c3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  float th = tanh_fast(__fmul_rn(0.7978846f, __fadd_rn(x, c3)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, th));
}
// GeluFast for the 16-bit epilogues: the same formula with fused multiply-adds and a fast
// division (a few ulp of fp32, far below the 16-bit output's resolution), as selects rather than
// branches.
__device__ __forceinline__ float gelu_fast16(float x) {
  const float u = 0.7978846f * fmaf(0.044715f * x, x * x, x);
  const float u2 = u * u;
  const float pade = __fdividef(u * (27.0f + u2), fmaf(9.0f, u2, 27.0f));
  const float th = fabsf(u) > 4.0f ? copysignf(1.0f, u) : pade;
  return 0.5f * x * (1.0f + th);
}
// SwiGLU element (cpu_backend.go:649-650): x / (1 + float32(exp(float64(-x)))) * y.
__device__ __forceinline__ float swiglu_exact(float x, float y) {
  float e = (float)exp(-(double)x);
  return __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, e)), y);
}

// Packed two-lane fp32 FMA / add / multiply (sm_100): one instruction for two values.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0, float c1) {
  asm("{\n .reg .b64 a, b, c, d;\n mov.b64 a, {%2, %3};\n mov.b64 b, {%4, %5};\n mov.b64 c, {%6, %7};\n"
      " fma.rn.f32x2 d, a, b, c;\n mov.b64 {%0, %1}, d;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1) {
  asm("{\n .reg .b64 a, d;\n mov.b64 d, {%0, %1};\n mov.b64 a, {%2, %3};\n add.rn.f32x2 d, d, a;\n"
      " mov.b64 {%0, %1}, d;\n}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1));
}
__device__ __forceinline__ void mul2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n .reg .b64 a, b, d;\n mov.b64 a, {%2, %3};\n mov.b64 b, {%4, %5};\n mul.rn.f32x2 d, a, b;\n"
      " mov.b64 {%0, %1}, d;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace fl
