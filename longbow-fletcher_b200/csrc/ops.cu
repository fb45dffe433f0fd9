// Memory-bound kernels: embedding + LayerNorm, residual + LayerNorm, RoPE, SwiGLU, pooling,
// softmax, elementwise, casts and weight packing.  One warp owns one row where rows are short
// (LayerNorm, embedding), with 128-bit vector loads and warp-shuffle reductions; fp32
// statistics throughout.
#include <algorithm>

#include "kernels.cuh"

namespace fl {

template <typename T, int VEC>
struct alignas(sizeof(T) * VEC) Vec {
  T d[VEC];
};

static inline int grid_for(int64_t n, int threads, int cap = 8192) {
  int64_t b = (n + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, cap));
}

// ---------------------------------------------------------------- LayerNorm core
// Two-pass statistics over the row held in registers (cpu_backend.go:579-600):
// mean = sum/c, var = sum((x-mean)^2)/c, invStd = 1/float32(sqrt(float64(var+eps))),
// y = (x-mean)*invStd*gamma + beta.  Sums are warp-tree reductions (order differs from the
// reference's sequential sum by rounding only).
template <typename T, int PER, int VEC>
__device__ __forceinline__ void ln_finish(float (&v)[PER], int lane, int cols, const float* __restrict__ g,
                                          const float* __restrict__ b, float eps, T* __restrict__ orow) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++) s += v[i];
  s = warp_sum(s);
  const float mean = __fdiv_rn(s, (float)cols);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    float d = __fsub_rn(v[i], mean);
    q = __fadd_rn(q, __fmul_rn(d, d));
  }
  q = warp_sum(q);
  const float var = __fdiv_rn(q, (float)cols);
  const float inv = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(var, eps)));
#pragma unroll
  for (int j = 0; j < PER / VEC; j++) {
    const int e = (j * 32 + lane) * VEC;
    Vec<float, VEC> gv = *reinterpret_cast<const Vec<float, VEC>*>(g + e);
    Vec<float, VEC> bv = *reinterpret_cast<const Vec<float, VEC>*>(b + e);
    Vec<T, VEC> o;
#pragma unroll
    for (int i = 0; i < VEC; i++)
      o.d[i] = from_f<T>(__fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j * VEC + i], mean), inv), gv.d[i]), bv.d[i]));
    *reinterpret_cast<Vec<T, VEC>*>(orow + e) = o;
  }
}

template <typename T, int PER, int VEC>
__global__ void __launch_bounds__(128) k_add_ln(const T* __restrict__ x, const T* __restrict__ res, T* out,
                                                const float* __restrict__ g, const float* __restrict__ b,
                                                int64_t rows, int cols, float eps) {
  pdl_wait();
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[PER];
  const T* xr = x + row * cols;
#pragma unroll
  for (int j = 0; j < PER / VEC; j++) {
    const int e = (j * 32 + lane) * VEC;
    Vec<T, VEC> a = *reinterpret_cast<const Vec<T, VEC>*>(xr + e);
#pragma unroll
    for (int i = 0; i < VEC; i++) v[j * VEC + i] = to_f<T>(a.d[i]);
    if (res) {
      Vec<T, VEC> r = *reinterpret_cast<const Vec<T, VEC>*>(res + row * cols + e);
#pragma unroll
      for (int i = 0; i < VEC; i++) v[j * VEC + i] = __fadd_rn(v[j * VEC + i], to_f<T>(r.d[i]));
    }
  }
  ln_finish<T, PER, VEC>(v, lane, cols, g, b, eps, out + row * cols);
}

// LayerNorm of a 16-bit row stream with no residual operand (the model's path: the residual add
// is fused into the GEMM before it).  Persistent warps walk rows with a stride and keep the next
// row's raw 16-bit data in flight while they normalise the current one: twice the bytes in
// flight per warp at the same occupancy (about 32 warps per SM at this register count), for
// the DRAM latency that bounds a one-row-per-warp kernel.  Same arithmetic as k_add_ln.
// LayerNorm of a row held as PER values per lane (lanes own 16-byte groups (j*32 + lane)*VEC),
// in packed f32x2 arithmetic: two-pass statistics (mean, then the mean of squared deviations),
// inv = 1/float32(sqrt(float64(var + eps))), y = (x - mean) * inv * gamma + beta with the last
// step fused.  Half the instructions of the scalar form; results differ from it by fp32
// rounding only.  v holds y on return.
template <int PER, int VEC>
__device__ __forceinline__ void ln_row_x2(float (&v)[PER], int lane, int cols, const float* __restrict__ g,
                                          const float* __restrict__ b, float eps) {
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i += 2) add2(s0, s1, v[i], v[i + 1]);
  const float mean = __fdiv_rn(warp_sum(s0 + s1), (float)cols);
  float q0 = 0.f, q1 = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i += 2) {
    add2(v[i], v[i + 1], -mean, -mean);
    fma2(q0, q1, v[i], v[i + 1], v[i], v[i + 1], q0, q1);
  }
  const float var = __fdiv_rn(warp_sum(q0 + q1), (float)cols);
  const float inv = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(var, eps)));
#pragma unroll
  for (int j = 0; j < PER / VEC; j++) {
    const int e = (j * 32 + lane) * VEC;
    Vec<float, VEC> gv = *reinterpret_cast<const Vec<float, VEC>*>(g + e);
    Vec<float, VEC> bv = *reinterpret_cast<const Vec<float, VEC>*>(b + e);
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      float* y = &v[j * VEC + i];
      mul2(y[0], y[1], y[0], y[1], inv, inv);
      fma2(y[0], y[1], y[0], y[1], gv.d[i], gv.d[i + 1], bv.d[i], bv.d[i + 1]);
    }
  }
}

constexpr int kLnPipeWarps = 8;
template <typename T, int PER, int VEC, int MINB>
__global__ void __launch_bounds__(kLnPipeWarps * 32, MINB) k_ln_pipe(const T* __restrict__ x, T* __restrict__ out,
                                                               const float* __restrict__ g,
                                                               const float* __restrict__ b, int64_t rows, int cols,
                                                               float eps) {
  constexpr int NV = PER / VEC;
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * kLnPipeWarps;
  int64_t row = (int64_t)blockIdx.x * kLnPipeWarps + (threadIdx.x >> 5);
  Vec<T, VEC> cur[NV], nxt[NV];
  if (row < rows) {
#pragma unroll
    for (int j = 0; j < NV; j++) cur[j] = *reinterpret_cast<const Vec<T, VEC>*>(x + row * cols + (j * 32 + lane) * VEC);
  }
  for (; row < rows; row += nw) {
    const int64_t nr = row + nw;
    if (nr < rows) {
#pragma unroll
      for (int j = 0; j < NV; j++) nxt[j] = *reinterpret_cast<const Vec<T, VEC>*>(x + nr * cols + (j * 32 + lane) * VEC);
    }
    float v[PER];
#pragma unroll
    for (int j = 0; j < NV; j++)
#pragma unroll
      for (int i = 0; i < VEC; i++) v[j * VEC + i] = to_f<T>(cur[j].d[i]);
    ln_row_x2<PER, VEC>(v, lane, cols, g, b, eps);
    T* orow = out + row * cols;
#pragma unroll
    for (int j = 0; j < NV; j++) {
      Vec<T, VEC> o;
#pragma unroll
      for (int i = 0; i < VEC; i++) o.d[i] = from_f<T>(v[j * VEC + i]);
      *reinterpret_cast<Vec<T, VEC>*>(orow + (j * 32 + lane) * VEC) = o;
      cur[j] = nxt[j];
    }
  }
}

// Fallback for rows that are not a multiple of 32 elements or longer than 1024: one block per
// row, three passes over global memory.
template <typename T>
__global__ void k_add_ln_generic(const T* x, const T* res, T* out, const float* g, const float* b,
                                 int64_t rows, int cols, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * cols;
  const T* rr = res ? res + row * cols : nullptr;
  auto val = [&](int j) { return rr ? __fadd_rn(to_f<T>(xr[j]), to_f<T>(rr[j])) : to_f<T>(xr[j]); };
  auto block_sum = [&](float s) {
    s = warp_sum(s);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
    return t;
  };
  float s = 0.f;
  for (int j = threadIdx.x; j < cols; j += blockDim.x) s += val(j);
  const float mean = __fdiv_rn(block_sum(s), (float)cols);
  float q = 0.f;
  for (int j = threadIdx.x; j < cols; j += blockDim.x) {
    float d = __fsub_rn(val(j), mean);
    q = __fadd_rn(q, __fmul_rn(d, d));
  }
  const float var = __fdiv_rn(block_sum(q), (float)cols);
  const float inv = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(var, eps)));
  __syncthreads();
  for (int j = threadIdx.x; j < cols; j += blockDim.x)
    out[row * cols + j] = from_f<T>(__fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(val(j), mean), inv), g[j]), b[j]));
}

template <typename T>
static int32_t add_ln_t(Ctx* c, const T* x, const T* res, T* out, const float* g, const float* b,
                        int64_t rows, int64_t cols, float eps) {
  if (rows == 0) return FLETCHER_OK;
  const int per = (int)(cols / 32);
  const int grid = (int)((rows * 32 + 127) / 128);
  constexpr int V16 = sizeof(T) == 2 ? 8 : 4;
  bool done = true;
  if constexpr (sizeof(T) == 2) {
    if (!res && (cols == 768 || cols == 1024 || cols == 512 || cols == 256)) {
      // Three 8-warp blocks per SM (80 registers, no spills); a fourth (forced to 64 registers)
      // spilled and measured 38.1-38.4 against 35.9 us for a cfg3-sized LayerNorm.
      const int64_t want = (rows + kLnPipeWarps - 1) / kLnPipeWarps;
      const int grid2 = (int)std::min<int64_t>(want, (int64_t)c->num_sms * 3);
#define FL_LNP2(PER_) \
  FL_CUDA(c, launch_pdl(k_ln_pipe<T, PER_, 8, 3>, dim3(grid2), dim3(kLnPipeWarps * 32), 0, c->stream, x, out, g, b, rows, (int)cols, eps))
      if (cols == 768) FL_LNP2(24);
      else if (cols == 1024) FL_LNP2(32);
      else if (cols == 512) FL_LNP2(16);
      else FL_LNP2(8);
#undef FL_LNP2
      FL_LAUNCH(c);
      return FLETCHER_OK;
    }
  }
  if (cols % 32 != 0) done = false;
#define FL_LN(PER_, VEC_) \
  FL_CUDA(c, launch_pdl(k_add_ln<T, PER_, VEC_>, dim3(grid), dim3(128), 0, c->stream, x, res, out, g, b, rows, (int)cols, eps))
  else if (per == 24 && cols % (32 * V16) == 0) FL_LN(24, V16);
  else if (per == 32 && cols % (32 * V16) == 0) FL_LN(32, V16);
  else if (per == 16 && cols % (32 * V16) == 0) FL_LN(16, V16);
  else if (per == 8 && cols % (32 * V16) == 0) FL_LN(8, V16);
  else if (per == 12 && cols % 128 == 0) FL_LN(12, 4);
  else if (per == 4 && cols % 128 == 0) FL_LN(4, 4);
  else if (per == 4) FL_LN(4, 1);
  else if (per == 2) FL_LN(2, 2);
  else if (per == 1) FL_LN(1, 1);
  else done = false;
#undef FL_LN
  if (!done) k_add_ln_generic<T><<<(unsigned)rows, 256, 0, c->stream>>>(x, res, out, g, b, rows, (int)cols, eps);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

int32_t launch_add_layernorm(Ctx* c, int32_t dt, const void* x, const void* res, void* out,
                             const float* g, const float* b, int64_t rows, int64_t cols, float eps) {
  if (dt == FLETCHER_F32) return add_ln_t<float>(c, (const float*)x, (const float*)res, (float*)out, g, b, rows, cols, eps);
  if (dt == FLETCHER_BF16)
    return add_ln_t<__nv_bfloat16>(c, (const __nv_bfloat16*)x, (const __nv_bfloat16*)res, (__nv_bfloat16*)out, g, b, rows, cols, eps);
  return add_ln_t<__half>(c, (const __half*)x, (const __half*)res, (__half*)out, g, b, rows, cols, eps);
}

// ---------------------------------------------------------------- embedding
// bert.go:215-261: word[id] + pos[min(p, P-1)] (absolute only) + type[0], then LayerNorm.
// The adds happen in the reference's order (word + pos, then + type) in fp32.
template <typename T, int PER, int VEC>
__global__ void __launch_bounds__(128) k_embed(const int32_t* __restrict__ ids, const int32_t* __restrict__ pos,
                                               const T* __restrict__ word, const T* __restrict__ ptab, int max_pos,
                                               const T* __restrict__ type0, const float* __restrict__ g,
                                               const float* __restrict__ b, T* __restrict__ out, int64_t rows,
                                               int cols, float eps) {
  pdl_wait();
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* wr = word + (int64_t)ids[row] * cols;
  const T* pr = nullptr;
  if (ptab) {
    int p = pos[row];
    pr = ptab + (int64_t)(p >= max_pos ? max_pos - 1 : p) * cols;
  }
  float v[PER];
#pragma unroll
  for (int j = 0; j < PER / VEC; j++) {
    const int e = (j * 32 + lane) * VEC;
    Vec<T, VEC> a = *reinterpret_cast<const Vec<T, VEC>*>(wr + e);
    Vec<T, VEC> t = *reinterpret_cast<const Vec<T, VEC>*>(type0 + e);
#pragma unroll
    for (int i = 0; i < VEC; i++) v[j * VEC + i] = to_f<T>(a.d[i]);
    if (pr) {
      Vec<T, VEC> p = *reinterpret_cast<const Vec<T, VEC>*>(pr + e);
#pragma unroll
      for (int i = 0; i < VEC; i++) v[j * VEC + i] = __fadd_rn(v[j * VEC + i], to_f<T>(p.d[i]));
    }
#pragma unroll
    for (int i = 0; i < VEC; i++) v[j * VEC + i] = __fadd_rn(v[j * VEC + i], to_f<T>(t.d[i]));
  }
  ln_finish<T, PER, VEC>(v, lane, cols, g, b, eps, out + row * cols);
}

template <typename T>
__global__ void k_embed_sum_generic(const int32_t* ids, const int32_t* pos, const T* word, const T* ptab,
                                    int max_pos, const T* type0, T* out, int64_t rows, int cols) {
  const int64_t row = blockIdx.x;
  const T* wr = word + (int64_t)ids[row] * cols;
  const T* pr = nullptr;
  if (ptab) {
    int p = pos[row];
    pr = ptab + (int64_t)(p >= max_pos ? max_pos - 1 : p) * cols;
  }
  for (int j = threadIdx.x; j < cols; j += blockDim.x) {
    float v = to_f<T>(wr[j]);
    if (pr) v = __fadd_rn(v, to_f<T>(pr[j]));
    out[row * cols + j] = from_f<T>(__fadd_rn(v, to_f<T>(type0[j])));
  }
}

template <typename T>
static int32_t embed_t(Ctx* c, const int32_t* ids, const int32_t* pos, const T* word, const T* ptab, int max_pos,
                       const T* type0, const float* g, const float* b, T* out, int64_t rows, int64_t cols, float eps) {
  if (rows == 0) return FLETCHER_OK;
  const int grid = (int)((rows * 32 + 127) / 128);
  constexpr int V16 = sizeof(T) == 2 ? 8 : 4;
  const int per = (int)(cols / 32);
  bool done = cols % 32 == 0;
#define FL_EM(PER_, VEC_)                                                                                     \
  FL_CUDA(c, launch_pdl(k_embed<T, PER_, VEC_>, dim3(grid), dim3(128), 0, c->stream, ids, pos, word, ptab, max_pos, \
                        type0, g, b, out, rows, (int)cols, eps))
  if (!done) {
  } else if (per == 24 && cols % (32 * V16) == 0) FL_EM(24, V16);
  else if (per == 32 && cols % (32 * V16) == 0) FL_EM(32, V16);
  else if (per == 16 && cols % (32 * V16) == 0) FL_EM(16, V16);
  else if (per == 8 && cols % (32 * V16) == 0) FL_EM(8, V16);
  else if (per == 12 && cols % 128 == 0) FL_EM(12, 4);
  else if (per == 4 && cols % 128 == 0) FL_EM(4, 4);
  else if (per == 4) FL_EM(4, 1);
  else done = false;
#undef FL_EM
  if (!done) {
    k_embed_sum_generic<T><<<(unsigned)rows, 256, 0, c->stream>>>(ids, pos, word, ptab, max_pos, type0, out, rows, (int)cols);
    FL_LAUNCH(c);
    return add_ln_t<T>(c, out, nullptr, out, g, b, rows, cols, eps);
  }
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

int32_t launch_embed(Ctx* c, int32_t dt, const int32_t* ids, const int32_t* pos, const void* word,
                     const void* ptab, int32_t max_pos, const void* type0, const float* g, const float* b,
                     void* out, int64_t T, int64_t H, float eps) {
  if (dt == FLETCHER_F32)
    return embed_t<float>(c, ids, pos, (const float*)word, (const float*)ptab, max_pos, (const float*)type0, g, b, (float*)out, T, H, eps);
  if (dt == FLETCHER_BF16)
    return embed_t<__nv_bfloat16>(c, ids, pos, (const __nv_bfloat16*)word, (const __nv_bfloat16*)ptab, max_pos,
                                  (const __nv_bfloat16*)type0, g, b, (__nv_bfloat16*)out, T, H, eps);
  return embed_t<__half>(c, ids, pos, (const __half*)word, (const __half*)ptab, max_pos, (const __half*)type0, g, b,
                         (__half*)out, T, H, eps);
}

// ---------------------------------------------------------------- positions
__global__ void k_positions(const int32_t* __restrict__ cu, int32_t* __restrict__ pos) {
  pdl_wait();
  const int s = blockIdx.x;
  const int a = cu[s], e = cu[s + 1];
  for (int i = a + threadIdx.x; i < e; i += blockDim.x) pos[i] = i - a;
}

int32_t launch_positions(Ctx* c, const int32_t* cu, int32_t B, int32_t* pos, int32_t) {
  if (B <= 0) return FLETCHER_OK;
  FL_CUDA(c, launch_pdl(k_positions, dim3(B), dim3(256), 0, c->stream, cu, pos));
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

// ---------------------------------------------------------------- mean pool + L2
// One block per sequence.  Threads split into column groups (VEC columns each, 128-bit loads)
// and row groups; each thread keeps four row loads in flight; partial sums meet in shared
// memory, then the L2 norm is a block reduction.
constexpr int kPoolThreads = 512;
template <typename T, int VEC>
__global__ void __launch_bounds__(kPoolThreads) k_mean_pool_l2(const T* __restrict__ h, const int32_t* __restrict__ cu,
                                                      int H, float* __restrict__ out) {
  pdl_wait();
  extern __shared__ float part[];  // [RG][H]
  __shared__ float red[kPoolThreads / 32];
  const int s = blockIdx.x;
  const int a = cu[s], e = cu[s + 1];
  const int CG = H / VEC;
  const bool wide = CG >= (int)blockDim.x;
  const int RG = wide ? 1 : (int)blockDim.x / CG;
  const int rg = wide ? 0 : (int)threadIdx.x / CG;
  if (rg < RG) {
    for (int cg = wide ? (int)threadIdx.x : (int)threadIdx.x % CG; cg < CG; cg += wide ? (int)blockDim.x : CG) {
      float acc[VEC];
#pragma unroll
      for (int i = 0; i < VEC; i++) acc[i] = 0.f;
      int r = a + rg;
      for (; r + 3 * RG < e; r += 4 * RG) {  // four independent row loads in flight
        Vec<T, VEC> x[4];
#pragma unroll
        for (int u = 0; u < 4; u++) x[u] = *reinterpret_cast<const Vec<T, VEC>*>(h + (int64_t)(r + u * RG) * H + cg * VEC);
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
          for (int i = 0; i < VEC; i++) acc[i] += to_f<T>(x[u].d[i]);
      }
      for (; r < e; r += RG) {
        Vec<T, VEC> x = *reinterpret_cast<const Vec<T, VEC>*>(h + (int64_t)r * H + cg * VEC);
#pragma unroll
        for (int i = 0; i < VEC; i++) acc[i] += to_f<T>(x.d[i]);
      }
#pragma unroll
      for (int i = 0; i < VEC; i++) part[rg * H + cg * VEC + i] = acc[i];
    }
  }
  __syncthreads();
  const float invn = e > a ? 1.0f / (float)(e - a) : 0.f;
  float sq = 0.f;
  for (int j = threadIdx.x; j < H; j += blockDim.x) {
    float t = 0.f;
    for (int g = 0; g < RG; g++) t += part[g * H + j];
    t *= invn;
    part[j] = t;  // row group 0 slot now holds the mean (only this thread touches column j)
    sq += t * t;
  }
  sq = warp_sum(sq);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += red[i];
  const float inv = tot > 0.f ? (float)(1.0 / sqrt((double)tot)) : 0.f;
  for (int j = threadIdx.x; j < H; j += blockDim.x) out[(int64_t)s * H + j] = part[j] * inv;
}

template <typename T>
static int32_t mean_pool_t(Ctx* c, const T* h, const int32_t* cu, int B, int64_t H, float* out) {
  constexpr int V = sizeof(T) == 2 ? 8 : 4;
  const bool vec = H % V == 0 && H / V <= kPoolThreads;
  if (B <= 0) return FLETCHER_OK;
  if (vec) {
    const int CG = (int)(H / V);
    const int RG = kPoolThreads / CG;
    FL_CUDA(c, launch_pdl(k_mean_pool_l2<T, V>, dim3(B), dim3(kPoolThreads), (size_t)RG * H * 4, c->stream, h, cu,
                          (int)H, out));
  } else {
    FL_CHECK(c, H <= 8192, "MeanPoolL2: hidden %lld too large", (long long)H);
    FL_CUDA(c, launch_pdl(k_mean_pool_l2<T, 1>, dim3(B), dim3(kPoolThreads),
                          (size_t)(H < kPoolThreads ? kPoolThreads / H : 1) * H * 4, c->stream, h, cu, (int)H, out));
  }
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

int32_t launch_mean_pool_l2(Ctx* c, int32_t dt, const void* h, const int32_t* cu, int32_t B, int64_t H, float* out) {
  if (dt == FLETCHER_F32) return mean_pool_t<float>(c, (const float*)h, cu, B, H, out);
  if (dt == FLETCHER_BF16) return mean_pool_t<__nv_bfloat16>(c, (const __nv_bfloat16*)h, cu, B, H, out);
  return mean_pool_t<__half>(c, (const __half*)h, cu, B, H, out);
}

// ---------------------------------------------------------------- LayerNorm fused into mean pool
// The last layer's LayerNorm and the mean-pool + L2 head in two passes, without writing the
// normalised [T, H] rows: stage 1 takes a chunk of up to kLnPoolRows rows of one sequence (grid:
// chunks x sequences; chunks past a sequence's end exit), normalises each row in registers with
// k_ln_pipe's arithmetic (one warp per row, rounded to the model dtype exactly as k_ln_pipe
// stores it) and writes the chunk's fp32 column sums; stage 2 adds a sequence's
// chunk sums in chunk order, divides by its length and L2-normalises.  Deterministic: the same
// summation order on every run.
constexpr int kLnPoolRows = 64, kLnPoolWarps = 8;

template <typename T, int PER, int VEC>
__global__ void __launch_bounds__(kLnPoolWarps * 32)
    k_ln_pool_partial(const T* __restrict__ x, const int32_t* __restrict__ cu, const float* __restrict__ g,
                      const float* __restrict__ b, float eps, int cols, int chunks, float* __restrict__ partial) {
  pdl_wait();
  extern __shared__ float red[];  // [kLnPoolWarps][cols]
  const int sq = blockIdx.y, ch = blockIdx.x;
  const int a = cu[sq] + ch * kLnPoolRows, e = min(cu[sq + 1], a + kLnPoolRows);
  if (a >= e) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float acc[PER];
#pragma unroll
  for (int i = 0; i < PER; i++) acc[i] = 0.f;
  constexpr int NV = PER / VEC;
  Vec<T, VEC> cur[NV], nxt[NV];
  if (a + warp < e) {
#pragma unroll
    for (int j = 0; j < NV; j++)
      cur[j] = *reinterpret_cast<const Vec<T, VEC>*>(x + (int64_t)(a + warp) * cols + (j * 32 + lane) * VEC);
  }
  for (int r = a + warp; r < e; r += kLnPoolWarps) {
    if (r + kLnPoolWarps < e) {  // the warp's next row loads while this one is normalised
#pragma unroll
      for (int j = 0; j < NV; j++)
        nxt[j] = *reinterpret_cast<const Vec<T, VEC>*>(x + (int64_t)(r + kLnPoolWarps) * cols + (j * 32 + lane) * VEC);
    }
    float v[PER];
#pragma unroll
    for (int j = 0; j < NV; j++) {
#pragma unroll
      for (int i = 0; i < VEC; i++) v[j * VEC + i] = to_f<T>(cur[j].d[i]);
      cur[j] = nxt[j];
    }
    ln_row_x2<PER, VEC>(v, lane, cols, g, b, eps);  // the same arithmetic as k_ln_pipe
#pragma unroll
    for (int i = 0; i < PER; i++) acc[i] += to_f<T>(from_f<T>(v[i]));  // rounded as the stored rows would be
  }
#pragma unroll
  for (int j = 0; j < PER / VEC; j++)
#pragma unroll
    for (int i = 0; i < VEC; i++) red[warp * cols + (j * 32 + lane) * VEC + i] = acc[j * VEC + i];
  __syncthreads();
  float* dst = partial + ((int64_t)sq * chunks + ch) * cols;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kLnPoolWarps; w++) t += red[w * cols + c];
    dst[c] = t;
  }
}

__global__ void __launch_bounds__(256) k_ln_pool_finish(const float* __restrict__ partial, const int32_t* __restrict__ cu,
                                                        int cols, int chunks, float* __restrict__ out) {
  pdl_wait();
  extern __shared__ float mean[];  // [cols]
  __shared__ float red[8];
  const int sq = blockIdx.x;
  const int len = cu[sq + 1] - cu[sq];
  const int nch = (len + kLnPoolRows - 1) / kLnPoolRows;
  const float invn = len > 0 ? 1.0f / (float)len : 0.f;
  float ss = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float t = 0.f;
    for (int k = 0; k < nch; k++) t += partial[((int64_t)sq * chunks + k) * cols + c];
    t *= invn;
    mean[c] = t;
    ss += t * t;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += red[i];
  const float inv = tot > 0.f ? (float)(1.0 / sqrt((double)tot)) : 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) out[(int64_t)sq * cols + c] = mean[c] * inv;
}

bool ln_pool_supported(int32_t dt, int64_t H) { return dt != FLETCHER_F32 && (H == 768 || H == 1024 || H == 512 || H == 256); }

int64_t ln_pool_workspace_bytes(int32_t B, int32_t max_len, int64_t H) {
  return (int64_t)B * ((max_len + kLnPoolRows - 1) / kLnPoolRows) * H * 4;
}

template <typename T>
static int32_t ln_pool_t(Ctx* c, const T* x, const int32_t* cu, const float* g, const float* b, float eps, int32_t B,
                         int32_t max_len, int64_t H, float* ws, float* out) {
  constexpr int V = 8;  // 16-bit rows: 128-bit loads
  const int chunks = (max_len + kLnPoolRows - 1) / kLnPoolRows;
  const dim3 grid((unsigned)chunks, (unsigned)B);
  const size_t smem = (size_t)kLnPoolWarps * H * 4;
#define FL_LNP(PER_)                                                                                                 \
  FL_CUDA(c, launch_pdl(k_ln_pool_partial<T, PER_, V>, grid, dim3(kLnPoolWarps * 32), smem, c->stream, x, cu, g, b, eps, \
                        (int)H, chunks, ws))
  if (H == 768) FL_LNP(24);
  else if (H == 1024) FL_LNP(32);
  else if (H == 512) FL_LNP(16);
  else FL_LNP(8);
#undef FL_LNP
  FL_LAUNCH(c);
  FL_CUDA(c, launch_pdl(k_ln_pool_finish, dim3((unsigned)B), dim3(256), (size_t)H * 4, c->stream, (const float*)ws, cu,
                        (int)H, chunks, out));
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

int32_t launch_ln_mean_pool_l2(Ctx* c, int32_t dt, const void* x, const int32_t* cu, const float* g, const float* b,
                               float eps, int32_t B, int32_t max_len, int64_t H, float* ws, float* out) {
  FL_CHECK(c, ln_pool_supported(dt, H), "ln_mean_pool: unsupported dtype/width");
  if (B <= 0) return FLETCHER_OK;
  if (dt == FLETCHER_BF16)
    return ln_pool_t<__nv_bfloat16>(c, (const __nv_bfloat16*)x, cu, g, b, eps, B, max_len, H, ws, out);
  return ln_pool_t<__half>(c, (const __half*)x, cu, g, b, eps, B, max_len, H, ws, out);
}

// ---------------------------------------------------------------- gather rows -> f32
template <typename T>
__global__ void k_gather_rows_f32(const T* __restrict__ src, const int32_t* __restrict__ idx, int64_t H,
                                  float* __restrict__ dst) {
  const int64_t i = blockIdx.x;
  const T* s = src + (int64_t)idx[i] * H;
  for (int64_t j = threadIdx.x; j < H; j += blockDim.x) dst[i * H + j] = to_f<T>(s[j]);
}

int32_t launch_gather_rows_f32(Ctx* c, int32_t dt, const void* src, const int32_t* idx, int64_t n, int64_t H, float* dst) {
  if (n <= 0) return FLETCHER_OK;
  if (dt == FLETCHER_F32) k_gather_rows_f32<float><<<(unsigned)n, 256, 0, c->stream>>>((const float*)src, idx, H, dst);
  else if (dt == FLETCHER_BF16) k_gather_rows_f32<__nv_bfloat16><<<(unsigned)n, 256, 0, c->stream>>>((const __nv_bfloat16*)src, idx, H, dst);
  else k_gather_rows_f32<__half><<<(unsigned)n, 256, 0, c->stream>>>((const __half*)src, idx, H, dst);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

// ---------------------------------------------------------------- RoPE
// cpu_backend.go:789-798: theta = pos * base^(-2i/dh) in float64, cos/sin rounded to float32,
// then (x1, x2) <- (x1*c - x2*s, x1*s + x2*c) in float32.
__global__ void k_rope_table(float* cos_t, float* sin_t, int len, int half, int dh, double base) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)len * half) return;
  const int p = (int)(i / half), k = (int)(i % half);
  const double theta = (double)p * pow(base, -2.0 * (double)k / (double)dh);
  cos_t[i] = (float)cos(theta);
  sin_t[i] = (float)sin(theta);
}

int32_t launch_rope_build_table(Ctx* c, float* cos_t, float* sin_t, int32_t len, int32_t dh, double base) {
  const int64_t n = (int64_t)len * (dh / 2);
  k_rope_table<<<(unsigned)((n + 255) / 256), 256, 0, c->stream>>>(cos_t, sin_t, len, dh / 2, dh, base);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

template <typename T>
__global__ void k_rope_apply(T* x, int64_t T_, int64_t ld, int64_t ncols, int dh, const int32_t* __restrict__ pos,
                             const float* __restrict__ ct, const float* __restrict__ st) {
  const int half = dh / 2;
  const int64_t per_row = ncols / 2;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= T_ * per_row) return;
  const int64_t r = i / per_row;
  const int64_t q = i % per_row;
  const int64_t head = q / half;
  const int k = (int)(q % half);
  T* p = x + r * ld + head * dh;
  const float cs = ct[(int64_t)pos[r] * half + k], sn = st[(int64_t)pos[r] * half + k];
  const float x1 = to_f<T>(p[k]), x2 = to_f<T>(p[k + half]);
  p[k] = from_f<T>(__fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn)));
  p[k + half] = from_f<T>(__fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs)));
}

int32_t launch_rope_table(Ctx* c, int32_t dt, void* x, int64_t T, int64_t ld, int64_t ncols, int32_t dh,
                          const int32_t* pos, const float* ct, const float* st) {
  const int64_t n = T * (ncols / 2);
  if (n <= 0) return FLETCHER_OK;
  const unsigned g = (unsigned)((n + 255) / 256);
  if (dt == FLETCHER_F32) k_rope_apply<float><<<g, 256, 0, c->stream>>>((float*)x, T, ld, ncols, dh, pos, ct, st);
  else if (dt == FLETCHER_BF16) k_rope_apply<__nv_bfloat16><<<g, 256, 0, c->stream>>>((__nv_bfloat16*)x, T, ld, ncols, dh, pos, ct, st);
  else k_rope_apply<__half><<<g, 256, 0, c->stream>>>((__half*)x, T, ld, ncols, dh, pos, ct, st);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

// ---------------------------------------------------------------- SwiGLU (cpu_backend.go:636-654)
template <typename T>
__global__ void k_swiglu(const T* __restrict__ in, T* __restrict__ out, int64_t rows, int64_t I) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * I; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / I, j = i % I;
    out[i] = from_f<T>(swiglu_exact(to_f<T>(in[r * 2 * I + j]), to_f<T>(in[r * 2 * I + j + I])));
  }
}

int32_t launch_swiglu(Ctx* c, int32_t dt, const void* in, void* out, int64_t rows, int64_t I) {
  const int g = grid_for(rows * I, 256);
  if (dt == FLETCHER_F32) k_swiglu<float><<<g, 256, 0, c->stream>>>((const float*)in, (float*)out, rows, I);
  else if (dt == FLETCHER_BF16) k_swiglu<__nv_bfloat16><<<g, 256, 0, c->stream>>>((const __nv_bfloat16*)in, (__nv_bfloat16*)out, rows, I);
  else k_swiglu<__half><<<g, 256, 0, c->stream>>>((const __half*)in, (__half*)out, rows, I);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

// ---------------------------------------------------------------- elementwise
template <typename T>
__global__ void k_scale_add(T* x, const T* other, float scale, float add, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = to_f<T>(x[i]);
    if (scale != 1.0f) v = __fmul_rn(v, scale);
    if (add != 0.0f) v = __fadd_rn(v, add);
    if (other) v = __fadd_rn(v, to_f<T>(other[i]));
    x[i] = from_f<T>(v);
  }
}
int32_t launch_scale_add(Ctx* c, int32_t dt, void* x, const void* other, float scale, float add, int64_t n) {
  const int g = grid_for(n, 256);
  if (n <= 0) return FLETCHER_OK;
  if (dt == FLETCHER_F32) k_scale_add<float><<<g, 256, 0, c->stream>>>((float*)x, (const float*)other, scale, add, n);
  else if (dt == FLETCHER_BF16) k_scale_add<__nv_bfloat16><<<g, 256, 0, c->stream>>>((__nv_bfloat16*)x, (const __nv_bfloat16*)other, scale, add, n);
  else k_scale_add<__half><<<g, 256, 0, c->stream>>>((__half*)x, (const __half*)other, scale, add, n);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

template <typename T>
__global__ void k_add_bias(T* x, const T* b, int64_t rows, int64_t cols) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * cols; i += (int64_t)gridDim.x * blockDim.x)
    x[i] = from_f<T>(__fadd_rn(to_f<T>(x[i]), to_f<T>(b[i % cols])));
}
int32_t launch_add_bias(Ctx* c, int32_t dt, void* x, const void* b, int64_t rows, int64_t cols) {
  const int g = grid_for(rows * cols, 256);
  if (rows * cols <= 0) return FLETCHER_OK;
  if (dt == FLETCHER_F32) k_add_bias<float><<<g, 256, 0, c->stream>>>((float*)x, (const float*)b, rows, cols);
  else if (dt == FLETCHER_BF16) k_add_bias<__nv_bfloat16><<<g, 256, 0, c->stream>>>((__nv_bfloat16*)x, (const __nv_bfloat16*)b, rows, cols);
  else k_add_bias<__half><<<g, 256, 0, c->stream>>>((__half*)x, (const __half*)b, rows, cols);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

// Softmax rows (SoftmaxFast, simd.go:78-99), one warp per row.
template <typename T>
__global__ void k_softmax_rows(T* x, int64_t rows, int64_t cols) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  T* r = x + row * cols;
  float m = -INFINITY;
  for (int64_t j = lane; j < cols; j += 32) m = fmaxf(m, to_f<T>(r[j]));
  m = warp_max(m);
  float s = 0.f;
  for (int64_t j = lane; j < cols; j += 32) s += exp_fast(__fsub_rn(to_f<T>(r[j]), m));
  s = warp_sum(s);
  const float inv = __fdiv_rn(1.0f, s);
  for (int64_t j = lane; j < cols; j += 32) r[j] = from_f<T>(__fmul_rn(exp_fast(__fsub_rn(to_f<T>(r[j]), m)), inv));
}

template <typename T>
__global__ void k_act(T* x, int64_t n, int32_t act) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = to_f<T>(x[i]);
    v = act == FLETCHER_ACT_GELU ? gelu_fast(v) : act == FLETCHER_ACT_TANH ? tanh_fast(v) : v;
    x[i] = from_f<T>(v);
  }
}

int32_t launch_activation(Ctx* c, int32_t dt, void* x, int64_t rows, int64_t cols, int32_t act) {
  if (rows * cols <= 0 || act == FLETCHER_ACT_IDENTITY) return FLETCHER_OK;
  if (act == FLETCHER_ACT_SOFTMAX) {
    const unsigned g = (unsigned)((rows * 32 + 255) / 256);
    if (dt == FLETCHER_F32) k_softmax_rows<float><<<g, 256, 0, c->stream>>>((float*)x, rows, cols);
    else if (dt == FLETCHER_BF16) k_softmax_rows<__nv_bfloat16><<<g, 256, 0, c->stream>>>((__nv_bfloat16*)x, rows, cols);
    else k_softmax_rows<__half><<<g, 256, 0, c->stream>>>((__half*)x, rows, cols);
  } else {
    FL_CHECK(c, act == FLETCHER_ACT_GELU || act == FLETCHER_ACT_TANH, "Activation: unsupported code %d", act);
    const int g = grid_for(rows * cols, 256);
    if (dt == FLETCHER_F32) k_act<float><<<g, 256, 0, c->stream>>>((float*)x, rows * cols, act);
    else if (dt == FLETCHER_BF16) k_act<__nv_bfloat16><<<g, 256, 0, c->stream>>>((__nv_bfloat16*)x, rows * cols, act);
    else k_act<__half><<<g, 256, 0, c->stream>>>((__half*)x, rows * cols, act);
  }
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

template <typename T>
__global__ void k_has_nan(const T* x, int64_t n, int32_t* flag) {
  bool bad = false;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    bad |= !isfinite(to_f<T>(x[i]));
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flag, 1);
}
int32_t launch_has_nan(Ctx* c, int32_t dt, const void* x, int64_t n, int32_t* flag) {
  if (n <= 0) return FLETCHER_OK;
  const int g = grid_for(n, 256, 4 * c->num_sms);
  if (dt == FLETCHER_F32) k_has_nan<float><<<g, 256, 0, c->stream>>>((const float*)x, n, flag);
  else if (dt == FLETCHER_BF16) k_has_nan<__nv_bfloat16><<<g, 256, 0, c->stream>>>((const __nv_bfloat16*)x, n, flag);
  else k_has_nan<__half><<<g, 256, 0, c->stream>>>((const __half*)x, n, flag);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

// ref: fp16 on either side uses the reference's conversion (utils.go:13-91) instead of IEEE
// round-to-nearest-even; the ABI's Cast and the model's fp16 output transport pass the
// context's mode, internal casts pass false.
template <typename S, typename D>
__global__ void k_cast(const S* s, D* d, int64_t n, bool ref) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    d[i] = from_f_host<D>(to_f_host<S>(s[i], ref), ref);
}
template <typename S>
static void cast_to(Ctx* c, const S* s, int32_t ddt, void* d, int64_t n, int g, bool ref) {
  if (ddt == FLETCHER_F32) k_cast<S, float><<<g, 256, 0, c->stream>>>(s, (float*)d, n, ref);
  else if (ddt == FLETCHER_BF16) k_cast<S, __nv_bfloat16><<<g, 256, 0, c->stream>>>(s, (__nv_bfloat16*)d, n, ref);
  else k_cast<S, __half><<<g, 256, 0, c->stream>>>(s, (__half*)d, n, ref);
}
int32_t launch_cast(Ctx* c, int32_t sdt, const void* s, int32_t ddt, void* d, int64_t n, bool ref) {
  if (n <= 0) return FLETCHER_OK;
  const int g = grid_for(n, 256);
  if (sdt == FLETCHER_F32) cast_to<float>(c, (const float*)s, ddt, d, n, g, ref);
  else if (sdt == FLETCHER_BF16) cast_to<__nv_bfloat16>(c, (const __nv_bfloat16*)s, ddt, d, n, g, ref);
  else cast_to<__half>(c, (const __half*)s, ddt, d, n, g, ref);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

// ---------------------------------------------------------------- weight packing
// dst[n', k] = src[k, col(n')]: (in,out) fp32 -> K-major 16-bit for the tensor-core GEMM.
// perm 1 interleaves a SwiGLU [gate | up] weight so that every block_n-row tile holds
// block_n/2 gate rows followed by the matching block_n/2 up rows.
__device__ __forceinline__ int64_t packed_src_col(int64_t n, int64_t N, int perm, int block_n) {
  if (perm == 0) return n;
  const int64_t half = block_n / 2, I = N / 2;
  const int64_t j = n / block_n, r = n % block_n;
  return r < half ? j * half + r : I + j * half + (r - half);
}

template <typename S, typename T>
__global__ void k_pack_kmajor(const S* __restrict__ src, int64_t K, int64_t N, T* __restrict__ dst, int perm,
                              int block_n, bool ref = false) {
  __shared__ float tile[32][33];
  const int64_t k0 = (int64_t)blockIdx.x * 32, n0 = (int64_t)blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t k = k0 + i, n = n0 + threadIdx.x;
    tile[i][threadIdx.x] = (k < K && n < N) ? to_f<S>(src[k * N + packed_src_col(n, N, perm, block_n)]) : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t n = n0 + i, k = k0 + threadIdx.x;
    if (n < N && k < K) dst[n * K + k] = from_f_host<T>(tile[threadIdx.x][i], ref);
  }
}

int32_t launch_pack_weight_kmajor(Ctx* c, const float* src, int64_t K, int64_t N, void* dst, int32_t dt,
                                  int32_t perm, int32_t block_n) {
  dim3 grid((unsigned)((K + 31) / 32), (unsigned)((N + 31) / 32)), blk(32, 8);
  if (dt == FLETCHER_BF16) k_pack_kmajor<float, __nv_bfloat16><<<grid, blk, 0, c->stream>>>(src, K, N, (__nv_bfloat16*)dst, perm, block_n);
  else if (dt == FLETCHER_F16)  // fp32 host weights -> fp16 as the reference's CopyFromFloat32 converts them
    k_pack_kmajor<float, __half><<<grid, blk, 0, c->stream>>>(src, K, N, (__half*)dst, perm, block_n,
                                                              c->half_mode == FLETCHER_HALF_REFERENCE);
  else k_pack_kmajor<float, float><<<grid, blk, 0, c->stream>>>(src, K, N, (float*)dst, perm, block_n);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

// Places one (in,out) [K, N] Linear weight, given as stored in a checkpoint (src_t: (out,in)
// [N, K], the SafeTensors / PyTorch layout) in any dtype, into a model weight buffer of another
// dtype: K-major rows [row_off + n', K] with the SwiGLU interleave applied to n (dst_kmajor),
// or (in,out) columns [K, ld] at col_off (fp32 models).  A 32x32 tile is transposed through
// shared memory when the source and destination layouts disagree, so both sides stay coalesced.
__device__ __forceinline__ int64_t packed_dst_row(int64_t n, int64_t N, int perm, int block_n) {
  if (perm == 0) return n;
  const int64_t half = block_n / 2, I = N / 2;
  const int64_t u = n < I ? n : n - I;
  return (u / half) * block_n + (n < I ? 0 : half) + u % half;
}

template <typename S, typename D>
__global__ void k_place_weight(const S* __restrict__ src, int64_t K, int64_t N, int src_t, D* __restrict__ dst,
                               int dst_kmajor, int64_t ld, int64_t off, int perm, int block_n, bool ref) {
  __shared__ float tile[32][33];
  const int64_t k0 = (int64_t)blockIdx.x * 32, n0 = (int64_t)blockIdx.y * 32;
  // Load: lanes run along the source's contiguous index.
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t k = src_t ? k0 + threadIdx.x : k0 + i, n = src_t ? n0 + i : n0 + threadIdx.x;
    float v = 0.f;
    if (k < K && n < N) v = to_f<S>(src_t ? src[n * K + k] : src[k * N + n]);
    if (src_t) tile[i][threadIdx.x] = v;  // tile[n][k]
    else tile[threadIdx.x][i] = v;        // tile[n][k]
  }
  __syncthreads();
  // Store: lanes run along the destination's contiguous index.
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    if (dst_kmajor) {
      const int64_t n = n0 + i, k = k0 + threadIdx.x;
      if (n < N && k < K) dst[(off + packed_dst_row(n, N, perm, block_n)) * K + k] = from_f_host<D>(tile[i][threadIdx.x], ref);
    } else {
      const int64_t k = k0 + i, n = n0 + threadIdx.x;
      if (n < N && k < K) dst[k * ld + off + n] = from_f_host<D>(tile[threadIdx.x][i], ref);
    }
  }
}

template <typename S>
static void place_from(Ctx* c, dim3 g, dim3 b, const S* src, int64_t K, int64_t N, int src_t, int32_t ddt, void* dst,
                       int dst_kmajor, int64_t ld, int64_t off, int perm, int block_n, bool ref) {
  if (ddt == FLETCHER_F32)
    k_place_weight<S, float><<<g, b, 0, c->stream>>>(src, K, N, src_t, (float*)dst, dst_kmajor, ld, off, perm, block_n, ref);
  else if (ddt == FLETCHER_BF16)
    k_place_weight<S, __nv_bfloat16><<<g, b, 0, c->stream>>>(src, K, N, src_t, (__nv_bfloat16*)dst, dst_kmajor, ld, off,
                                                             perm, block_n, ref);
  else
    k_place_weight<S, __half><<<g, b, 0, c->stream>>>(src, K, N, src_t, (__half*)dst, dst_kmajor, ld, off, perm, block_n,
                                                      ref);
}

int32_t launch_place_weight(Ctx* c, int32_t sdt, const void* src, int64_t K, int64_t N, int src_t, int32_t ddt,
                            void* dst, int dst_kmajor, int64_t ld, int64_t off, int perm, int block_n) {
  if (K <= 0 || N <= 0) return FLETCHER_OK;
  // fp32 checkpoint values become fp16 as the reference's CopyFromFloat32 converts them.
  const bool ref = sdt == FLETCHER_F32 && c->half_mode == FLETCHER_HALF_REFERENCE;
  dim3 grid((unsigned)((K + 31) / 32), (unsigned)((N + 31) / 32)), blk(32, 8);
  if (sdt == FLETCHER_F32)
    place_from<float>(c, grid, blk, (const float*)src, K, N, src_t, ddt, dst, dst_kmajor, ld, off, perm, block_n, ref);
  else if (sdt == FLETCHER_BF16)
    place_from<__nv_bfloat16>(c, grid, blk, (const __nv_bfloat16*)src, K, N, src_t, ddt, dst, dst_kmajor, ld, off, perm,
                              block_n, ref);
  else
    place_from<__half>(c, grid, blk, (const __half*)src, K, N, src_t, ddt, dst, dst_kmajor, ld, off, perm, block_n, ref);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

int32_t launch_pack_kmajor_16(Ctx* c, int32_t dt, const void* src, int64_t K, int64_t N, void* dst, int32_t perm,
                              int32_t block_n) {
  dim3 grid((unsigned)((K + 31) / 32), (unsigned)((N + 31) / 32)), blk(32, 8);
  if (dt == FLETCHER_BF16)
    k_pack_kmajor<__nv_bfloat16, __nv_bfloat16><<<grid, blk, 0, c->stream>>>((const __nv_bfloat16*)src, K, N, (__nv_bfloat16*)dst, perm, block_n);
  else
    k_pack_kmajor<__half, __half><<<grid, blk, 0, c->stream>>>((const __half*)src, K, N, (__half*)dst, perm, block_n);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

}  // namespace fl
