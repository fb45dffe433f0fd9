// Bidirectional multi-head attention over packed variable-length sequences.
//
// Reference: BertSelfAttention.ForwardBatch (bert.go:610-728) -> CPUTensor.Attention
// (cpu_backend.go:662-758): per sequence, per head, P = SoftmaxFast(scale * Q_h K_h^T),
// O_h = P V_h.  Sequences are described by cu_seqlens (prefix sums of the lengths); keys past
// a sequence's end are masked, so packing replaces padding.
//
// Two kernels:
//  - k_attn_f32: fp32 parity mode.  One CTA per (query row, head); scores in shared memory,
//    the reference's ExpFast softmax (max, ExpFast(s-max), sum, * 1/sum) then P.V.
//  - k_flash_attn: bf16/f16 mode.  Flash-style: 64-row query tile per CTA (16 rows per warp),
//    64-key K/V blocks double-buffered through cp.async into XOR-swizzled shared memory,
//    QK^T and PV on mma.sync m16n8k16 with fp32 accumulators, online softmax with exp2.
//    Head dim 64.  Query tiles come from a host-built list, longest sequences first.
#include "kernels.cuh"

namespace fl {

// ---------------------------------------------------------------- fp32 parity kernel
__device__ __forceinline__ int find_seq(const int32_t* cu, int B, int64_t row) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= row) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(128) k_attn_f32(const float* __restrict__ q, const float* __restrict__ k,
                                                  const float* __restrict__ v, int64_t ld_in, float* __restrict__ out,
                                                  int64_t ld_out, const int32_t* __restrict__ cu, int B, int dh,
                                                  float scale) {
  extern __shared__ float sh[];  // [dh] q, [max_len] scores, [128] reduction scratch
  __shared__ float red[4];
  const int64_t row = blockIdx.x;
  const int h = blockIdx.y;
  const int s = find_seq(cu, B, row);
  const int a = cu[s], L = cu[s + 1] - a;
  float* qs = sh;
  float* sc = sh + dh;
  float* part = sc + L;
  const int tid = threadIdx.x;
  for (int d = tid; d < dh; d += blockDim.x) qs[d] = q[row * ld_in + (int64_t)h * dh + d];
  __syncthreads();
  float mx = -INFINITY;
  for (int j = tid; j < L; j += blockDim.x) {
    const float* kr = k + (int64_t)(a + j) * ld_in + (int64_t)h * dh;
    float dot = 0.f;
    for (int d = 0; d < dh; d++) dot = fmaf(qs[d], kr[d], dot);
    const float sv = __fmul_rn(scale, dot);  // sgemm with alpha = scale
    sc[j] = sv;
    mx = fmaxf(mx, sv);
  }
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  float sum = 0.f;
  for (int j = tid; j < L; j += blockDim.x) {
    const float e = exp_fast(__fsub_rn(sc[j], mx));
    sc[j] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if ((tid & 31) == 0) red[tid >> 5] = sum;
  __syncthreads();
  sum = (red[0] + red[1]) + (red[2] + red[3]);
  const float inv = __fdiv_rn(1.0f, sum);
  for (int j = tid; j < L; j += blockDim.x) sc[j] = __fmul_rn(sc[j], inv);
  __syncthreads();
  // O = P V: thread (d, g) accumulates keys j = g, g+G, ...
  const int G = blockDim.x / dh > 0 ? blockDim.x / dh : 1;
  for (int d0 = 0; d0 < dh; d0 += blockDim.x) {
    const int d = d0 + (tid % (dh < (int)blockDim.x ? dh : blockDim.x));
    const int g = dh < (int)blockDim.x ? tid / dh : 0;
    float acc = 0.f;
    if (g < G && d < dh)
      for (int j = g; j < L; j += G) acc = fmaf(sc[j], v[(int64_t)(a + j) * ld_in + (int64_t)h * dh + d], acc);
    if (g < G && d < dh) part[g * dh + (d - d0)] = acc;
    __syncthreads();
    if (tid < dh && d0 + tid < dh) {
      float t = 0.f;
      for (int gg = 0; gg < G; gg++) t += part[gg * dh + tid];
      out[row * ld_out + (int64_t)h * dh + d0 + tid] = t;
    }
    __syncthreads();
  }
}

int32_t launch_attention_f32(Ctx* c, const float* q, const float* k, const float* v, int64_t ld_in, float* out,
                             int64_t ld_out, const int32_t* cu, int32_t B, int64_t T, int32_t nh, int32_t dh,
                             float scale, int32_t max_len) {
  if (T <= 0) return FLETCHER_OK;
  const int G = 128 / dh > 0 ? 128 / dh : 1;
  const size_t smem = (size_t)(dh + max_len + G * (dh < 128 ? dh : 128)) * 4;
  FL_CHECK(c, smem <= 200 * 1024, "attention_f32: sequence length %d too long for the fp32 kernel", max_len);
  if (smem > 48 * 1024) FL_CUDA(c, cudaFuncSetAttribute(k_attn_f32, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((unsigned)T, (unsigned)nh);
  k_attn_f32<<<grid, 128, smem, c->stream>>>(q, k, v, ld_in, out, ld_out, cu, B, dh, scale);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

// ---------------------------------------------------------------- bf16/f16 flash kernel
namespace {
constexpr int FQ = 64, FK = 64, FD = 64;

__device__ __forceinline__ uint32_t s_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
// Element offset of 16-byte chunk `ch` (0..7) of row r in a 64-wide swizzled tile.
__device__ __forceinline__ int swz(int r, int ch) { return r * 64 + ((ch ^ (r & 7)) << 3); }

__device__ __forceinline__ void cp16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s_u32(p)));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float x, float y) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <typename T>
__device__ __forceinline__ void load_tile(T* s, const T* base, int64_t ld, int row0, int nrows_valid, int tid) {
  // 64 rows x 8 chunks of 16 B; 128 threads x 4 chunks.
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int idx = tid + i * 128;
    const int r = idx >> 3, ch = idx & 7;
    const bool ok = r < nrows_valid;
    const T* src = base + (int64_t)(row0 + (ok ? r : 0)) * ld + ch * 8;
    cp16(s + swz(r, ch), src, ok);
  }
}
}  // namespace

template <typename T>
__global__ void __launch_bounds__(128) k_flash_attn(const T* __restrict__ Q, const T* __restrict__ K,
                                                    const T* __restrict__ V, int64_t ld_in, T* __restrict__ O,
                                                    int64_t ld_out, const int32_t* __restrict__ cu,
                                                    const int2* __restrict__ tiles, float scale_log2) {
  __shared__ __align__(128) T sQ[FQ * FD];
  __shared__ __align__(128) T sK[2][FK * FD];
  __shared__ __align__(128) T sV[2][FK * FD];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int2 tile = tiles[blockIdx.x];
  const int h = blockIdx.y;
  const int a = cu[tile.x], L = cu[tile.x + 1] - a;
  const int q0 = tile.y;
  const T* qb = Q + (int64_t)a * ld_in + h * FD;
  const T* kb = K + (int64_t)a * ld_in + h * FD;
  const T* vb = V + (int64_t)a * ld_in + h * FD;
  const int nkb = (L + FK - 1) / FK;

  load_tile(sQ, qb, ld_in, q0, L - q0, tid);
  load_tile(sK[0], kb, ld_in, 0, L, tid);
  load_tile(sV[0], vb, ld_in, 0, L, tid);
  cp_commit();

  uint32_t qf[4][4];
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int g = lane >> 2, t = lane & 3;

  for (int j = 0; j < nkb; j++) {
    const int buf = j & 1;
    if (j + 1 < nkb) {
      load_tile(sK[buf ^ 1], kb, ld_in, (j + 1) * FK, L - (j + 1) * FK, tid);
      load_tile(sV[buf ^ 1], vb, ld_in, (j + 1) * FK, L - (j + 1) * FK, tid);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; kk++) ldsm_x4(qf[kk], sQ + swz(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)));
    }
    // S = Q K^T for this warp's 16 rows x 64 keys.
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; np++) {
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        uint32_t r[4];
        ldsm_x4(r, sK[buf] + swz(np * 16 + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1)));
        mma16816<T>(s[2 * np], qf[kk], r[0], r[1]);
        mma16816<T>(s[2 * np + 1], qf[kk], r[2], r[3]);
      }
    }
    // Mask keys past the end of the sequence.
    const int kbase = j * FK;
    if (kbase + FK > L) {
#pragma unroll
      for (int nt = 0; nt < 8; nt++) {
        const int c0 = kbase + nt * 8 + 2 * t;
        if (c0 >= L) s[nt][0] = s[nt][2] = -INFINITY;
        if (c0 + 1 >= L) s[nt][1] = s[nt][3] = -INFINITY;
      }
    }
    // Online softmax (rows g and g+8 of the warp's 16).
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float al0 = exp2f((m0 - mx0) * scale_log2), al1 = exp2f((m1 - mx1) * scale_log2);
    m0 = mx0;
    m1 = mx1;
    const float ms0 = mx0 * scale_log2, ms1 = mx1 * scale_log2;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
      s[nt][0] = exp2f(fmaf(s[nt][0], scale_log2, -ms0));
      s[nt][1] = exp2f(fmaf(s[nt][1], scale_log2, -ms0));
      s[nt][2] = exp2f(fmaf(s[nt][2], scale_log2, -ms1));
      s[nt][3] = exp2f(fmaf(s[nt][3], scale_log2, -ms1));
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
      o[nt][0] *= al0;
      o[nt][1] *= al0;
      o[nt][2] *= al1;
      o[nt][3] *= al1;
    }
    // O += P V.
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      uint32_t pa[4];
      pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 4; dp++) {
        uint32_t r[4];
        ldsm_x4_t(r, sV[buf] + swz(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), dp * 2 + (lane >> 4)));
        mma16816<T>(o[2 * dp], pa, r[0], r[1]);
        mma16816<T>(o[2 * dp + 1], pa, r[2], r[3]);
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = 1.0f / l0, i1 = 1.0f / l1;
  const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int nt = 0; nt < 8; nt++) {
    const int col = h * FD + nt * 8 + 2 * t;
    if (r0 < L) *reinterpret_cast<uint32_t*>(O + (int64_t)(a + r0) * ld_out + col) = pack2<T>(o[nt][0] * i0, o[nt][1] * i0);
    if (r1 < L) *reinterpret_cast<uint32_t*>(O + (int64_t)(a + r1) * ld_out + col) = pack2<T>(o[nt][2] * i1, o[nt][3] * i1);
  }
}

int32_t launch_flash_attention_ld(Ctx* c, int32_t dt, const void* q, const void* k, const void* v, int64_t ld_in,
                                  void* out, int64_t ld_out, const int32_t* cu, const int2* tiles, int32_t num_tiles,
                                  int32_t nh, float scale) {
  if (num_tiles <= 0) return FLETCHER_OK;
  FL_CHECK(c, ld_in % 8 == 0 && ld_out % 8 == 0 && ((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 &&
                  ((uintptr_t)v & 15) == 0,
           "flash_attention: q/k/v rows must be 16-byte aligned");
  dim3 grid((unsigned)num_tiles, (unsigned)nh);
  const float sl2 = scale * 1.4426950408889634f;
  if (dt == FLETCHER_BF16)
    k_flash_attn<__nv_bfloat16><<<grid, 128, 0, c->stream>>>((const __nv_bfloat16*)q, (const __nv_bfloat16*)k,
                                                              (const __nv_bfloat16*)v, ld_in, (__nv_bfloat16*)out,
                                                              ld_out, cu, tiles, sl2);
  else
    k_flash_attn<__half><<<grid, 128, 0, c->stream>>>((const __half*)q, (const __half*)k, (const __half*)v, ld_in,
                                                       (__half*)out, ld_out, cu, tiles, sl2);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

}  // namespace fl
