// SIMT GEMM (fp32 FFMA): the fp32 parity path of Linear (cpu_backend.go:612-624 -> sgemm), and
// the fallback for 16-bit shapes the tensor-core kernel does not take.  128x128 CTA tile,
// 8-deep K slices, 8x8 outputs per thread, bias + activation fused in the epilogue.
// Results equal OpenBLAS sgemm up to summation order.
#include "gemm.cuh"

namespace fl {

namespace {
constexpr int TM = 128, TN = 128, TK = 8;

// A(m, k) = A[m*sam + k*sak] and B(k, n) = B[k*sbk + n*sbn]: unit inner strides for the
// row-major Linear, swapped ones for Mul's transposed views.
template <typename T>
__global__ void __launch_bounds__(256) k_sgemm(const T* __restrict__ A, int64_t sam, int64_t sak,
                                               const T* __restrict__ B, int64_t sbk, int64_t sbn, T* __restrict__ C,
                                               int64_t ldc, int64_t M, int64_t N, int64_t K,
                                               const T* __restrict__ bias, int act) {
  __shared__ __align__(16) float As[TK][TM];
  __shared__ __align__(16) float Bs[TK][TN];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t m0 = (int64_t)blockIdx.y * TM, n0 = (int64_t)blockIdx.x * TN;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

  for (int64_t k0 = 0; k0 < K; k0 += TK) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int idx = tid * 4 + i;
      const int r = idx / TK, cc = idx % TK;
      const int64_t gm = m0 + r, gk = k0 + cc;
      As[cc][r] = (gm < M && gk < K) ? to_f<T>(A[gm * sam + gk * sak]) : 0.f;
      const int br = idx / TN, bc = idx % TN;
      const int64_t bk = k0 + br, bn = n0 + bc;
      Bs[br][bc] = (bk < K && bn < N) ? to_f<T>(B[bk * sbk + bn * sbn]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; kk++) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ty * 4 + 64]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4 + 64]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int64_t gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int64_t gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (gn >= N) continue;
      float v = acc[i][j];
      if (bias) v = __fadd_rn(v, to_f<T>(bias[gn]));  // AddBias after the product (cpu_backend.go:619-621)
      if (act == FLETCHER_ACT_GELU) v = gelu_fast(v);
      else if (act == FLETCHER_ACT_TANH) v = tanh_fast(v);
      C[gm * ldc + gn] = from_f<T>(v);
    }
  }
}
}  // namespace

int32_t launch_gemm_simt_strided(Ctx* c, int32_t dt, const void* A, int64_t sam, int64_t sak, const void* B,
                                 int64_t sbk, int64_t sbn, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                                 const void* bias, int32_t act) {
  if (M <= 0 || N <= 0) return FLETCHER_OK;
  FL_CHECK(c, (N + TN - 1) / TN < 65536 * 1024 && (M + TM - 1) / TM < 65536, "gemm_simt: shape too large");
  dim3 grid((unsigned)((N + TN - 1) / TN), (unsigned)((M + TM - 1) / TM));
  if (dt == FLETCHER_F32)
    k_sgemm<float><<<grid, 256, 0, c->stream>>>((const float*)A, sam, sak, (const float*)B, sbk, sbn, (float*)C, ldc,
                                                M, N, K, (const float*)bias, act);
  else if (dt == FLETCHER_BF16)
    k_sgemm<__nv_bfloat16><<<grid, 256, 0, c->stream>>>((const __nv_bfloat16*)A, sam, sak, (const __nv_bfloat16*)B,
                                                        sbk, sbn, (__nv_bfloat16*)C, ldc, M, N, K,
                                                        (const __nv_bfloat16*)bias, act);
  else
    k_sgemm<__half><<<grid, 256, 0, c->stream>>>((const __half*)A, sam, sak, (const __half*)B, sbk, sbn, (__half*)C,
                                                 ldc, M, N, K, (const __half*)bias, act);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

int32_t launch_gemm_simt(Ctx* c, int32_t dt, const void* A, int64_t lda, const void* B, int64_t ldb, void* C,
                         int64_t ldc, int64_t M, int64_t N, int64_t K, const void* bias, int32_t act) {
  return launch_gemm_simt_strided(c, dt, A, lda, 1, B, ldb, 1, C, ldc, M, N, K, bias, act);
}

// Kept for callers that only deal in fp32.
int32_t launch_sgemm(Ctx* c, const float* A, int64_t lda, const float* Bm, int64_t ldb, float* C, int64_t ldc,
                     int64_t M, int64_t N, int64_t K, const float* bias, int32_t act) {
  return launch_gemm_simt(c, FLETCHER_F32, A, lda, Bm, ldb, C, ldc, M, N, K, bias, act);
}

}  // namespace fl
