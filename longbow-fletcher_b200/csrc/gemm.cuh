// GEMM entry points: the tcgen05 tensor-core GEMM (gemm_tc.cu) and the SIMT GEMM (gemm_simt.cu).
#pragma once
#include "kernels.cuh"

namespace fl {

// Fused epilogues of the tensor-core GEMM.
enum Epi : int {
  EPI_STORE = 0,    // out = acc + bias
  EPI_ROPE = 1,     // out = rope(acc + bias) on columns < rope_cols (head_dim 64), pos[row]
  EPI_GELU = 2,     // out = GeluFast(acc + bias)
  EPI_SWIGLU = 3,   // out[:, j] = silu(gate + bg) * (up + bu), W packed gate/up-interleaved
  EPI_RESIDUAL = 4,  // out = acc + bias + residual
  EPI_PARTIAL = 5,   // internal (split-K): fp32 sums of one K range to a workspace, finished later
  EPI_RESIDUAL_TMA = 6  // internal: EPI_RESIDUAL with the residual loaded by TMA (chosen for K <= 1024)
};

struct GemmArgs {
  int64_t M, N;
  int K;
  int num_m_tiles, num_n_tiles;
  void* out;
  int64_t ld_out;
  const float* bias;
  const void* residual;
  int64_t ld_res;
  const int32_t* pos;
  const float* cos_t;
  const float* sin_t;
  int64_t rope_cols;
  int32_t* err;
  int splits;      // K ranges per output tile (1 unless EPI_PARTIAL)
  int kb_per;      // 64-wide K blocks per range
  float* partial;  // EPI_PARTIAL: [splits, M, N] fp32
};

bool gemm_tc_supported(int64_t M, int64_t N, int64_t K, int bn);

// Split-K for GEMMs with few output tiles: the plan's fp32 workspace bytes (0 = no split).  A
// launch splits only when the context's workspace (Ctx::splitk, lent by the model that owns
// it) is large enough; launches never allocate.
int64_t gemm_splitk_plan(const Ctx* c, int64_t M, int64_t N, int64_t K, int* splits, int* kb_per);

// A: [M, K] row-major 16-bit; W: [N, K] (K-major) 16-bit; bias fp32 [N] (packed order) or null.
int32_t launch_gemm_tc(Ctx* c, int32_t dtype, int epi, int bn, const void* A, int64_t M, int64_t K, const void* W,
                       int64_t N, void* out, int64_t ld_out, const float* bias, const void* residual, int64_t ld_res,
                       const int32_t* pos, const float* cos_t, const float* sin_t, int64_t rope_cols);

// SIMT GEMM for any dtype (fp32 compute): C[M,N] = act(A[M,K] . B[K,N] + bias) with B row-major
// (in, out) and optional row gather of A.  Used for fp32 parity mode and small/odd shapes.
int32_t launch_gemm_simt(Ctx* c, int32_t dtype, const void* A, int64_t lda, const void* B, int64_t ldb, void* C,
                         int64_t ldc, int64_t M, int64_t N, int64_t K, const void* bias, int32_t act);

// The same with element strides: A(m, k) = A[m*sam + k*sak], B(k, n) = B[k*sbk + n*sbn].
int32_t launch_gemm_simt_strided(Ctx* c, int32_t dtype, const void* A, int64_t sam, int64_t sak, const void* B,
                                 int64_t sbk, int64_t sbn, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                                 const void* bias, int32_t act);

}  // namespace fl
