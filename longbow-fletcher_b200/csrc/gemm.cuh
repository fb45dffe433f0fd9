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
  EPI_RESIDUAL = 4  // out = acc + bias + residual
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
};

bool gemm_tc_supported(int64_t M, int64_t N, int64_t K, int bn);

// A: [M, K] row-major 16-bit; W: [N, K] (K-major) 16-bit; bias fp32 [N] (packed order) or null.
int32_t launch_gemm_tc(Ctx* c, int32_t dtype, int epi, int bn, const void* A, int64_t M, int64_t K, const void* W,
                       int64_t N, void* out, int64_t ld_out, const float* bias, const void* residual, int64_t ld_res,
                       const int32_t* pos, const float* cos_t, const float* sin_t, int64_t rope_cols);

// SIMT GEMM for any dtype (fp32 compute): C[M,N] = act(A[M,K] . B[K,N] + bias) with B row-major
// (in, out) and optional row gather of A.  Used for fp32 parity mode and small/odd shapes.
int32_t launch_gemm_simt(Ctx* c, int32_t dtype, const void* A, int64_t lda, const void* B, int64_t ldb, void* C,
                         int64_t ldc, int64_t M, int64_t N, int64_t K, const void* bias, int32_t act);

}  // namespace fl
