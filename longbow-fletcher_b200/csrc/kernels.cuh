// Launchers shared between the tensor-op ABI (ops.cu) and the whole-model path (model.cu).
#pragma once
#include "common.cuh"

namespace fl {

int32_t convert_from_f32(Ctx* c, const float* src, void* dst, int32_t dtype, int64_t n);
int32_t convert_to_f32(Ctx* c, const void* src, int32_t dtype, float* dst, int64_t n);
int32_t check_device_flag(Ctx* c);

// out[r] = LayerNorm(x[r] (+ res[r])) with fp32 statistics; gamma/beta fp32.  out may alias x.
int32_t launch_add_layernorm(Ctx* c, int32_t dtype, const void* x, const void* res, void* out,
                             const float* gamma, const float* beta, int64_t rows, int64_t cols,
                             float eps);

// Embedding: out[t] = LN(word[ids[t]] (+ pos_table[min(pos[t], P-1)]) + type0) (bert.go:215-261).
int32_t launch_embed(Ctx* c, int32_t dtype, const int32_t* ids, const int32_t* pos,
                     const void* word, const void* pos_table, int32_t max_pos, const void* type0,
                     const float* gamma, const float* beta, void* out, int64_t T, int64_t H,
                     float eps);

// pos[t] = index of row t within its sequence; cu_seqlens has B+1 entries.
int32_t launch_positions(Ctx* c, const int32_t* cu_seqlens, int32_t B, int32_t* pos, int32_t max_len);

// Mean over each sequence's rows, then L2-normalised; out fp32 [B, H].
int32_t launch_mean_pool_l2(Ctx* c, int32_t dtype, const void* hidden, const int32_t* cu_seqlens,
                            int32_t B, int64_t H, float* out);

// The final LayerNorm fused into mean pooling + L2 (16-bit models): out[s] = L2(mean over the
// rows of sequence s of LayerNorm(x[r])), without writing the normalised rows.  ws holds
// ln_pool_workspace_bytes() of chunk sums.
bool ln_pool_supported(int32_t dtype, int64_t H);
int64_t ln_pool_workspace_bytes(int32_t B, int32_t max_len, int64_t H);
int32_t launch_ln_mean_pool_l2(Ctx* c, int32_t dtype, const void* x, const int32_t* cu, const float* gamma,
                               const float* beta, float eps, int32_t B, int32_t max_len, int64_t H, float* ws,
                               float* out);

// Gathers rows rows_idx[i] of src (dtype) into dst fp32 [n, H].
int32_t launch_gather_rows_f32(Ctx* c, int32_t dtype, const void* src, const int32_t* rows_idx,
                               int64_t n, int64_t H, float* dst);

// RoPE (rotate-half) in place on the first `ncols_rot` columns of rows [T, ld] using the
// cos/sin table [table_len, dh/2] (fp32): every dh-wide head block is rotated.
int32_t launch_rope_table(Ctx* c, int32_t dtype, void* x, int64_t T, int64_t ld, int64_t ncols_rot,
                          int32_t dh, const int32_t* pos, const float* cos_t, const float* sin_t);
// Builds the cos/sin table with float64 trig (cpu_backend.go:790-792).
int32_t launch_rope_build_table(Ctx* c, float* cos_t, float* sin_t, int32_t len, int32_t dh,
                                double base);

// fp32 SIMT GEMM: C[M,N] = act(A[M,K] . B[K,N] + bias), B row-major (in, out).
// lda/ldb/ldc in elements.  act: FLETCHER_ACT_* (IDENTITY, GELU, TANH).
int32_t launch_sgemm(Ctx* c, const float* A, int64_t lda, const float* Bm, int64_t ldb, float* C,
                     int64_t ldc, int64_t M, int64_t N, int64_t K, const float* bias, int32_t act);

// SwiGLU over [rows, 2I] -> [rows, I] with the reference's float64 exp.
int32_t launch_swiglu(Ctx* c, int32_t dtype, const void* in, void* out, int64_t rows, int64_t I);

// fp32 attention with the reference's SoftmaxFast (parity mode).  q/k/v rows have stride
// ld_in (elements), output stride ld_out.  cu_seqlens [B+1].
int32_t launch_attention_f32(Ctx* c, const float* q, const float* k, const float* v, int64_t ld_in,
                             float* out, int64_t ld_out, const int32_t* cu_seqlens, int32_t B,
                             int64_t T, int32_t nh, int32_t dh, float scale, int32_t max_len);

// bf16/f16 flash attention on tcgen05 (attention_tc.cu), head_dim 64: q/k/v [T, H] views with
// row stride ld_in; tiles128: one attn_tile() per 128-row query tile.
int32_t launch_flash_attention_tc(Ctx* c, int32_t dtype, const void* q, const void* k, const void* v,
                                  int64_t ld_in, int64_t T, int64_t H, void* out, int64_t ld_out,
                                  const int32_t* cu_seqlens, const int2* tiles128, int32_t num_tiles,
                                  int32_t nh, float scale);
// Query-tile height of launch_flash_attention_tc, and the longest sequence it takes.
constexpr int kAttnTileRows = 128;
constexpr int kAttnMaxLen = 65535;
// Query-tile descriptor: {first row of the sequence, (sequence length << 16) | first query row
// of the tile within the sequence}; self-contained, so the kernel decodes it with one load.
inline int2 attn_tile(int32_t seq_start, int32_t len, int32_t q0) {
  return make_int2(seq_start, (int32_t)(((uint32_t)len << 16) | (uint32_t)q0));
}

// Elementwise helpers.
int32_t launch_scale_add(Ctx* c, int32_t dtype, void* x, const void* other, float scale,
                         float add, int64_t n);  // x = x*scale + add (+ other)
int32_t launch_add_bias(Ctx* c, int32_t dtype, void* x, const void* bias, int64_t rows, int64_t cols);
int32_t launch_activation(Ctx* c, int32_t dtype, void* x, int64_t rows, int64_t cols, int32_t act);
int32_t launch_has_nan(Ctx* c, int32_t dtype, const void* x, int64_t n, int32_t* d_flag);
// ref: use the reference's fp16 conversion (pass ctx->half_mode == FLETCHER_HALF_REFERENCE for
// host-facing casts); internal casts round to nearest even.
int32_t launch_cast(Ctx* c, int32_t sdt, const void* s, int32_t ddt, void* d, int64_t n, bool ref = false);

// Weight packing: dst[n', k] (row-major, K contiguous) = src[k, perm(n')] for fp32 src (in,out);
// an fp16 destination uses the context's host conversion mode.
// perm: 0 identity; 1 = SwiGLU interleave of 128-column gate/up blocks (see gemm_tc.cu).
int32_t launch_pack_weight_kmajor(Ctx* c, const float* src, int64_t K, int64_t N, void* dst,
                                  int32_t dtype, int32_t perm, int32_t block_n);

// Same packing from a 16-bit (in,out) [K, N] matrix of dtype dt into K-major [N', K].
int32_t launch_pack_kmajor_16(Ctx* c, int32_t dt, const void* src, int64_t K, int64_t N, void* dst, int32_t perm,
                              int32_t block_n);

// One checkpoint weight (in,out) [K, N] (src_t = 1: stored (out,in)) of dtype sdt into a model
// buffer of dtype ddt: K-major rows at row offset `off` with permutation perm (dst_kmajor = 1),
// or (in,out) with row stride ld at column offset `off`.
int32_t launch_place_weight(Ctx* c, int32_t sdt, const void* src, int64_t K, int64_t N, int src_t, int32_t ddt,
                            void* dst, int dst_kmajor, int64_t ld, int64_t off, int perm, int block_n);

}  // namespace fl
