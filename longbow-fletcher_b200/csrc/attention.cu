// fp32 attention over packed variable-length sequences (the parity path; the bf16/f16 path is
// attention_tc.cu).
//
// Reference: BertSelfAttention.ForwardBatch (bert.go:610-728) -> CPUTensor.Attention
// (cpu_backend.go:662-758): per sequence, per head, P = SoftmaxFast(scale * Q_h K_h^T),
// O_h = P V_h.  Sequences are described by cu_seqlens (prefix sums of the lengths); keys past
// a sequence's end are masked, so packing replaces padding.
//
// k_attn_f32: one CTA per (query row, head); scores in shared memory, the reference's ExpFast
// softmax (max, ExpFast(s-max), sum, * 1/sum) then P.V.
#include <atomic>

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
  // The attribute is per device; set it once to the cap checked above, so that replica threads
  // sharing a GPU never lower it between another thread's set and launch.
  static std::atomic<bool> attr_set[64] = {};
  if (smem > 48 * 1024 && c->device < 64 && !attr_set[c->device].load(std::memory_order_acquire)) {
    FL_CUDA(c, cudaFuncSetAttribute(k_attn_f32, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set[c->device].store(true, std::memory_order_release);
  }
  dim3 grid((unsigned)T, (unsigned)nh);
  k_attn_f32<<<grid, 128, smem, c->stream>>>(q, k, v, ld_in, out, ld_out, cu, B, dh, scale);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

}  // namespace fl
