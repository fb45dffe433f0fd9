// Flash attention on the 5th-generation tensor cores (tcgen05 / TMEM / TMA), bf16 or fp16,
// head_dim 64, packed variable-length sequences.
//
// Reference semantics: BertSelfAttention.ForwardBatch (bert.go:610-728) -> CPUTensor.Attention
// (cpu_backend.go:662-758): per sequence and head, O = softmax(scale * Q K^T) V, keys limited to
// the sequence (cu_seqlens).
//
// Persistent kernel: each CTA walks work items w = (128-query tile, head) in a strided order
// (tiles come longest-sequence first).  The three roles run through one continuous sequence of
// 64-key blocks g across all of the CTA's work items, so the next item's Q load and first
// Q K^T overlap the previous item's tail.  192 threads:
//   warp 0    : TMA producer — Q tile per work item (2 buffers), K and V blocks (2-stage ring);
//   warp 1    : MMA issuer — S_g = Q K_g^T (M=128, N=64, K=64) into TMEM S buffer g&1, and
//               O_g = P_g V_g (M=128, N=64, K=64 keys; V read MN-major straight from its TMA
//               tile) into TMEM O buffer g&1; S_{g+1} is issued before waiting for P_g;
//   warps 2-5 : softmax — thread = query row: tcgen05.ld its S row, mask keys past the
//               sequence end, online max / exp2 / row sum, write P (16-bit) to 128B-swizzled
//               smem for the PV MMA, accumulate O_g from TMEM into fp32 registers with the exact
//               rescale exp2((m_old - m_new) * scale * log2 e), and store finished rows.
// TMEM: 2 x 64 (S) + 2 x 64 (O) = 256 columns; ~97 KB smem -> two CTAs per SM.
// All mbarrier waits are bounded (device error flag + abort, as in the GEMM).  No multicast.
#include "tc_common.cuh"

namespace fl {
namespace tca {

using namespace tc;

constexpr int BQ = 128, BKV = 64, D = 64;
constexpr int kThreads = 192;
constexpr int Q_BYTES = BQ * D * 2;
constexpr int KV_BYTES = BKV * D * 2;
constexpr int P_BYTES = BQ * BKV * 2;
constexpr int OFF_Q = 0;  // 2 buffers
constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
constexpr int OFF_V = OFF_K + 2 * KV_BYTES;
constexpr int OFF_P = OFF_V + 2 * KV_BYTES;
constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr int TMEM_COLS = 256;  // S0 [0,64) S1 [64,128) O0 [128,192) O1 [192,256)

struct AttnArgs {
  const int32_t* cu;
  const int2* tiles;
  int num_work;  // tiles * heads
  int nh;
  void* out;
  int64_t ld_out;
  float sl2;  // scale * log2(e)
  int32_t* err;
};

struct Work {
  int start, L, q0, h, nb;
};

// 2^x on the SFU (one instruction; -inf -> 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Packed two-lane fp32 FMA / add (sm_100): one instruction for two values.
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

__device__ __forceinline__ Work decode(const AttnArgs& a, int w) {
  const int2 t = a.tiles[w / a.nh];
  Work r;
  r.h = w % a.nh;
  r.start = a.cu[t.x];
  r.L = a.cu[t.x + 1] - r.start;
  r.q0 = t.y;
  r.nb = (r.L + BKV - 1) / BKV;
  return r;
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

template <typename T>
__device__ __forceinline__ void store_row(const AttnArgs& a, const Work& wk, int r, const float (&o)[D], float l) {
  if (wk.q0 + r >= wk.L) return;
  const float inv = 1.0f / l;
  T* dst = reinterpret_cast<T*>(a.out) + (int64_t)(wk.start + wk.q0 + r) * a.ld_out + wk.h * D;
#pragma unroll
  for (int c = 0; c < 8; c++) {
    const float* v = &o[c * 8];
    reinterpret_cast<uint4*>(dst)[c] =
        make_uint4(pack2<T>(v[0] * inv, v[1] * inv), pack2<T>(v[2] * inv, v[3] * inv),
                   pack2<T>(v[4] * inv, v[5] * inv), pack2<T>(v[6] * inv, v[7] * inv));
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    k_attn_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;         // [2]
  uint64_t* q_empty = bars + 2;    // [2]
  uint64_t* kv_full = bars + 4;    // [2]
  uint64_t* kv_empty = bars + 6;   // [2]
  uint64_t* s_full = bars + 8;     // [2]
  uint64_t* s_free = bars + 10;    // [2]
  uint64_t* p_full = bars + 12;    // [2]
  uint64_t* o_full = bars + 14;    // [2]
  uint64_t* o_free = bars + 16;    // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 128);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmQ) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmK) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmV) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0, t = 0;
      for (int w = blockIdx.x; w < args.num_work; w += gridDim.x, ++t) {
        const Work wk = decode(args, w);
        const int qb = t & 1;
        if (!mbar_wait(&q_empty[qb], ((t >> 1) & 1) ^ 1, abort, args.err)) break;
        mbar_expect_tx(&q_full[qb], Q_BYTES);
        tma_load_2d(smem + OFF_Q + qb * Q_BYTES, &tmQ, &q_full[qb], wk.h * D, wk.start + wk.q0);
        bool ok = true;
        for (int j = 0; j < wk.nb; j++, g++) {
          const int b = g & 1;
          if (!mbar_wait(&kv_empty[b], ((g >> 1) & 1) ^ 1, abort, args.err)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&kv_full[b], 2 * KV_BYTES);
          tma_load_2d(smem + OFF_K + b * KV_BYTES, &tmK, &kv_full[b], wk.h * D, wk.start + j * BKV);
          tma_load_2d(smem + OFF_V + b * KV_BYTES, &tmV, &kv_full[b], wk.h * D, wk.start + j * BKV);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = idesc<T, BQ, BKV>();
      const uint32_t id_o = idesc<T, BQ, D, true>();
      // O_i = P_i V_i for block i (buffers i&1).
      auto issue_pv = [&](int i) -> bool {
        const int b = i & 1;
        if (!mbar_wait(&p_full[b], (i >> 1) & 1, abort, args.err)) return false;
        if (!mbar_wait(&o_free[b], ((i >> 1) & 1) ^ 1, abort, args.err)) return false;
        tc_fence_after();
        const uint64_t p_desc = sw128_desc(smem_u32(smem + OFF_P + b * P_BYTES));
        const uint64_t v_desc = sw128_desc_mn(smem_u32(smem + OFF_V + b * KV_BYTES));
#pragma unroll
        for (int k = 0; k < BKV / 16; k++)  // 16 keys per step: +32 B in P's K-major atom, +2 KB in V
          mma_f16(tmem + 2 * BKV + b * D, p_desc + 2 * k, v_desc + (uint64_t)k * (2048 >> 4), id_o, k > 0);
        mma_commit(&o_full[b]);
        mma_commit(&kv_empty[b]);
        return true;
      };
      int g = 0, t = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < args.num_work && ok; w += gridDim.x, ++t) {
        const Work wk = decode(args, w);
        const int qb = t & 1;
        if (!mbar_wait(&q_full[qb], (t >> 1) & 1, abort, args.err)) break;
        const uint64_t q_desc = sw128_desc(smem_u32(smem + OFF_Q + qb * Q_BYTES));
        for (int j = 0; j < wk.nb; j++, g++) {
          const int b = g & 1;
          if (!mbar_wait(&kv_full[b], (g >> 1) & 1, abort, args.err) ||
              !mbar_wait(&s_free[b], ((g >> 1) & 1) ^ 1, abort, args.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t k_desc = sw128_desc(smem_u32(smem + OFF_K + b * KV_BYTES));
#pragma unroll
          for (int k = 0; k < D / 16; k++) mma_f16(tmem + b * BKV, q_desc + 2 * k, k_desc + 2 * k, id_s, k > 0);
          mma_commit(&s_full[b]);
          if (j == wk.nb - 1) mma_commit(&q_empty[qb]);  // Q buffer free once these MMAs finish
          if (g >= 1 && !issue_pv(g - 1)) {
            ok = false;
            break;
          }
        }
      }
      if (ok && g >= 1) issue_pv(g - 1);
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;  // query row within the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const float sl2 = args.sl2;
    float o[D];
#pragma unroll
    for (int i = 0; i < D; i++) o[i] = 0.f;
    float m = -INFINITY, l = 0.f, m_o = -INFINITY;
    Work prev{};
    int g = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < args.num_work && ok; w += gridDim.x) {
      const Work wk = decode(args, w);
      for (int j = 0; j < wk.nb; j++, g++) {
        const int b = g & 1;
        if (!mbar_wait(&s_full[b], (g >> 1) & 1, abort, args.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int kbase = j * BKV;
        const int valid = wk.L - kbase;  // keys of this block inside the sequence (>= 1)
        // m_pb: the max that P_{g-1} was computed with; l_prev: finished row sum of the previous item.
        const float m_pb = m;
        const float l_prev = l;
        if (j == 0) {
          m = -INFINITY;
          l = 0.f;
        }
        // The block's S row (one 64-column TMEM load), masked past the sequence end.
        float sv[BKV];
        tmem_ld64(tmem + lane_off + b * BKV, sv);
        tc_fence_before();
        mbar_arrive(&s_free[b]);
        if (valid < BKV) {  // only a sequence's last block needs the key mask
#pragma unroll
          for (int i = 0; i < BKV; i++)
            if (i >= valid) sv[i] = -INFINITY;
        }
        // Row max as a tree (8 independent chains, then a pairwise fold) to keep latency short.
        float mp[8];
#pragma unroll
        for (int k = 0; k < 8; k++) mp[k] = fmaxf(sv[k], sv[8 + k]);
#pragma unroll
        for (int i = 16; i < BKV; i += 8)
#pragma unroll
          for (int k = 0; k < 8; k++) mp[k] = fmaxf(mp[k], sv[i + k]);
        const float mx = fmaxf(m, fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                                         fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7]))));
        const float corr = ex2((m - mx) * sl2);
        const float ms = mx * sl2;
        m = mx;
        // P = exp2(S*scale*log2e - max) -> smem (row r, 64 keys = 128 B, 128-byte swizzle, K-major
        // for the PV MMA).  P buffer g&1 is free: PV_{g-2} finished before O_{g-2} was read.
        float ra[4][2] = {};  // four independent packed partial sums
#pragma unroll
        for (int i = 0; i < BKV; i += 2) {
          fma2(sv[i], sv[i + 1], sv[i], sv[i + 1], sl2, sl2, -ms, -ms);
          sv[i] = ex2(sv[i]);
          sv[i + 1] = ex2(sv[i + 1]);
          add2(ra[(i >> 1) & 3][0], ra[(i >> 1) & 3][1], sv[i], sv[i + 1]);
        }
        const float rsum = ((ra[0][0] + ra[0][1]) + (ra[1][0] + ra[1][1])) + ((ra[2][0] + ra[2][1]) + (ra[3][0] + ra[3][1]));
        uint8_t* prow = smem + OFF_P + b * P_BYTES + r * 128;
#pragma unroll
        for (int c = 0; c < 8; c++) {
          const float* v = &sv[c * 8];
          uint4 wv = make_uint4(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]), pack2<T>(v[4], v[5]), pack2<T>(v[6], v[7]));
          *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = wv;
        }
        l = l * corr + rsum;
        fence_async_smem();
        mbar_arrive(&p_full[b]);
        if (g >= 1) {  // O_{g-1} is ready once PV_{g-1} ran; that also frees P buffer (g-1)&1
          const int i = g - 1, bo = i & 1;
          if (!mbar_wait(&o_full[bo], (i >> 1) & 1, abort, args.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float f = exp2f((m_o - m_pb) * sl2);
          {
            float tt[D];
            tmem_ld64(tmem + lane_off + 2 * BKV + bo * D, tt);
#pragma unroll
            for (int c = 0; c < D; c += 2) fma2(o[c], o[c + 1], o[c], o[c + 1], f, f, tt[c], tt[c + 1]);
          }
          tc_fence_before();
          mbar_arrive(&o_free[bo]);
          m_o = m_pb;
          if (j == 0) {  // block g-1 closed the previous work item
            store_row<T>(args, prev, r, o, l_prev);
#pragma unroll
            for (int c = 0; c < D; c++) o[c] = 0.f;
            m_o = -INFINITY;
          }
        }
      }
      prev = wk;
    }
    if (ok && g >= 1) {
      const int i = g - 1, bo = i & 1;
      if (mbar_wait(&o_full[bo], (i >> 1) & 1, abort, args.err)) {
        tc_fence_after();
        const float f = exp2f((m_o - m) * sl2);
        {
          float tt[D];
          tmem_ld64(tmem + lane_off + 2 * BKV + bo * D, tt);
#pragma unroll
          for (int c = 0; c < D; c += 2) fma2(o[c], o[c + 1], o[c], o[c + 1], f, f, tt[c], tt[c + 1]);
        }
        store_row<T>(args, prev, r, o, l);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

}  // namespace tca

int32_t make_tma_map_2d(Ctx* c, CUtensorMap* m, int32_t dtype, const void* ptr, uint64_t rows, uint64_t cols,
                        uint64_t ld, uint32_t box_cols, uint32_t box_rows);

int32_t launch_flash_attention_tc(Ctx* c, int32_t dt, const void* q, const void* k, const void* v, int64_t ld_in,
                                  int64_t T, int64_t H, void* out, int64_t ld_out, const int32_t* cu,
                                  const int2* tiles128, int32_t num_tiles, int32_t nh, float scale) {
  using namespace tca;
  if (num_tiles <= 0) return FLETCHER_OK;
  FL_CHECK(c, H == (int64_t)nh * D, "attention_tc: head_dim must be 64");
  FL_CHECK(c, ld_in % 8 == 0 && ld_out % 8 == 0 && ((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 &&
                  ((uintptr_t)v & 15) == 0 && ((uintptr_t)out & 15) == 0,
           "attention_tc: rows must be 16-byte aligned");
  FL_CHECK(c, (int64_t)num_tiles * nh < (1ll << 31), "attention_tc: too many work items");
  CUtensorMap mq, mk, mv;
  int32_t rc;
  if ((rc = make_tma_map_2d(c, &mq, dt, q, (uint64_t)T, (uint64_t)H, (uint64_t)ld_in, D, BQ))) return rc;
  if ((rc = make_tma_map_2d(c, &mk, dt, k, (uint64_t)T, (uint64_t)H, (uint64_t)ld_in, D, BKV))) return rc;
  if ((rc = make_tma_map_2d(c, &mv, dt, v, (uint64_t)T, (uint64_t)H, (uint64_t)ld_in, D, BKV))) return rc;
  const int work = num_tiles * nh;
  AttnArgs a{cu, tiles128, work, nh, out, ld_out, scale * 1.4426950408889634f, c->d_err};
  static bool attr_set[2][64] = {};
  const int ti = dt == FLETCHER_BF16 ? 0 : 1;
  if (!attr_set[ti][c->device & 63]) {
    if (dt == FLETCHER_BF16)
      FL_CUDA(c, cudaFuncSetAttribute(k_attn_tc<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    else
      FL_CUDA(c, cudaFuncSetAttribute(k_attn_tc<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    attr_set[ti][c->device & 63] = true;
  }
  const int grid = work < 2 * c->num_sms ? work : 2 * c->num_sms;
  if (dt == FLETCHER_BF16)
    k_attn_tc<__nv_bfloat16><<<grid, kThreads, SMEM, c->stream>>>(mq, mk, mv, a);
  else
    k_attn_tc<__half><<<grid, kThreads, SMEM, c->stream>>>(mq, mk, mv, a);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

}  // namespace fl
