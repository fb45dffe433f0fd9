// Flash attention on tcgen05 with S double-buffered in tensor memory: while the softmax warps
// work on block j, S for block j+1 is already complete in the other buffer, so no softmax ever
// waits for an S round trip.
//
// Reference semantics as attention_tc.cu: BertSelfAttention.ForwardBatch (bert.go:610-728) ->
// CPUTensor.Attention (cpu_backend.go:662-758): per sequence and head O = softmax(scale QK^T) V.
//
// One query-tile slot per CTA, two CTAs per SM, 160 threads:
//   warp 0    : one control thread — TMA loads (Q per work item in a 2-deep ring; K in a 3-stage
//               ring freed by the S MMAs; V in a 2-stage ring freed by the PV MMAs) and MMA issue
//               over the CTA's whole stream of 64-key blocks g = 0, 1, 2, ... (all blocks of all
//               its work items, in order):
//                 S_g = Q K_g^T        (M=128, N=64, K=64) into S buffer g % 2,
//                 O  += P_g V_g        (P_g read from TMEM over S buffer g % 2's upper half),
//               issuing S_{g+2} right after PV_g (same buffer; tcgen05.mma runs in issue order);
//   warps 1-4 : softmax, thread = query row, as in attention_tc.cu: tcgen05.ld the S row, exp2
//               against a lazily moved reference max, tcgen05.st the 16-bit P row.
// TMEM: S buffer 0 columns [0, 64), S buffer 1 [64, 128), O [128, 192); 256 allocated.
// Shared memory: Q 2 x 16 KB, K 3 x 8 KB, V 2 x 8 KB (72 KB).  Every mbarrier wait is bounded
// (device error flag + abort); no multicast.
#include <atomic>

#include "attn_common.cuh"
#include "kernels.cuh"

namespace fl {
namespace tcd {

using namespace tc;
using namespace tca;

constexpr int BQ = 128, BKV = 64, D = 64;
constexpr int kThreads = 32 + 128;
constexpr int Q_BYTES = BQ * D * 2, KV_BYTES = BKV * D * 2;
constexpr int KST = 3, VST = 2;  // K and V ring depths
constexpr int OFF_Q = 0, OFF_K = 2 * Q_BYTES, OFF_V = OFF_K + KST * KV_BYTES;
constexpr int OFF_BAR = OFF_V + VST * KV_BYTES;
constexpr int kBars = 24;
constexpr int SMEM = OFF_BAR + kBars * 8 + 16 + 1024;
constexpr int TMEM_COLS = 256;

struct DbArgs {
  const int2* tiles;
  int num_work;  // tiles * heads
  int nh;
  void* out;
  int64_t ld_out;
  float sl2;  // scale * log2(e)
  int32_t* err;
  int st256;  // output rows 32-byte aligned: 256-bit stores
};

struct Item {
  int start, L, q0, h, nb;
};

__device__ __forceinline__ Item decode_item(const DbArgs& a, int w) {
  const int2 t = a.tiles[w / a.nh];
  Item r;
  r.h = w % a.nh;
  r.start = t.x;
  r.L = (int)((uint32_t)t.y >> 16);
  r.q0 = t.y & 0xFFFF;
  r.nb = (r.L + BKV - 1) / BKV;
  return r;
}

// A position in the CTA's block stream: item ordinal k (work item blockIdx.x + k * gridDim.x),
// block j of that item.
struct Cursor {
  int k = 0, j = 0;
  Item it{};
  bool valid = false;
  __device__ void start(const DbArgs& a) {
    k = 0;
    j = 0;
    valid = (int)blockIdx.x < a.num_work;
    if (valid) it = decode_item(a, blockIdx.x);
  }
  __device__ void next(const DbArgs& a) {
    if (!valid) return;
    if (++j < it.nb) return;
    j = 0;
    ++k;
    const int w = (int)blockIdx.x + k * (int)gridDim.x;
    valid = w < a.num_work;
    if (valid) it = decode_item(a, w);
  }
};

struct Bars {
  uint64_t *q_full, *q_empty, *k_full, *k_empty, *v_full, *v_empty, *s_full, *p_full, *pv_done, *o_full, *o_free,
      *drain;
  __device__ Bars(uint64_t* b)
      : q_full(b), q_empty(b + 2), k_full(b + 4), k_empty(b + 7), v_full(b + 10), v_empty(b + 12), s_full(b + 14),
        p_full(b + 16), pv_done(b + 18), o_full(b + 19), o_free(b + 20), drain(b + 21) {}
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    k_attn_db(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmV, const DbArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  Bars B(bars);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&B.q_full[i], 1);
      mbar_init(&B.q_empty[i], 1);
      mbar_init(&B.v_full[i], 1);
      mbar_init(&B.v_empty[i], 1);
      mbar_init(&B.s_full[i], 1);
      mbar_init(&B.p_full[i], 128);
    }
    for (int i = 0; i < KST; i++) {
      mbar_init(&B.k_full[i], 1);
      mbar_init(&B.k_empty[i], 1);
    }
    mbar_init(B.pv_done, 1);
    mbar_init(B.o_full, 1);
    mbar_init(B.o_free, 128);
    mbar_init(B.drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmQ) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmK) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmV) : "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();  // the setup above overlapped the previous kernel; its outputs are visible now

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t id_s = idesc<T, BQ, BKV>();
      const uint32_t id_o = idesc<T, BQ, D, true>();
      bool ok = true;
      // Cursors: PV (g), S (g + 2), K loads (g + 3), V loads (g + 2), Q loads (item k + 2).
      Cursor pv, sc, kl, vl;
      pv.start(args);
      sc = pv;
      kl = pv;
      vl = pv;
      uint32_t g = 0, gs = 0, gk = 0, gv = 0;  // blocks: PV'd, S issued, K loaded, V loaded
      int kq = 0;                              // items whose Q was loaded
      auto load_q = [&]() -> bool {            // Q of item kq into buffer kq % 2
        const int w = (int)blockIdx.x + kq * (int)gridDim.x;
        if (w >= args.num_work) return true;
        const int b = kq & 1;
        if (kq >= 2 && !mbar_wait(&B.q_empty[b], ((kq >> 1) - 1) & 1, abort, args.err)) return false;
        const Item it = decode_item(args, w);
        mbar_expect_tx(&B.q_full[b], Q_BYTES);
        tma_load_2d(smem + OFF_Q + b * Q_BYTES, &tmQ, &B.q_full[b], it.h * D, it.start + it.q0);
        kq++;
        return true;
      };
      auto load_k = [&]() -> bool {  // the next K block, once the S that last read its stage ran
        if (!kl.valid) return true;
        const int b = gk % KST;
        if (gk >= KST && !mbar_wait(&B.k_empty[b], ((gk / KST) - 1) & 1, abort, args.err)) return false;
        mbar_expect_tx(&B.k_full[b], KV_BYTES);
        tma_load_2d(smem + OFF_K + b * KV_BYTES, &tmK, &B.k_full[b], kl.it.h * D, kl.it.start + kl.j * BKV);
        gk++;
        kl.next(args);
        return true;
      };
      auto load_v = [&]() -> bool {  // the next V block, once the PV that last read its stage ran
        if (!vl.valid) return true;
        const int b = gv % VST;
        if (gv >= VST && !mbar_wait(&B.v_empty[b], ((gv / VST) - 1) & 1, abort, args.err)) return false;
        mbar_expect_tx(&B.v_full[b], KV_BYTES);
        tma_load_2d(smem + OFF_V + b * KV_BYTES, &tmV, &B.v_full[b], vl.it.h * D, vl.it.start + vl.j * BKV);
        gv++;
        vl.next(args);
        return true;
      };
      auto issue_s = [&]() -> bool {  // S for block gs into buffer gs % 2
        if (!sc.valid) return true;
        while (sc.j == 0 && kq <= sc.k)  // this item's Q (item sc.k exists, so each call loads one)
          if (!load_q()) return false;
        const int qb = sc.k & 1;
        if (sc.j == 0 && !mbar_wait(&B.q_full[qb], (sc.k >> 1) & 1, abort, args.err)) return false;
        const int kb = gs % KST;
        if (!mbar_wait(&B.k_full[kb], (gs / KST) & 1, abort, args.err)) return false;
        tc_fence_after();
        const uint64_t q_desc = sw128_desc(smem_u32(smem + OFF_Q + qb * Q_BYTES));
        const uint64_t k_desc = sw128_desc(smem_u32(smem + OFF_K + kb * KV_BYTES));
        const uint32_t t_s = tmem + (gs & 1) * 64;
#pragma unroll
        for (int k = 0; k < D / 16; k++) mma_f16(t_s, q_desc + 2 * k, k_desc + 2 * k, id_s, k > 0);
        mma_commit(&B.s_full[gs & 1]);
        mma_commit(&B.k_empty[kb]);
        if (sc.j == sc.it.nb - 1) mma_commit(&B.q_empty[qb]);  // the item's last S has read its Q
        gs++;
        sc.next(args);
        return true;
      };
      if (pv.valid) {
        ok = load_q() && load_q() && load_k() && load_k() && load_k() && load_v() && load_v() && issue_s() &&
             issue_s();
        while (ok && pv.valid) {
          const int pb = g & 1;
          if (!mbar_wait(&B.p_full[pb], (g >> 1) & 1, abort, args.err) ||
              (pv.j == 0 && pv.k > 0 && !mbar_wait(B.o_free, (pv.k - 1) & 1, abort, args.err)) ||
              !mbar_wait(&B.v_full[g % VST], (g / VST) & 1, abort, args.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t v_desc = sw128_desc_mn(smem_u32(smem + OFF_V + (g % VST) * KV_BYTES));
          const uint32_t t_p = tmem + pb * 64 + 32;
#pragma unroll
          for (int k = 0; k < BKV / 16; k++)  // 16 keys per step: 8 TMEM columns of P, +2 KB in V
            mma_f16_ts(tmem + 128, t_p + 8 * k, v_desc + (uint64_t)k * (2048 >> 4), id_o, (pv.j > 0 || k > 0) ? 1u : 0u);
          mma_commit(&B.v_empty[g % VST]);
          mma_commit(B.pv_done);
          if (pv.j == pv.it.nb - 1) mma_commit(B.o_full);
          // S_{g+2} into the buffer PV_g just read (issued after it, so it runs after it).
          if (!(ok = issue_s())) break;
          g++;
          pv.next(args);
          // Refill: K two blocks ahead of S, V two ahead of PV, Q two items ahead.
          while (ok && kl.valid && gk < gs + 2) ok = load_k();
          while (ok && vl.valid && gv < g + 2) ok = load_v();
          while (ok && kq < pv.k + 2 && (int)blockIdx.x + kq * (int)gridDim.x < args.num_work) ok = load_q();
        }
      }
      if (*abort) {  // leaving early: the MMAs and loads issued so far land before TMEM is freed
        mma_commit(B.drain);
        mbar_drain(B.drain, 0);
        for (uint32_t i = gs; i < gk; i++) mbar_drain(&B.k_full[i % KST], (i / KST) & 1);
        for (uint32_t i = g; i < gv; i++) mbar_drain(&B.v_full[i % VST], (i / VST) & 1);
        // Q loads of items whose first S was not issued.
        for (int i = sc.valid ? sc.k + (sc.j > 0 ? 1 : 0) : kq; i < kq; i++) mbar_drain(&B.q_full[i & 1], (i >> 1) & 1);
      }
    }
  } else {
    const int q = warp & 3;        // TMEM lane quarter of this warp (warp id % 4)
    const int r = q * 32 + lane;   // query row within the tile
    const uint32_t t_row = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t t_o = t_row + 128;
    const float sl2 = args.sl2;
    uint32_t g = 0;
    int k = 0;
    for (int w = blockIdx.x; w < args.num_work; w += gridDim.x, ++k) {
      const Item it = decode_item(args, w);
      float m_ref = 0.f, l = 0.f;
      bool ok = true;
      const bool live = it.q0 + q * 32 < it.L;
      for (int j = 0; j < it.nb; j++, g++) {
        const uint32_t t_s = t_row + (g & 1) * 64, t_p = t_s + 32;
        if (!mbar_wait(&B.s_full[g & 1], (g >> 1) & 1, abort, args.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (!live) {  // rows past the sequence end: no softmax, no P (their O rows are never stored)
          tc_fence_before();
          mbar_arrive(&B.p_full[g & 1]);
          continue;
        }
        float sv[BKV];
        tmem_ld64(t_s, sv);
        const int valid = it.L - j * BKV;
        if (valid < BKV) mask_tail(sv, valid);
        if (j == 0) m_ref = sv[0];
        float rsum;
        uint32_t pk[32];
        exp_row<T, BKV>(sv, sl2, m_ref * sl2, pk, rsum);
        const bool need = !(rsum <= kPMax<T>());
        if (__any_sync(0xffffffffu, need)) {
          // Rare path (see attention_tc.cu): the reference max moves.  S_g is still intact (its
          // buffer is rewritten only after PV_g); O holds PV of blocks 0..j-1 of this item once
          // PV_{g-1} has completed.
          if (j > 0 && !mbar_wait(B.pv_done, (g - 1) & 1, abort, args.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tmem_ld64(t_s, sv);
          if (valid < BKV) mask_tail(sv, valid);
          const float mx = row_max(sv);
          float f = 1.0f;
          if (need) {
            f = ex2((m_ref - mx) * sl2);
            m_ref = mx;
            l *= f;
          }
          if (j > 0) {
#pragma unroll 1
            for (int hh = 0; hh < 2; hh++) {
              float ov[32];
              tmem_ld32(t_o + hh * 32, ov);
              uint32_t ou[32];
#pragma unroll
              for (int c = 0; c < 32; c++) ou[c] = __float_as_uint(ov[c] * f);
              tmem_st32(t_o + hh * 32, ou);
            }
          }
          tmem_ld64(t_s, sv);
          if (valid < BKV) mask_tail(sv, valid);
          exp_row<T, BKV>(sv, sl2, m_ref * sl2, pk, rsum);
        }
        tmem_st32(t_p, pk);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&B.p_full[g & 1]);
        l += rsum;
      }
      if (!ok || !mbar_wait(B.o_full, k & 1, abort, args.err)) break;
      tc_fence_after();
      if (!live) {
        tc_fence_before();
        mbar_arrive(B.o_free);
        continue;
      }
      float o[D];
      tmem_ld64(t_o, o);
      tc_fence_before();
      mbar_arrive(B.o_free);
      if (it.q0 + r < it.L) {
        const float inv = __frcp_rn(l);
        T* dst = reinterpret_cast<T*>(args.out) + (int64_t)(it.start + it.q0 + r) * args.ld_out + it.h * D;
        if (args.st256) {
#pragma unroll
          for (int c = 0; c < 4; c++) {
            const float* v = &o[c * 16];
            uint32_t u[8];
#pragma unroll
            for (int e = 0; e < 8; e++) u[e] = pack2<T>(v[2 * e] * inv, v[2 * e + 1] * inv);
            st_global_256(reinterpret_cast<uint8_t*>(dst) + c * 32, u);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 8; c++) {
            const float* v = &o[c * 8];
            reinterpret_cast<uint4*>(dst)[c] =
                make_uint4(pack2<T>(v[0] * inv, v[1] * inv), pack2<T>(v[2] * inv, v[3] * inv),
                           pack2<T>(v[4] * inv, v[5] * inv), pack2<T>(v[6] * inv, v[7] * inv));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

}  // namespace tcd

int32_t make_tma_map_2d(Ctx* c, CUtensorMap* m, int32_t dtype, const void* ptr, uint64_t rows, uint64_t cols,
                        uint64_t ld, uint32_t box_cols, uint32_t box_rows);

template <typename T>
static int32_t launch_db(Ctx* c, int32_t dt, const void* q, const void* k, const void* v, int64_t ld_in, int64_t T_,
                         int64_t H, void* out, int64_t ld_out, const int2* tiles128, int32_t num_tiles, int32_t nh,
                         float scale) {
  using namespace tcd;
  CUtensorMap mq, mk, mv;
  int32_t rc;
  if ((rc = make_tma_map_2d(c, &mq, dt, q, (uint64_t)T_, (uint64_t)H, (uint64_t)ld_in, D, BQ))) return rc;
  if ((rc = make_tma_map_2d(c, &mk, dt, k, (uint64_t)T_, (uint64_t)H, (uint64_t)ld_in, D, BKV))) return rc;
  if ((rc = make_tma_map_2d(c, &mv, dt, v, (uint64_t)T_, (uint64_t)H, (uint64_t)ld_in, D, BKV))) return rc;
  const int work = num_tiles * nh;
  const int st256 = ((uintptr_t)out & 31) == 0 && (ld_out * 2) % 32 == 0;
  DbArgs a{tiles128, work, nh, out, ld_out, scale * 1.4426950408889634f, c->d_err, st256};
  static std::atomic<bool> attr_set[64] = {};
  if (!attr_set[c->device & 63].load(std::memory_order_acquire)) {
    FL_CUDA(c, cudaFuncSetAttribute(k_attn_db<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    attr_set[c->device & 63].store(true, std::memory_order_release);
  }
  const int grid = work < 2 * c->num_sms ? work : 2 * c->num_sms;
  FL_CUDA(c, launch_pdl(k_attn_db<T>, dim3(grid), dim3(kThreads), SMEM, c->stream, mq, mk, mv, a));
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

int32_t launch_flash_attention_db(Ctx* c, int32_t dt, const void* q, const void* k, const void* v, int64_t ld_in,
                                  int64_t T, int64_t H, void* out, int64_t ld_out, const int2* tiles128,
                                  int32_t num_tiles, int32_t nh, float scale) {
  if (dt == FLETCHER_BF16)
    return launch_db<__nv_bfloat16>(c, dt, q, k, v, ld_in, T, H, out, ld_out, tiles128, num_tiles, nh, scale);
  return launch_db<__half>(c, dt, q, k, v, ld_in, T, H, out, ld_out, tiles128, num_tiles, nh, scale);
}

}  // namespace fl
