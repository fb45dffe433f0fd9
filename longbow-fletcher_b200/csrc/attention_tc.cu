// Flash attention on the 5th-generation tensor cores (tcgen05 / TMEM / TMA), bf16 or fp16,
// head_dim 64, packed variable-length sequences.
//
// Reference semantics: BertSelfAttention.ForwardBatch (bert.go:610-728) -> CPUTensor.Attention
// (cpu_backend.go:662-758): per sequence and head, O = softmax(scale * Q K^T) V, keys limited to
// the sequence (cu_seqlens).
//
// Persistent kernel, two query-tile slots per CTA and two CTAs per SM.  Each slot walks its own
// work items w = (128-query tile, head) in a strided order (tiles come longest-sequence first)
// through 64-key blocks.  320 threads:
//   warps 0-1 : control thread of slot 0 / slot 1 — TMA loads (Q tile per work item, K and V
//               blocks in a 2-stage ring; the next item's Q and first block are fetched during
//               the current item's last block) and MMA issue: S_j = Q K_j^T (M=128, N=64, K=64)
//               into the slot's TMEM S columns, then O += P_j V_j with P_j read from TMEM (A
//               operand) and V_j MN-major straight from its TMA tile.  tcgen05.mma runs in issue
//               order, so S_{j+1} may overwrite P_j's columns once PV_j has been issued;
//   warps 2-5 : softmax of slot 0, warps 6-9 softmax of slot 1 — thread = query row: tcgen05.ld
//               its S row, mask keys past the sequence end, exp2 against a lazily updated
//               reference max, and tcgen05.st P (16-bit pairs) over the upper half of S.  The
//               reference max starts at the row's first key and moves only when some P exceeds
//               2^64 (bf16; 2^15 for fp16), found from the block's largest P after the exps; then
//               O (complete, because S_j's commit follows PV_{j-1}) is rescaled in TMEM.  At the end of an item the row of O is divided by its sum and stored.
// TMEM per slot: S/P 64 columns + O 64 columns; 256 per CTA.  ~98 KB smem.  All mbarrier waits
// are bounded (device error flag + abort, as in the GEMM).  No multicast.
#include <atomic>

#include "attn_common.cuh"

namespace fl {
namespace tca {

using namespace tc;

constexpr int BQ = 128, D = 64;
constexpr int Q_BYTES = BQ * D * 2;
constexpr int kBarsPerSlot = 11;

// Kernel shape: BKV keys per block, SLOTS query-tile slots per CTA, two CTAs per SM.
//   BKV = 64,  SLOTS = 2: per slot S 64 columns (P over its upper 32), O 64 -> 4 slots per SM;
//   BKV = 128, SLOTS = 1: per slot S 128 columns (P over its upper 64), O 64 -> 2 slots per SM,
//     every MMA at N = 128 (full rate) for S and twice the softmax work per round trip.
template <int BKV_, int SLOTS_>
struct AttnCfg {
  static constexpr int BKV = BKV_, SLOTS = SLOTS_;
  static constexpr int kThreads = 32 * SLOTS + 128 * SLOTS;
  static constexpr int KV_BYTES = BKV * D * 2;
  // Per slot: Q, K[2], V[2] (each 1024-byte aligned).
  static constexpr int SLOT_Q = 0, SLOT_K = Q_BYTES, SLOT_V = Q_BYTES + 2 * KV_BYTES;
  static constexpr int SLOT_BYTES = Q_BYTES + 4 * KV_BYTES;
  static constexpr int OFF_BAR = SLOTS * SLOT_BYTES;
  static constexpr int SMEM = OFF_BAR + SLOTS * kBarsPerSlot * 8 + 16 + 1024;
  // TMEM per slot: S [0, BKV) with P (16-bit pairs) over its upper half, O [BKV, BKV + 64).
  static constexpr int SLOT_COLS = BKV + D;
  static constexpr int TMEM_COLS = 256;
  static_assert(SLOTS * SLOT_COLS <= TMEM_COLS, "TMEM columns");
};

struct AttnArgs {
  const int32_t* cu;
  const int2* tiles;
  int num_work;  // tiles * heads
  int nh;
  void* out;
  int64_t ld_out;
  float sl2;  // scale * log2(e)
  int32_t* err;
  int st256;  // output rows 32-byte aligned: 256-bit stores
};

struct Work {
  int start, L, q0, h, nb;
};

// Barriers of one slot.
struct SlotBars {
  uint64_t *q_full, *q_empty, *kv_full, *kv_empty, *s_full, *p_full, *o_full, *o_free, *drain;
  __device__ SlotBars(uint64_t* b)
      : q_full(b), q_empty(b + 1), kv_full(b + 2), kv_empty(b + 4), s_full(b + 6), p_full(b + 7), o_full(b + 8),
        o_free(b + 9), drain(b + 10) {}
};

template <int BKV>
__device__ __forceinline__ Work decode(const AttnArgs& a, int w) {
  const int2 t = a.tiles[w / a.nh];
  Work r;
  r.h = w % a.nh;
  r.start = t.x;
  r.L = (int)((uint32_t)t.y >> 16);
  r.q0 = t.y & 0xFFFF;
  r.nb = (r.L + BKV - 1) / BKV;
  return r;
}

template <typename T, int BKV_, int SLOTS_>
__global__ void __launch_bounds__(AttnCfg<BKV_, SLOTS_>::kThreads, 2)
    k_attn_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  using C = AttnCfg<BKV_, SLOTS_>;
  constexpr int BKV = C::BKV, kSlots = C::SLOTS, KV_BYTES = C::KV_BYTES;
  constexpr int SLOT_Q = C::SLOT_Q, SLOT_K = C::SLOT_K, SLOT_V = C::SLOT_V, SLOT_BYTES = C::SLOT_BYTES;
  constexpr int OFF_BAR = C::OFF_BAR, TMEM_COLS = C::TMEM_COLS, SLOT_COLS = C::SLOT_COLS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kSlots * kBarsPerSlot);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vstride = gridDim.x * kSlots;  // virtual slots in the grid

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; s++) {
      SlotBars B(bars + s * kBarsPerSlot);
      mbar_init(B.q_full, 1);
      mbar_init(B.q_empty, 1);
      for (int i = 0; i < 2; i++) {
        mbar_init(&B.kv_full[i], 1);
        mbar_init(&B.kv_empty[i], 1);
      }
      mbar_init(B.s_full, 1);
      mbar_init(B.p_full, 128);
      mbar_init(B.o_full, 1);
      mbar_init(B.o_free, 128);
      mbar_init(B.drain, 1);
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
  pdl_wait();  // the setup above overlapped the previous kernel; its outputs are visible now

  if (warp < kSlots) {
    // Control thread of slot `warp`: TMA loads and MMA issue with sleeping bounded waits.
    if (lane == 0) {
      const int s = warp;
      SlotBars B(bars + s * kBarsPerSlot);
      uint8_t* sb = smem + s * SLOT_BYTES;
      const uint32_t t_s = tmem + s * SLOT_COLS, t_p = t_s + BKV / 2, t_o = t_s + BKV;
      const uint32_t id_s = idesc<T, BQ, BKV>();
      const uint32_t id_o = idesc<T, BQ, D, true>();
      uint32_t gl = 0, gc = 0, gs = 0;  // K/V blocks loaded, K/V blocks consumed, S blocks
      uint32_t qn = 0, qw = 0;          // Q tiles loaded, Q tiles waited for
      auto load_q = [&](const Work& wk, uint32_t t) -> bool {
        if (!mbar_wait(B.q_empty, (t & 1) ^ 1, abort, args.err)) return false;
        mbar_expect_tx(B.q_full, Q_BYTES);
        tma_load_2d(sb + SLOT_Q, &tmQ, B.q_full, wk.h * D, wk.start + wk.q0);
        qn++;
        return true;
      };
      auto load_kv = [&](const Work& wk, int j) -> bool {
        const int b = gl & 1;
        if (!mbar_wait(&B.kv_empty[b], ((gl >> 1) & 1) ^ 1, abort, args.err)) return false;
        mbar_expect_tx(&B.kv_full[b], 2 * KV_BYTES);
        tma_load_2d(sb + SLOT_K + b * KV_BYTES, &tmK, &B.kv_full[b], wk.h * D, wk.start + j * BKV);
        tma_load_2d(sb + SLOT_V + b * KV_BYTES, &tmV, &B.kv_full[b], wk.h * D, wk.start + j * BKV);
        gl++;
        return true;
      };
      auto issue_s = [&]() -> bool {  // S = Q K^T for the next block in consumption order
        const int b = gc & 1;
        if (!mbar_wait(&B.kv_full[b], (gc >> 1) & 1, abort, args.err)) return false;
        tc_fence_after();
        const uint64_t q_desc = sw128_desc(smem_u32(sb + SLOT_Q));
        const uint64_t k_desc = sw128_desc(smem_u32(sb + SLOT_K + b * KV_BYTES));
#pragma unroll
        for (int k = 0; k < D / 16; k++) mma_f16(t_s, q_desc + 2 * k, k_desc + 2 * k, id_s, k > 0);
        mma_commit(B.s_full);
        return true;
      };
      int w = blockIdx.x * kSlots + s;
      if (w < args.num_work) {
        Work cur = decode<BKV>(args, w);
        int nl = 1;  // blocks of `cur` whose loads were issued
        bool ok = load_q(cur, 0) && load_kv(cur, 0);
        for (uint32_t t = 0; ok; t++) {
          const int wn = w + vstride;
          const bool has_next = wn < args.num_work;
          Work nxt{};
          if (has_next) nxt = decode<BKV>(args, wn);
          if (!mbar_wait(B.q_full, t & 1, abort, args.err)) break;
          qw++;
          if (!issue_s()) break;
          if (cur.nb == 1) mma_commit(B.q_empty);  // Q free once the item's last S ran
          if (nl < cur.nb && !(ok = load_kv(cur, nl++))) break;
          for (int j = 0; j < cur.nb && ok; j++) {
            if (j == cur.nb - 1 && has_next && !(ok = load_q(nxt, t + 1) && load_kv(nxt, 0))) break;
            if (!mbar_wait(B.p_full, gs & 1, abort, args.err) ||
                (j == 0 && !mbar_wait(B.o_free, (t & 1) ^ 1, abort, args.err))) {  // previous item's O read
              ok = false;
              break;
            }
            tc_fence_after();
            const int b = gc & 1;
            const uint64_t v_desc = sw128_desc_mn(smem_u32(sb + SLOT_V + b * KV_BYTES));
#pragma unroll
            for (int k = 0; k < BKV / 16; k++)  // 16 keys per step: 8 TMEM columns of P, +2 KB in V
              mma_f16_ts(t_o, t_p + 8 * k, v_desc + (uint64_t)k * (2048 >> 4), id_o, (j > 0 || k > 0) ? 1u : 0u);
            mma_commit(&B.kv_empty[b]);
            gc++;
            gs++;
            if (j + 1 < cur.nb) {
              if (!(ok = issue_s())) break;
              if (j + 2 == cur.nb) mma_commit(B.q_empty);
              if (nl < cur.nb && !(ok = load_kv(cur, nl++))) break;
            }
          }
          if (!ok) break;
          mma_commit(B.o_full);
          if (!has_next) break;
          w = wn;
          cur = nxt;
          nl = 1;
        }
      }
      if (*abort) {  // leaving early: this slot's MMAs and loads land before TMEM is freed
        mma_commit(B.drain);
        mbar_drain(B.drain, 0);
        for (uint32_t i = gc; i < gl; i++) mbar_drain(&B.kv_full[i & 1], (i >> 1) & 1);
        if (qn > qw) mbar_drain(B.q_full, (qn - 1) & 1);
      }
    }
  } else {
    const int s = (warp - kSlots) >> 2;
    const int q = warp & 3;  // a warp reaches TMEM lanes 32 * (warp id % 4) ..
    const int r = q * 32 + lane;  // query row within the tile
    SlotBars B(bars + s * kBarsPerSlot);
    const uint32_t t_s = tmem + ((uint32_t)(q * 32) << 16) + s * SLOT_COLS, t_p = t_s + BKV / 2, t_o = t_s + BKV;
    const float sl2 = args.sl2;
    uint32_t gs = 0, t = 0;
    int w = blockIdx.x * kSlots + s;
    Work nxt{};
    if (w < args.num_work) nxt = decode<BKV>(args, w);
    for (; w < args.num_work; w += vstride, ++t) {
      const Work wk = nxt;
      // The next item's descriptor is fetched now; its loads complete during this item.
      if (w + vstride < args.num_work) nxt = decode<BKV>(args, w + vstride);
      float m_ref = 0.f, l = 0.f;
      bool ok = true;
      // A warp whose 32 query rows all lie past the sequence end (the tail of its last tile)
      // skips the softmax: its P and O rows are never stored.  It still follows S_full (S_{j+1}
      // comes only after PV_j has read P_j) and arrives on every barrier, keeping the phases.
      const bool live = wk.q0 + q * 32 < wk.L;
      for (int j = 0; j < wk.nb; j++, gs++) {
        if (!mbar_wait(B.s_full, gs & 1, abort, args.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (!live) {
          tc_fence_before();
          mbar_arrive(B.p_full);
          continue;
        }
        float sv[BKV];
        tmem_ld_row<BKV>(t_s, sv);
        const int valid = wk.L - j * BKV;  // keys of this block inside the sequence (>= 1)
        if (valid < BKV) mask_tail(sv, valid);
        // P against the current reference max (for block 0: the row's first key, which is never
        // above the row max, so the dominant terms cannot underflow); the block max is checked
        // afterwards through the largest P.
        if (j == 0) m_ref = sv[0];
        float rsum;
        uint32_t pk[BKV / 2];
        exp_row<T, BKV>(sv, sl2, m_ref * sl2, pk, rsum);
        // The row sum bounds every P of the row, so a sum within the P range proves that no P
        // left it (a NaN fails the test too).  A sum beyond the range with every P inside it only
        // costs a needless rescale.
        const bool need = !(rsum <= kPMax<T>());
        if (__any_sync(0xffffffffu, need)) {
          // Rare path: some row's max moved by more than the P range allows.  S is still in
          // TMEM (P is not written yet); O holds PV_0..PV_{j-1} complete (S_j's commit came
          // after PV_{j-1}).
          tmem_ld_row<BKV>(t_s, sv);
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
          tmem_ld_row<BKV>(t_s, sv);
          if (valid < BKV) mask_tail(sv, valid);
          exp_row<T, BKV>(sv, sl2, m_ref * sl2, pk, rsum);
        }
        tmem_st_p<BKV>(t_p, pk);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(B.p_full);
        l += rsum;
      }
      if (!ok || !mbar_wait(B.o_full, t & 1, abort, args.err)) break;
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
      if (wk.q0 + r < wk.L) {
        const float inv = __frcp_rn(l);
        T* dst = reinterpret_cast<T*>(args.out) + (int64_t)(wk.start + wk.q0 + r) * args.ld_out + wk.h * D;
        if (args.st256) {  // four 32-byte stores: one full sector per lane
#pragma unroll
          for (int c = 0; c < 4; c++) {
            const float* v = &o[c * 16];
            uint32_t u[8];
#pragma unroll
            for (int k = 0; k < 8; k++) u[k] = pack2<T>(v[2 * k] * inv, v[2 * k + 1] * inv);
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
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

}  // namespace tca

int32_t make_tma_map_2d(Ctx* c, CUtensorMap* m, int32_t dtype, const void* ptr, uint64_t rows, uint64_t cols,
                        uint64_t ld, uint32_t box_cols, uint32_t box_rows);

template <typename T, int BKV, int SLOTS>
static int32_t launch_attn_variant(Ctx* c, int32_t dt, const void* q, const void* k, const void* v, int64_t ld_in,
                                   int64_t T_, int64_t H, void* out, int64_t ld_out, const int32_t* cu,
                                   const int2* tiles128, int32_t num_tiles, int32_t nh, float scale) {
  using namespace tca;
  using C = AttnCfg<BKV, SLOTS>;
  CUtensorMap mq, mk, mv;
  int32_t rc;
  if ((rc = make_tma_map_2d(c, &mq, dt, q, (uint64_t)T_, (uint64_t)H, (uint64_t)ld_in, D, BQ))) return rc;
  if ((rc = make_tma_map_2d(c, &mk, dt, k, (uint64_t)T_, (uint64_t)H, (uint64_t)ld_in, D, BKV))) return rc;
  if ((rc = make_tma_map_2d(c, &mv, dt, v, (uint64_t)T_, (uint64_t)H, (uint64_t)ld_in, D, BKV))) return rc;
  const int work = num_tiles * nh;
  const int st256 = ((uintptr_t)out & 31) == 0 && (ld_out * 2) % 32 == 0;
  AttnArgs a{cu, tiles128, work, nh, out, ld_out, scale * 1.4426950408889634f, c->d_err, st256};
  // Per device; host threads of several replicas may get here at once (idempotent).
  static std::atomic<bool> attr_set[64] = {};
  if (!attr_set[c->device & 63].load(std::memory_order_acquire)) {
    FL_CUDA(c, cudaFuncSetAttribute(k_attn_tc<T, BKV, SLOTS>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set[c->device & 63].store(true, std::memory_order_release);
  }
  const int want = (work + SLOTS - 1) / SLOTS;
  const int grid = want < 2 * c->num_sms ? want : 2 * c->num_sms;
  FL_CUDA(c, launch_pdl(k_attn_tc<T, BKV, SLOTS>, dim3(grid), dim3(C::kThreads), C::SMEM, c->stream, mq, mk, mv, a));
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

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
  // 64-key blocks, two slots per CTA, two CTAs per SM.  Two other shapes measured slower, A/B on
  // one box at 1.91-1.97 GHz (attention ms per cfg3 step): 128-key blocks with one slot per CTA
  // (N = 128 MMAs for S, half the slots per SM) 2.70-2.75 against 2.24-2.30; two query tiles of a
  // sequence sharing each K/V block with P in shared memory and S_{j+1} issued before PV_j, one
  // control thread for both tiles, 3.10 against 2.30-2.32; one slot per CTA with S double-buffered
  // in TMEM (S_{j+2} issued right after PV_j, so the softmax never waits for S) 3.25-3.28 against
  // 2.28-2.29: with half the slots per SM the softmax warps, not the S round trip, set the pace;
  // eight softmax warps per slot, two per TMEM lane quarter each taking half of a row's keys (their
  // halves meeting through a pair mbarrier), 2.75-2.78 against 2.27; the exponentials as
  // ex2.approx.f16x2 (half the MUFU instructions, fp16 exponents, P range 2^15) 2.56-2.63 against
  // 2.27-2.30: the extra conversions cost more than the MUFU time saved.
  if (dt == FLETCHER_BF16)
    return launch_attn_variant<__nv_bfloat16, 64, 2>(c, dt, q, k, v, ld_in, T, H, out, ld_out, cu, tiles128, num_tiles,
                                                     nh, scale);
  return launch_attn_variant<__half, 64, 2>(c, dt, q, k, v, ld_in, T, H, out, ld_out, cu, tiles128, num_tiles, nh,
                                            scale);
}

}  // namespace fl
