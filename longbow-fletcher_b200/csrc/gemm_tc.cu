// tcgen05 / TMEM / TMA GEMM for sm_100a: out = epilogue(A[M,K] . W[N,K]^T).
//
// The dense contractions of the encoder (QKV, attention output, FFN up and down; the
// reference's Linear -> mulBLAS, cpu_backend.go:350-372, and Cuda_Linear_Fused,
// cuda_backend.cu:65-92) run here in bf16 or fp16 with fp32 accumulation in tensor memory.
//
// Layout: A is the activation, row-major [M, K] (K contiguous).  W is the weight packed
// K-major [N, K] at model load (the reference stores Linear weights (in, out) = [K, N]).
// Both are fetched by TMA in 128-byte-swizzled 64-wide K slabs.
//
// Kernel structure (persistent, one CTA per SM, 320 threads):
//   warp 0   : TMA producer — one thread streams A/W slabs into a STAGES-deep smem ring;
//   warp 1   : MMA issuer — one thread issues tcgen05.mma (M=128, N=BN, K=16) into one of two
//              TMEM accumulators and commits to mbarriers; the warp also owns TMEM alloc;
//   warps 2-9: epilogue — for store / RoPE / GELU two groups of four warps take alternate
//              tiles (accumulator 0 / 1), for residual / SwiGLU warps 2-5 and 6-9 take the
//              two column halves of every tile; warp w reads TMEM lane quarter w%4 with
//              tcgen05.ld, applies bias /
//              RoPE / GELU / SwiGLU / residual in registers, writes 32x64 output boxes into a
//              per-warp 128B-swizzled smem buffer and stores them with TMA bulk-tensor stores
//              (full-line, asynchronous writes instead of per-thread 16-byte row stores).
// Two accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
// Every mbarrier wait is bounded: on expiry the kernel records an error in a device flag,
// raises a CTA-wide abort flag and all roles leave their loops.
// No TMA multicast is used.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <atomic>
#include <mutex>

#include "gemm.cuh"
#include "tc_common.cuh"

namespace fl {
namespace tc {

constexpr int BM = 128, BK = 64;
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;            // + producer warp + MMA warp
constexpr int kStageOut = 32 * 128;                    // per-warp output box: 32 rows x 64 cols x 2 B
// Epilogues drained by alternating warp groups (see the epilogue section of k_gemm_tc).
template <int EPI>
constexpr bool kEpiGroups = EPI == 0 || EPI == 1 || EPI == 2 || EPI == 5;  // STORE, ROPE, GELU, PARTIAL
// Output boxes per warp: two where a warp writes four boxes per tile (the groups) and for the
// TMA-residual epilogue (one per 64-column unit: each box arrives holding the residual rows and
// leaves holding the sums); one for the register-residual and SwiGLU epilogues, whose shared
// memory goes to an extra operand stage.
template <int EPI>
constexpr int kOutBufs = kEpiGroups<EPI> || EPI == 6 ? 2 : 1;
// Both residual epilogues: out = acc + bias + residual.
template <int EPI>
constexpr bool kResidual = EPI == 4 || EPI == 6;

// PAIR: the tile is computed by a cluster of two CTAs on two SMs with tcgen05 cta_group::2
// (M = 256 per MMA): each CTA loads its 128 rows of A and half of the tile's BN rows of W, and
// holds its 128 rows of the accumulator.  Per SM that is a third less operand traffic than a
// 128 x 256 tile on one SM.
template <int BN, bool PAIR, int OUT_BUFS>
struct Cfg {
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows of W loaded by one CTA
  static constexpr int TILE_M = PAIR ? 2 * BM : BM;  // rows of a tile
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int OUT_BYTES = kEpiWarps * OUT_BUFS * kStageOut;
  // As many operand stages as fit next to the output staging (at most 8).
  static constexpr int STAGES_FIT = (232448 - 1024 - 384 - OUT_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT < 8 ? STAGES_FIT : 8;
  static constexpr int OUT_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = OUT_OFF + OUT_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = BAR_OFF + 384 /*barriers*/ + 1024 /*alignment slack*/;
  static_assert((2 * STAGES + 7 + 2 * kEpiWarps) * 8 <= 384, "barrier area");
  static_assert(SMEM <= 232448, "shared memory budget");
};


// Writes this lane's row (64 values: a = columns 0-31, b = 32-63) of a 32x64 output box into
// the warp's staging buffer in the TMA 128-byte swizzle layout: 16-byte chunk j of row r sits
// at r*128 + (j ^ (r & 7))*16.
template <typename T>
__device__ __forceinline__ void stage_row(uint8_t* buf, int r, const float (&a)[32], const float (&b)[32]) {
  uint8_t* row = buf + r * 128;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const float* v = j < 4 ? &a[j * 8] : &b[(j - 4) * 8];
    uint4 w = make_uint4(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]), pack2<T>(v[4], v[5]), pack2<T>(v[6], v[7]));
    *reinterpret_cast<uint4*>(row + ((j ^ (r & 7)) << 4)) = w;
  }
}

// v[i] += the 32 16-bit values in q[0..3].
// stage_row with the box's current contents (this row's 64 residual values, as TMA loaded
// them) added: row = a|b + residual, in place.
template <typename T>
__device__ __forceinline__ void add_packed(float (&v)[32], const uint4* q4) {
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint4 q = q4[i];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
        v[8 * i + 2 * j] += f.x;
        v[8 * i + 2 * j + 1] += f.y;
      } else {
        float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
        v[8 * i + 2 * j] += f.x;
        v[8 * i + 2 * j + 1] += f.y;
      }
    }
  }
}

template <typename T>
__device__ __forceinline__ void stage_row_add(uint8_t* buf, int r, const float (&a)[32], const float (&b)[32]) {
  uint8_t* row = buf + r * 128;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const float* v = j < 4 ? &a[j * 8] : &b[(j - 4) * 8];
    uint4* p = reinterpret_cast<uint4*>(row + ((j ^ (r & 7)) << 4));
    const uint4 q = *p;
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    float f[8];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      float2 t;
      if constexpr (std::is_same<T, __nv_bfloat16>::value)
        t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
      else
        t = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
      f[2 * k] = v[2 * k] + t.x;
      f[2 * k + 1] = v[2 * k + 1] + t.y;
    }
    *p = make_uint4(pack2<T>(f[0], f[1]), pack2<T>(f[2], f[3]), pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
  }
}

template <typename T, int BN, int EPI, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR, const GemmArgs args) {
  using C = Cfg<BN, PAIR, kOutBufs<EPI>>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::STAGES;
  uint64_t* tfull = bars + 2 * C::STAGES;
  uint64_t* tempty = bars + 2 * C::STAGES + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * C::STAGES + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
  uint64_t* rbar = bars + 2 * C::STAGES + 6;  // residual box loaded: one per epilogue warp and box
  uint64_t* drain = rbar + 2 * kEpiWarps;      // an aborting MMA thread's issued MMAs are complete

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = args.num_n_tiles;
  const int splits = args.splits;  // K ranges per output tile (split-K partial sums)
  const int num_tiles = args.num_m_tiles * n_tiles * splits;
  const int num_kb = args.K / BK;
  auto kb_range = [&](int tile, int& kb0, int& kb1) {
    kb0 = (tile % splits) * args.kb_per;
    kb1 = kb0 + args.kb_per < num_kb ? kb0 + args.kb_per : num_kb;
  };
  // Pair mode: clusters of two consecutive CTAs; CTA rank 0 issues the MMAs.
  const uint32_t crank = PAIR ? cluster_ctarank() : 0;
  const int first_tile = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tile_stride = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tfull[i], 1);
      // One arrival per draining warp (of both CTAs).
      mbar_init(&tempty[i], (kEpiGroups<EPI> ? kEpiWarps / 2 : kEpiWarps) * (PAIR ? 2 : 1));
    }
    *abort = 0;
    mbar_init(drain, 1);
    if constexpr (EPI == EPI_RESIDUAL_TMA)
      for (int i = 0; i < 2 * kEpiWarps; i++) mbar_init(&rbar[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmC) : "memory");
    if constexpr (EPI == EPI_RESIDUAL_TMA) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmR) : "memory");
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                   "r"(C::TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                   "r"(C::TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // both CTAs' barriers are initialised before any cross-CTA signal
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_wait();  // the setup above overlapped the previous kernel; its outputs are visible now

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_par = 0;  // per stage: loaded at least once; parity of the last load
      for (int tile = first_tile; tile < num_tiles; tile += tile_stride) {
        const int mb = tile / splits / n_tiles, nb = tile / splits % n_tiles;
        int kb0, kb1;
        kb_range(tile, kb0, kb1);
        const int a_row = mb * C::TILE_M + (int)crank * BM;
        const int b_row = nb * BN + (int)crank * C::B_ROWS;
        for (int kb = kb0; kb < kb1; kb++) {
          if (!mbar_wait_spin(&empty[stage], phase ^ 1, abort, args.err)) goto producer_done;
          if constexpr (PAIR) {
            // Both CTAs' loads complete on the even CTA's barrier, which expects both.
            if (crank == 0) mbar_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            tma_load_2d_pair(sA + stage * C::A_BYTES, &tmA, fb, kb * BK, a_row);
            tma_load_2d_pair(sB + stage * C::B_BYTES, &tmB, fb, kb * BK, b_row);
          } else {
            mbar_expect_tx(&full[stage], C::STAGE_BYTES);
            tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * BK, a_row);
            tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BK, b_row);
          }
          issued |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:
      // Aborting: the operand loads still in flight land before the CTA exits.  In pair mode
      // both CTAs' loads complete on the even CTA's barriers, which that CTA drains.
      if (*abort && crank == 0)
        for (int s = 0; s < C::STAGES; s++)
          if ((issued >> s) & 1) mbar_drain(&full[s], (issued_par >> s) & 1);
      // The odd CTA cannot see its own loads complete (they signal the even CTA's barriers).
      // It needs no wait of its own: the even CTA's producer drains both CTAs' loads above
      // before its threads reach the final cluster barrier, and the odd CTA cannot pass that
      // barrier (or free anything) until they do.
    }
  } else if (warp == 1) {
    if (lane == 0 && crank == 0) {
      const uint32_t id = idesc<T, C::TILE_M, BN>();
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = first_tile; tile < num_tiles; tile += tile_stride, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait_spin(&tempty[acc], acc_phase ^ 1, abort, args.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        int kb0, kb1;
        kb_range(tile, kb0, kb1);
        for (int kb = kb0; kb < kb1; kb++) {
          if (!mbar_wait_spin(&full[stage], phase, abort, args.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_desc = sw128_desc(smem_u32(sA + stage * C::A_BYTES));
          const uint64_t b_desc = sw128_desc(smem_u32(sB + stage * C::B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; k++) {  // +32 bytes per K=16 step inside the swizzle atom
            if constexpr (PAIR)
              mma_f16_pair(d_tmem, a_desc + 2 * k, b_desc + 2 * k, id, (kb > kb0 || k > 0) ? 1u : 0u);
            else
              mma_f16(d_tmem, a_desc + 2 * k, b_desc + 2 * k, id, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          if constexpr (PAIR)
            mma_commit_pair(&empty[stage]);  // frees the stage in both CTAs
          else
            mma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (PAIR)
          mma_commit_pair(&tfull[acc]);
        else
          mma_commit(&tfull[acc]);
      }
      if (*abort) {  // the MMAs issued so far complete before TMEM is freed
        if constexpr (PAIR)
          mma_commit_pair(drain);
        else
          mma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
  } else {
    // Epilogue.  Warp w reads TMEM lanes [32*(w%4), 32*(w%4)+32): rows q*32.. of the tile.
    // GROUPS (store / RoPE / GELU): two groups of four warps take alternate tiles (group g
    // always drains accumulator g), so each group has two tiles' worth of MMA time for its tile
    // and one group's RoPE-table latency overlaps the other's work.  Otherwise (residual,
    // SwiGLU, whose per-unit loads or math want fewer units per warp) all eight warps drain
    // every tile, warps 2-5 the first half of its columns and warps 6-9 the second.
    constexpr bool GROUPS = kEpiGroups<EPI>;
    const int q = warp & 3;
    const int grp = GROUPS ? (warp - 2) >> 2 : 0;
    const int col0 = GROUPS ? 0 : ((warp - 2) >> 2) * (EPI == EPI_SWIGLU ? 64 : BN / 2);
    uint8_t* stg0 = smem + C::OUT_OFF + (warp - 2) * kOutBufs<EPI> * kStageOut;
    int ob = 0;  // output buffer of the next box
    uint32_t rph = 0;    // residual: phase bit of each box's load barrier
    uint32_t rpend = 0;  // residual: boxes whose load is issued and not yet waited for
    // 64-column output units per warp: SwiGLU halves the width (BN/2 outputs per tile).
    constexpr int UNITS = (EPI == EPI_SWIGLU ? BN / 128 : BN / 64) / (GROUPS ? 1 : 2);
    const int tstep = GROUPS ? 2 : 1;
    const int64_t n_out = EPI == EPI_SWIGLU ? args.N / 2 : args.N;
    int it = grp;
    const uint32_t tempty_lead = PAIR ? mapa_shared(smem_u32(tempty), 0) : 0;
    auto tile_row = [&](int t) -> int64_t {
      return (int64_t)(t / splits / n_tiles) * C::TILE_M + (int)crank * BM + q * 32 + lane;
    };
    // RoPE positions run one tile ahead, so a tile's table loads need no dependent load.
    const int t0 = first_tile + grp * tile_stride;
    int pos_next = 0;
    if constexpr (EPI == EPI_ROPE) {
      if (t0 < num_tiles && tile_row(t0) < args.M) pos_next = args.pos[tile_row(t0)];
    }
    for (int tile = t0; tile < num_tiles; tile += tstep * tile_stride, it += tstep) {
      const int mb = tile / splits / n_tiles, nb = tile / splits % n_tiles;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int row0 = mb * C::TILE_M + (int)crank * BM + q * 32;
      const int64_t row = (int64_t)row0 + lane;
      const bool row_ok = row < args.M;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      // RoPE: every 64-wide head of this row uses the same cos/sin (same position, same
      // frequencies), so the row's table entries are loaded once per tile, not once per head;
      // they are requested before the wait for the accumulator.
      float rc[EPI == EPI_ROPE ? 32 : 1], rs[EPI == EPI_ROPE ? 32 : 1];
      if constexpr (EPI == EPI_ROPE) {
        const int p = pos_next;
        const int nt = tile + tstep * tile_stride;
        if (nt < num_tiles && tile_row(nt) < args.M) pos_next = args.pos[tile_row(nt)];
        if (row_ok && (int64_t)nb * BN < args.rope_cols) {
          const float4* ct = reinterpret_cast<const float4*>(args.cos_t + (int64_t)p * 32);
          const float4* st = reinterpret_cast<const float4*>(args.sin_t + (int64_t)p * 32);
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const float4 cv = __ldg(ct + i), sv = __ldg(st + i);
            rc[4 * i] = cv.x; rc[4 * i + 1] = cv.y; rc[4 * i + 2] = cv.z; rc[4 * i + 3] = cv.w;
            rs[4 * i] = sv.x; rs[4 * i + 1] = sv.y; rs[4 * i + 2] = sv.z; rs[4 * i + 3] = sv.w;
          }
        }
      }
      // Register residual: each unit's 128 bytes of the row are requested before its
      // accumulator load (the first unit's before the wait for the accumulator).
      uint4 res[EPI == EPI_RESIDUAL ? 8 : 1];
      auto load_res = [&](int u) {
        if constexpr (EPI == EPI_RESIDUAL) {
          const int64_t oc = (int64_t)nb * BN + col0 + u * 64;
          if (row_ok && oc < args.N) {
            const uint4* rp =
                reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(args.residual) + row * args.ld_res + oc);
#pragma unroll
            for (int i = 0; i < 8; i++) res[i] = rp[i];
          }
        }
      };
      load_res(0);
      // TMA residual: unit u's 32 x 64 box of the residual rows is loaded into the warp's output
      // box u (free once the previous tile's stores have read it) before the wait for the
      // accumulator; the sums are added into the box in place and stored from it.  Coalesced,
      // and no row-per-lane loads through L1.
      if constexpr (EPI == EPI_RESIDUAL_TMA) {
        if (lane == 0) bulk_wait_read0();
        if (row0 < args.M) {
#pragma unroll
          for (int u = 0; u < UNITS; u++) {
            const int64_t oc = (int64_t)nb * BN + col0 + u * 64;
            if (oc < args.N) {
              rpend |= 1u << u;
              if (lane == 0) {
                uint64_t* rb = &rbar[(warp - 2) * 2 + u];
                mbar_expect_tx(rb, kStageOut);
                tma_load_2d(stg0 + u * kStageOut, &tmR, rb, (int)oc, row0);
              }
            }
          }
        }
        __syncwarp();
      }
      if (!mbar_wait_spin(&tfull[acc], acc_phase, abort, args.err)) break;
      tc_fence_after();
#pragma unroll 1
      for (int u = 0; u < UNITS; u++) {
        float a[32], b[32];
        int64_t ocol;
        if constexpr (EPI == EPI_SWIGLU) {
          // Tile columns [0, BN/2) hold gate rows, [BN/2, BN) the matching up rows; this unit
          // produces output columns [col0 + u*64, col0 + u*64 + 64) of the tile's BN/2.
          const int g0 = col0 + u * 64;  // gate column within the tile
          float g[32], v[32];
          tmem_ld32x2(tbase + g0, tbase + BN / 2 + g0, g, v);
          const int pcol = nb * BN + g0;
          if (args.bias) {
#pragma unroll
            for (int i = 0; i < 32; i++) {
              g[i] += args.bias[pcol + i];
              v[i] += args.bias[pcol + BN / 2 + i];
            }
          }
#pragma unroll
          for (int i = 0; i < 32; i++) a[i] = __fdividef(g[i], 1.0f + __expf(-g[i])) * v[i];
          tmem_ld32x2(tbase + g0 + 32, tbase + BN / 2 + g0 + 32, g, v);
          if (args.bias) {
#pragma unroll
            for (int i = 0; i < 32; i++) {
              g[i] += args.bias[pcol + 32 + i];
              v[i] += args.bias[pcol + BN / 2 + 32 + i];
            }
          }
#pragma unroll
          for (int i = 0; i < 32; i++) b[i] = __fdividef(g[i], 1.0f + __expf(-g[i])) * v[i];
          ocol = (int64_t)nb * (BN / 2) + g0;
        } else {
          const int c0 = col0 + u * 64;  // first column of the unit within the tile
          ocol = (int64_t)nb * BN + c0;
          if (u > 0) load_res(u);
          tmem_ld32x2(tbase + c0, a, b);
          if (ocol < args.N) {
            if (args.bias) {
#pragma unroll
              for (int i = 0; i < 32; i++) {
                a[i] += args.bias[ocol + i];
                b[i] += args.bias[ocol + 32 + i];
              }
            }
            if constexpr (EPI == EPI_ROPE) {
              // Rotate-half on a 64-wide head: (x1, x2) = (a, b).
              if (ocol < args.rope_cols && row_ok) {
#pragma unroll
                for (int i = 0; i < 32; i++) {
                  const float x1 = a[i], x2 = b[i];
                  a[i] = x1 * rc[i] - x2 * rs[i];
                  b[i] = x1 * rs[i] + x2 * rc[i];
                }
              }
            }
            if constexpr (EPI == EPI_GELU) {
#pragma unroll
              for (int i = 0; i < 32; i++) {
                a[i] = gelu_fast16(a[i]);
                b[i] = gelu_fast16(b[i]);
              }
            }
            if constexpr (EPI == EPI_RESIDUAL) {
              if (row_ok) {
                add_packed<T>(a, res);
                add_packed<T>(b, res + 4);
              }
            }
          }
        }
        if (u == UNITS - 1) {  // every TMEM read of this tile is done: release the accumulator
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR)
              mbar_arrive_cluster(tempty_lead + acc * 8);  // the even CTA's MMA waits for both CTAs
            else
              mbar_arrive(&tempty[acc]);
          }
        }
        if constexpr (EPI == EPI_PARTIAL) {  // fp32 sums of this K range, 8 x 32-byte stores
          if (ocol < args.N && row_ok) {
            float* dst = args.partial + ((int64_t)(tile % splits) * args.M + row) * args.N + ocol;
#pragma unroll
            for (int c = 0; c < 8; c++) {
              const float* v = c < 4 ? &a[c * 8] : &b[(c - 4) * 8];
              asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst + c * 8), "f"(v[0]),
                           "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
                           : "memory");
            }
          }
        } else if (ocol < n_out && row0 < args.M) {
          uint8_t* stg = stg0 + ob * kStageOut;
          if constexpr (EPI == EPI_RESIDUAL_TMA) {  // box u holds this unit's residual rows
            stg = stg0 + u * kStageOut;
            if (!mbar_wait_spin(&rbar[(warp - 2) * 2 + u], (rph >> u) & 1, abort, args.err)) break;
            rph ^= 1u << u;
            rpend &= ~(1u << u);
            stage_row_add<T>(stg, lane, a, b);
          } else {
            if (lane == 0) {  // the box stored from this buffer has left it
              if constexpr (kOutBufs<EPI> == 2)
                bulk_wait_read1();
              else
                bulk_wait_read0();
            }
            __syncwarp();
            stage_row<T>(stg, lane, a, b);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            // rows >= M are clipped by TMA; the residual sum is kept in L2 for the LayerNorm after it
            if constexpr (kResidual<EPI>)
              tma_store_2d_keep(&tmC, stg, (int)ocol, row0);
            else
              tma_store_2d(&tmC, stg, (int)ocol, row0);
            bulk_commit();
          }
          ob = (ob + 1) % kOutBufs<EPI>;
        }
      }
    }
    if (lane == 0) bulk_wait0();
    if constexpr (EPI == EPI_RESIDUAL_TMA) {
      // Left early (aborting): this warp's residual loads land before the CTA exits.
      for (int u = 0; u < 2; u++)
        if ((rpend >> u) & 1) mbar_drain(&rbar[(warp - 2) * 2 + u], (rph >> u) & 1);
    }
  }

  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // no cross-CTA signal or MMA is in flight past this point
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::TMEM_COLS)
                   : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::TMEM_COLS)
                   : "memory");
  }
}

// Split-K finish: out = epilogue(sum over splits of the fp32 partial sums), the same epilogues
// as the tensor-core kernel (same formulas, same packed column order for SwiGLU).  One thread
// per output pair: columns (2i, 2i+1), or for RoPE a head's (c, c+32), or for SwiGLU the gate /
// up columns of two outputs.
template <typename T, int EPI>
__global__ void __launch_bounds__(256)
    k_splitk_finish(const float* __restrict__ part, int splits, int64_t M, int64_t N, T* __restrict__ out,
                    int64_t ld_out, const float* __restrict__ bias, const T* __restrict__ res, int64_t ld_res,
                    const int32_t* __restrict__ pos, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                    int64_t rope_cols) {
  pdl_wait();
  const int64_t n_out = EPI == EPI_SWIGLU ? N / 2 : N;
  const int64_t pairs = M * (n_out / 2);
  const int64_t plane = M * N;
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < pairs; p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = p / (n_out / 2);
    const int64_t k = p % (n_out / 2);
    // Packed columns read (c0, c1) and the output columns written (o0, o1).
    int64_t c0, c1, o0, o1;
    if constexpr (EPI == EPI_ROPE) {
      c0 = (k / 32) * 64 + k % 32;  // x1 and x2 of one rotate-half pair
      c1 = c0 + 32;
      o0 = c0;
      o1 = c1;
    } else {
      o0 = 2 * k;
      o1 = o0 + 1;
      c0 = o0;
      c1 = o1;
    }
    const float* pr = part + row * N;
    if constexpr (EPI == EPI_SWIGLU) {
      // Output j: gate column (j/128)*256 + j%128, up column gate + 128 (the weight packing).
      float y[2];
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int64_t j = o0 + e;
        const int64_t gcol = (j / 128) * 256 + j % 128, ucol = gcol + 128;
        float g = 0.f, v = 0.f;
        for (int sp = 0; sp < splits; sp++) {
          g += pr[sp * plane + gcol];
          v += pr[sp * plane + ucol];
        }
        if (bias) {
          g += bias[gcol];
          v += bias[ucol];
        }
        y[e] = __fdividef(g, 1.0f + __expf(-g)) * v;
      }
      *reinterpret_cast<uint32_t*>(out + row * ld_out + o0) = pack2<T>(y[0], y[1]);
    } else {
      float a = 0.f, b = 0.f;
      for (int sp = 0; sp < splits; sp++) {
        a += pr[sp * plane + c0];
        b += pr[sp * plane + c1];
      }
      if (bias) {
        a += bias[c0];
        b += bias[c1];
      }
      if constexpr (EPI == EPI_ROPE) {
        if (c0 < rope_cols) {
          const int i = (int)(k % 32);
          const float cs = cos_t[(int64_t)pos[row] * 32 + i], sn = sin_t[(int64_t)pos[row] * 32 + i];
          const float x1 = a, x2 = b;
          a = x1 * cs - x2 * sn;
          b = x1 * sn + x2 * cs;
        }
        out[row * ld_out + o0] = from_f<T>(a);
        out[row * ld_out + o1] = from_f<T>(b);
      } else {
        if constexpr (EPI == EPI_GELU) {
          a = gelu_fast16(a);
          b = gelu_fast16(b);
        }
        if constexpr (EPI == EPI_RESIDUAL) {
          a += to_f<T>(res[row * ld_res + o0]);
          b += to_f<T>(res[row * ld_res + o1]);
        }
        *reinterpret_cast<uint32_t*>(out + row * ld_out + o0) = pack2<T>(a, b);
      }
    }
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2D row-major map over [rows, cols] with row stride ld (elements): box {box_cols, box_rows},
// 128-byte swizzle, out-of-bounds reads as zero (stores are clipped).
static int32_t make_map(Ctx* c, CUtensorMap* m, int32_t dtype, const void* ptr, uint64_t rows, uint64_t cols,
                        uint64_t ld, uint32_t box_cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(c, FLETCHER_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dtype == FLETCHER_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(c, FLETCHER_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FLETCHER_OK;
}

template <typename T, int BN, int EPI, bool PAIR>
static int32_t run(Ctx* c, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mr,
                   GemmArgs a) {
  using Cf = Cfg<BN, PAIR, kOutBufs<EPI>>;
  auto kern = k_gemm_tc<T, BN, EPI, PAIR>;
  // Per device; host threads of several replicas may get here at once (the call is idempotent).
  static std::atomic<bool> attr_set[64] = {};
  if (!attr_set[c->device & 63].load(std::memory_order_acquire)) {
    FL_CUDA(c, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM));
    attr_set[c->device & 63].store(true, std::memory_order_release);
  }
  a.num_m_tiles = (int)((a.M + Cf::TILE_M - 1) / Cf::TILE_M);
  a.num_n_tiles = (int)((a.N + BN - 1) / BN);
  const int tiles = a.num_m_tiles * a.num_n_tiles * a.splits;
  if constexpr (PAIR) {
    const int pairs = c->num_sms / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (tiles < pairs ? tiles : pairs));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cf::SMEM;
    cfg.stream = c->stream;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    FL_CUDA(c, cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, mr, a));
  } else {
    const int grid = tiles < c->num_sms ? tiles : c->num_sms;
    FL_CUDA(c, launch_pdl(kern, dim3(grid), dim3(kThreads), Cf::SMEM, c->stream, ma, mb, mc, mr, a));
  }
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

template <typename T, bool PAIR>
static int32_t dispatch(Ctx* c, int epi, int bn, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                        const CUtensorMap& mr, const GemmArgs& a) {
#define FL_EPI(E)                                                                            \
  case E:                                                                                    \
    return bn == 256 ? run<T, 256, E, PAIR>(c, ma, mb, mc, mr, a) : run<T, 128, E, PAIR>(c, ma, mb, mc, mr, a);
  switch (epi) {
    FL_EPI(EPI_STORE)
    FL_EPI(EPI_ROPE)
    FL_EPI(EPI_GELU)
    FL_EPI(EPI_RESIDUAL)
    FL_EPI(EPI_RESIDUAL_TMA)
    case EPI_SWIGLU:
      return run<T, 256, EPI_SWIGLU, PAIR>(c, ma, mb, mc, mr, a);
    case EPI_PARTIAL:
      return run<T, 128, EPI_PARTIAL, false>(c, ma, mb, mc, mr, a);
  }
#undef FL_EPI
  return set_error(c, FLETCHER_ERR_INVALID, "gemm: unknown epilogue %d", epi);
}

}  // namespace tc

int32_t make_tma_map_2d(Ctx* c, CUtensorMap* m, int32_t dtype, const void* ptr, uint64_t rows, uint64_t cols,
                        uint64_t ld, uint32_t box_cols, uint32_t box_rows) {
  return tc::make_map(c, m, dtype, ptr, rows, cols, ld, box_cols, box_rows);
}

// FLETCHER_GEMM_PAIR=0 selects single-SM tiles everywhere (for A/B measurement).
bool gemm_pair_enabled() {
  static const bool on = [] {
    const char* e = getenv("FLETCHER_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Split-K plan for a GEMM whose output tiles (128 x 128) cannot fill the GPU: K ranges per tile
// such that tiles x ranges reaches about one CTA per SM, at least two 64-wide K blocks each.
// Returns the fp32 workspace bytes ([splits, M, N]), 0 when no split is worthwhile.
int64_t gemm_splitk_plan(const Ctx* c, int64_t M, int64_t N, int64_t K, int* splits, int* kb_per) {
  const int64_t tiles = ((M + 127) / 128) * ((N + 127) / 128);
  const int kb = (int)(K / tc::BK);
  if (M > 1024 || tiles * 2 > c->num_sms || kb < 4 || N % 128 != 0) return 0;
  int sp = (int)((c->num_sms + tiles - 1) / tiles);
  if (sp > kb / 2) sp = kb / 2;
  const int per = (kb + sp - 1) / sp;
  sp = (kb + per - 1) / per;
  if (sp < 2) return 0;
  *splits = sp;
  *kb_per = per;
  return (int64_t)sp * M * N * 4;
}

// Partial-sum GEMM (tcgen05, 128 x 128 tiles, `splits` K ranges) + finishing epilogue kernel.
static int32_t launch_gemm_splitk(Ctx* c, int32_t dtype, int epi, const void* A, int64_t M, int64_t K, const void* W,
                                  int64_t N, void* out, int64_t ld_out, const float* bias, const void* residual,
                                  int64_t ld_res, const int32_t* pos, const float* cos_t, const float* sin_t,
                                  int64_t rope_cols, int splits, int kb_per) {
  CUtensorMap ma, mb;
  int32_t rc = tc::make_map(c, &ma, dtype, A, (uint64_t)M, (uint64_t)K, (uint64_t)K, tc::BK, tc::BM);
  if (rc) return rc;
  if ((rc = tc::make_map(c, &mb, dtype, W, (uint64_t)N, (uint64_t)K, (uint64_t)K, tc::BK, 128))) return rc;
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = (int)K;
  a.err = c->d_err;
  a.splits = splits;
  a.kb_per = kb_per;
  a.partial = c->splitk;
  if (dtype == FLETCHER_BF16)
    rc = tc::dispatch<__nv_bfloat16, false>(c, EPI_PARTIAL, 128, ma, mb, ma, ma, a);
  else
    rc = tc::dispatch<__half, false>(c, EPI_PARTIAL, 128, ma, mb, ma, ma, a);
  if (rc) return rc;
  const int64_t n_out = epi == EPI_SWIGLU ? N / 2 : N;
  const int64_t pairs = M * (n_out / 2);
  const int grid = (int)std::min<int64_t>((pairs + 255) / 256, (int64_t)c->num_sms * 8);
#define FL_FIN(TT, E)                                                                                         \
  FL_CUDA(c, launch_pdl(tc::k_splitk_finish<TT, E>, dim3(grid), dim3(256), 0, c->stream, (const float*)c->splitk, \
                        splits, M, N, (TT*)out, ld_out, bias, (const TT*)residual, ld_res, pos, cos_t, sin_t, rope_cols))
#define FL_FIN_T(TT)                 \
  switch (epi) {                     \
    case EPI_STORE:                  \
      FL_FIN(TT, EPI_STORE);         \
      break;                         \
    case EPI_ROPE:                   \
      FL_FIN(TT, EPI_ROPE);          \
      break;                         \
    case EPI_GELU:                   \
      FL_FIN(TT, EPI_GELU);          \
      break;                         \
    case EPI_SWIGLU:                 \
      FL_FIN(TT, EPI_SWIGLU);        \
      break;                         \
    default:                         \
      FL_FIN(TT, EPI_RESIDUAL);      \
      break;                         \
  }
  if (dtype == FLETCHER_BF16) {
    FL_FIN_T(__nv_bfloat16)
  } else {
    FL_FIN_T(__half)
  }
#undef FL_FIN_T
#undef FL_FIN
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

bool gemm_tc_supported(int64_t M, int64_t N, int64_t K, int bn) {
  return M > 0 && M < (1ll << 31) && K % tc::BK == 0 && K > 0 && N % 64 == 0 && (bn == 128 || bn == 256);
}

int32_t launch_gemm_tc(Ctx* c, int32_t dtype, int epi, int bn, const void* A, int64_t M, int64_t K, const void* W,
                       int64_t N, void* out, int64_t ld_out, const float* bias, const void* residual, int64_t ld_res,
                       const int32_t* pos, const float* cos_t, const float* sin_t, int64_t rope_cols) {
  FL_CHECK(c, dtype == FLETCHER_BF16 || dtype == FLETCHER_F16, "gemm_tc: 16-bit dtypes only");
  FL_CHECK(c, gemm_tc_supported(M, N, K, bn), "gemm_tc: unsupported shape M=%lld N=%lld K=%lld BN=%d",
           (long long)M, (long long)N, (long long)K, bn);
  FL_CHECK(c, ((uintptr_t)A & 15) == 0 && ((uintptr_t)W & 15) == 0 && ((uintptr_t)out & 15) == 0 && ld_out % 8 == 0,
           "gemm_tc: operands must be 16-byte aligned");
  FL_CHECK(c, epi != EPI_SWIGLU || (bn == 256 && N % 256 == 0), "gemm_tc: SwiGLU needs BN = 256 and N %% 256 == 0");
  FL_CHECK(c, epi != EPI_RESIDUAL || (((uintptr_t)residual & 15) == 0 && ld_res % 8 == 0),
           "gemm_tc: residual must be 16-byte aligned");
  const int64_t n_out = epi == EPI_SWIGLU ? N / 2 : N;
  // Few output tiles (small batches, single requests): split K so that enough CTAs stream the
  // weights, then finish the sums with the epilogue in a second kernel.
  {
    int splits = 0, kb_per = 0;
    const int64_t need = gemm_splitk_plan(c, M, N, K, &splits, &kb_per);
    if (need > 0 && need <= c->splitk_bytes)
      return launch_gemm_splitk(c, dtype, epi, A, M, K, W, N, out, ld_out, bias, residual, ld_res, pos, cos_t, sin_t,
                                rope_cols, splits, kb_per);
  }
  // CTA pairs (2-SM MMAs) once there are enough 256-row tiles to fill the GPU.
  const bool pair = gemm_pair_enabled() && M >= 2048;
  CUtensorMap ma, mb, mc;
  int32_t rc = tc::make_map(c, &ma, dtype, A, (uint64_t)M, (uint64_t)K, (uint64_t)K, tc::BK, tc::BM);
  if (rc) return rc;
  rc = tc::make_map(c, &mb, dtype, W, (uint64_t)N, (uint64_t)K, (uint64_t)K, tc::BK, (uint32_t)(pair ? bn / 2 : bn));
  if (rc) return rc;
  rc = tc::make_map(c, &mc, dtype, out, (uint64_t)M, (uint64_t)n_out, (uint64_t)ld_out, 64, 32);
  if (rc) return rc;
  // Short-K residual GEMMs are epilogue-bound: their residual rows come by TMA into the output
  // boxes.  Long-K ones keep the register path and the extra operand stage it leaves.
  if (epi == EPI_RESIDUAL && K <= 1024) epi = EPI_RESIDUAL_TMA;
  CUtensorMap mr = mc;  // the residual rows, read as the output boxes they are added into
  if (epi == EPI_RESIDUAL_TMA &&
      (rc = tc::make_map(c, &mr, dtype, residual, (uint64_t)M, (uint64_t)N, (uint64_t)ld_res, 64, 32)))
    return rc;
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = (int)K;
  a.out = out;
  a.ld_out = ld_out;
  a.bias = bias;
  a.residual = residual;
  a.ld_res = ld_res;
  a.pos = pos;
  a.cos_t = cos_t;
  a.sin_t = sin_t;
  a.rope_cols = rope_cols;
  a.err = c->d_err;
  a.splits = 1;
  a.kb_per = (int)(K / tc::BK);
  if (pair) {
    if (dtype == FLETCHER_BF16) return tc::dispatch<__nv_bfloat16, true>(c, epi, bn, ma, mb, mc, mr, a);
    return tc::dispatch<__half, true>(c, epi, bn, ma, mb, mc, mr, a);
  }
  if (dtype == FLETCHER_BF16) return tc::dispatch<__nv_bfloat16, false>(c, epi, bn, ma, mb, mc, mr, a);
  return tc::dispatch<__half, false>(c, epi, bn, ma, mb, mc, mr, a);
}

}  // namespace fl
