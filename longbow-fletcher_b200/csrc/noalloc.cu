// Cuda_Attention_VarLen_NoAlloc: variable-length attention that allocates no memory.
//
// Cuda_Attention_VarLen allocates a small device array per call for its launch metadata (the
// cu_seqlens prefix sums and, in 16-bit mode, the list of 128-row query tiles).  Some callers
// cannot allocate at that point: a server whose device memory is fully reserved up front by
// its admission control (every byte is accounted before a request is accepted), or a host
// framework that owns the device allocator and forbids other allocations.  This entry point
// keeps that metadata in a fixed, file-scope device array instead, so the call performs no
// cudaMalloc/cudaFree and no other allocation; the caller still passes q, k, v and result.
//
// Limits and sharing rules:
//   - the array holds FLETCHER_NOALLOC_SCRATCH_INTS int32 values (1 MiB) on every GPU that
//     loads the library, for the life of the process;
//   - one call needs (numSeqs + 1) ints in 32-bit mode, plus 2 ints per 128-row query tile
//     (sum over sequences of ceil(length / 128)) in 16-bit mode; larger calls are rejected with
//     FLETCHER_ERR_INVALID before anything is launched;
//   - every call on a device shares the one array and it keeps the previous call's contents
//     (each call rewrites the part it reads, so nothing has to start at zero); calls whose work
//     overlaps on the GPU — from two contexts or streams of the same device — race on it.
//     Calls on one context are ordered on its stream and are safe;
//   - the first call on each device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current); make that first call before any stream
//     capture begins.
#include <mutex>

#include "kernels.cuh"

namespace fl {

static __device__ __align__(256) int32_t g_noalloc_scratch[FLETCHER_NOALLOC_SCRATCH_INTS];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
int32_t* g_dev_ptr[kMaxDevices] = {};  // device address of g_noalloc_scratch, per device
// Host staging for the metadata.  Copies from pageable host memory are staged by the driver
// before cudaMemcpyAsync returns, so the buffer is free again when the call returns.
int32_t g_host[FLETCHER_NOALLOC_SCRATCH_INTS];

// The host-side name g_noalloc_scratch is only a stand-in for the device array; kernels must
// get the address that cudaGetSymbolAddress returns for the current device.
int32_t scratch_ptr(Ctx* c, int32_t** out) {
  if (c->device < 0 || c->device >= kMaxDevices) return set_error(c, FLETCHER_ERR_INVALID, "device index too large");
  if (!g_dev_ptr[c->device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(c, FLETCHER_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
    g_dev_ptr[c->device] = static_cast<int32_t*>(p);
  }
  *out = g_dev_ptr[c->device];
  return FLETCHER_OK;
}
}  // namespace

}  // namespace fl

using namespace fl;

extern "C" int32_t Cuda_Attention_VarLen_NoAlloc(CudaContextRef ctx, CudaBufferRef qb, CudaBufferRef kb,
                                                 CudaBufferRef vb, CudaBufferRef rb, const int32_t* lengths,
                                                 int32_t numSeqs, int64_t hidden, int32_t nh, float scale) {
  Ctx* c = reinterpret_cast<Ctx*>(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *q = reinterpret_cast<Buf*>(qb), *k = reinterpret_cast<Buf*>(kb), *v = reinterpret_cast<Buf*>(vb),
      *o = reinterpret_cast<Buf*>(rb);
  FL_CHECK(c, q && k && v && o, "AttentionVarLen_NoAlloc: null buffer");
  FL_CHECK(c, numSeqs >= 0 && (lengths || numSeqs == 0), "AttentionVarLen_NoAlloc: bad lengths");
  const int32_t dt = q->dtype;
  FL_CHECK(c, k->dtype == dt && v->dtype == dt && o->dtype == dt, "AttentionVarLen_NoAlloc: dtype mismatch");
  FL_CHECK(c, nh > 0 && hidden > 0 && hidden % nh == 0, "AttentionVarLen_NoAlloc: hidden %% heads != 0");
  const int32_t dh = (int32_t)(hidden / nh);
  FL_CHECK(c, dt == FLETCHER_F32 || dh == 64, "AttentionVarLen_NoAlloc: 16-bit attention needs head_dim 64");
  int64_t T = 0, tiles = 0;
  int32_t mx = 0;
  for (int i = 0; i < numSeqs; i++) {
    FL_CHECK(c, lengths[i] >= 0, "AttentionVarLen_NoAlloc: negative length");
    T += lengths[i];
    tiles += (lengths[i] + kAttnTileRows - 1) / kAttnTileRows;
    mx = lengths[i] > mx ? lengths[i] : mx;
  }
  FL_CHECK(c, dt == FLETCHER_F32 || mx <= kAttnMaxLen,
           "AttentionVarLen_NoAlloc: 16-bit attention takes sequences up to %d rows (got %d)", kAttnMaxLen, mx);
  const int64_t es = dtype_size(dt);
  FL_CHECK(c, T * hidden * es <= q->bytes && T * hidden * es <= k->bytes && T * hidden * es <= v->bytes &&
                  T * hidden * es <= o->bytes,
           "AttentionVarLen_NoAlloc: buffers smaller than the batch");
  const int64_t tiles_off = numSeqs + 1 + ((numSeqs + 1) & 1);  // keep the int2 tile list 8-byte aligned
  const int64_t need = dt == FLETCHER_F32 ? numSeqs + 1 : tiles_off + 2 * tiles;
  FL_CHECK(c, need <= FLETCHER_NOALLOC_SCRATCH_INTS,
           "AttentionVarLen_NoAlloc: batch needs %lld scratch ints, the limit is %d (FLETCHER_NOALLOC_SCRATCH_INTS)",
           (long long)need, (int)FLETCHER_NOALLOC_SCRATCH_INTS);
  if (T == 0) return FLETCHER_OK;
  // The metadata goes through a pageable host array, which a stream capture cannot record (and a
  // recorded copy would replay whatever a later call left in it): refuse capture outright.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  FL_CUDA(c, cudaStreamIsCapturing(c->stream, &cap));
  FL_CHECK(c, cap == cudaStreamCaptureStatusNone,
           "AttentionVarLen_NoAlloc: cannot be captured into a CUDA graph (its metadata is copied from a host array)");
  touch(o);

  std::lock_guard<std::mutex> lock(g_mu);
  int32_t* dscr = nullptr;
  int32_t rc = scratch_ptr(c, &dscr);
  if (rc) return rc;
  g_host[0] = 0;
  for (int i = 0; i < numSeqs; i++) g_host[i + 1] = g_host[i] + lengths[i];
  if (dt != FLETCHER_F32) {
    int64_t t = tiles_off;
    for (int s = 0; s < numSeqs; s++)
      for (int q0 = 0; q0 < lengths[s]; q0 += kAttnTileRows) {
        const int2 d = attn_tile(g_host[s], lengths[s], q0);
        g_host[t++] = d.x;
        g_host[t++] = d.y;
      }
  }
  FL_CUDA(c, cudaMemcpyAsync(dscr, g_host, need * 4, cudaMemcpyHostToDevice, c->stream));
  if (dt == FLETCHER_F32)
    return launch_attention_f32(c, (const float*)q->ptr, (const float*)k->ptr, (const float*)v->ptr, hidden,
                                (float*)o->ptr, hidden, dscr, numSeqs, T, nh, dh, scale, mx);
  return launch_flash_attention_tc(c, dt, q->ptr, k->ptr, v->ptr, hidden, T, hidden, o->ptr, hidden, dscr,
                                   reinterpret_cast<const int2*>(dscr + tiles_off), (int32_t)tiles, nh, scale);
}
