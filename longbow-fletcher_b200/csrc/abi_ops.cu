// Tensor-op entry points of the C ABI (include/fletcher_cuda.h): the device.Tensor methods the
// reference's Go wrapper forwards over cgo (cuda_linux.go -> cuda_bridge.h).  Each validates
// shapes and dtypes against the buffers, binds the context's device and enqueues on its stream.
#include <algorithm>
#include <vector>

#include "gemm.cuh"

using namespace fl;

namespace {

Ctx* C(CudaContextRef r) { return reinterpret_cast<Ctx*>(r); }
Buf* B(CudaBufferRef r) { return reinterpret_cast<Buf*>(r); }

bool fits(const Buf* b, int64_t elems) { return b && elems >= 0 && elems * dtype_size(b->dtype) <= b->bytes; }

// Temporary device array for small per-call metadata; freed in stream order.
struct Temp {
  Ctx* c;
  void* p = nullptr;
  int64_t n = 0;
  Temp(Ctx* c_) : c(c_) {}
  int32_t alloc(int64_t bytes) {
    n = bytes;
    return dev_alloc(c, &p, bytes);
  }
  ~Temp() {
    if (p) dev_free(c, p, n);
  }
};

// Small per-call host metadata -> a stream-ordered temporary, copied through the context's
// pinned staging ring (no host synchronisation; the caller may free its array on return).
int32_t upload(Ctx* c, Temp& t, const void* h, int64_t bytes) {
  int32_t rc = t.alloc(bytes);
  if (rc) return rc;
  return stage_to_device(c, t.p, h, bytes);
}

// Cuda_Linear_Fused's 16-bit weight in the tensor-core layout (K-major [N', K], SwiGLU
// interleaved), built once per weight contents and layout and kept with the weight buffer.
int32_t packed_weight(Ctx* c, Buf* w, int64_t K, int64_t N, bool swiglu, int bn, const void** out) {
  const int key = (swiglu ? 1 : 0) | (bn << 1);
  const int64_t bytes = K * N * 2;
  if (!(w->packed && w->packed_key == key && w->packed_ver == w->version && w->packed_bytes == bytes)) {
    dev_free(c, w->packed, w->packed_bytes);
    w->packed = nullptr;
    w->packed_bytes = 0;
    int32_t rc = dev_alloc(c, &w->packed, bytes);
    if (rc) return rc;
    w->packed_bytes = bytes;
    if ((rc = launch_pack_kmajor_16(c, w->dtype, w->ptr, K, N, w->packed, swiglu ? 1 : 0, bn))) {
      w->packed_key = -1;
      return rc;
    }
    w->packed_key = key;
    w->packed_ver = w->version;
  }
  *out = w->packed;
  return FLETCHER_OK;
}

// The bias widened to fp32 in the packed column order, cached like the weight.
int32_t packed_bias(Ctx* c, Buf* b, int64_t N, bool swiglu, int bn, const float** out) {
  const int key = (swiglu ? 1 : 0) | (bn << 1);
  if (!(b->bias32 && b->bias32_key == key && b->bias32_ver == b->version && b->bias32_bytes == N * 4)) {
    dev_free(c, b->bias32, b->bias32_bytes);
    b->bias32 = nullptr;
    b->bias32_bytes = 0;
    int32_t rc = dev_alloc(c, (void**)&b->bias32, N * 4);
    if (rc) return rc;
    b->bias32_bytes = N * 4;
    b->bias32_key = -1;
    if (swiglu) {  // interleave the bias like the weight rows: pack a [1, N] row as K=1
      Temp b16(c);
      if ((rc = b16.alloc(N * 2))) return rc;
      if ((rc = launch_pack_kmajor_16(c, b->dtype, b->ptr, 1, N, b16.p, 1, bn))) return rc;
      if ((rc = launch_cast(c, b->dtype, b16.p, FLETCHER_F32, b->bias32, N))) return rc;
    } else if ((rc = launch_cast(c, b->dtype, b->ptr, FLETCHER_F32, b->bias32, N))) {
      return rc;
    }
    b->bias32_key = key;
    b->bias32_ver = b->version;
  }
  *out = b->bias32;
  return FLETCHER_OK;
}

}  // namespace

extern "C" {

int32_t Cuda_Linear_Fused(CudaContextRef ctx, CudaBufferRef input, int64_t rows, int64_t inCols, CudaBufferRef weight,
                          int64_t outCols, CudaBufferRef bias, CudaBufferRef result, int32_t activation) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *x = B(input), *w = B(weight), *b = B(bias), *y = B(result);
  FL_CHECK(c, x && w && y, "Linear: null buffer");
  const int32_t dt = x->dtype;
  FL_CHECK(c, w->dtype == dt && y->dtype == dt && (!b || b->dtype == dt), "Linear: dtype mismatch");
  const bool swiglu = activation == FLETCHER_ACT_SWIGLU;
  FL_CHECK(c, !swiglu || outCols % 2 == 0, "Linear: SwiGLU needs an even output width");
  const int64_t ycols = swiglu ? outCols / 2 : outCols;
  FL_CHECK(c, fits(x, rows * inCols) && fits(w, inCols * outCols) && fits(y, rows * ycols) && (!b || fits(b, outCols)),
           "Linear: buffer smaller than its shape");
  const int act = (activation == FLETCHER_ACT_GELU || activation == FLETCHER_ACT_TANH) ? activation : FLETCHER_ACT_IDENTITY;
  int32_t rc;
  touch(y);
  // 16-bit: tensor-core GEMM on the cached K-major packing of the (in,out) weight (SwiGLU
  // weights gate/up-interleaved per tile) and the cached fp32 bias.
  const int bn = swiglu || (outCols % 256 == 0 && outCols >= 1024) ? 256 : 128;
  const bool tc_act = activation == FLETCHER_ACT_IDENTITY || activation == FLETCHER_ACT_GELU || swiglu;
  if (dt != FLETCHER_F32 && tc_act && gemm_tc_supported(rows, outCols, inCols, bn) && (!swiglu || outCols % bn == 0)) {
    const void* wk = nullptr;
    const float* bf = nullptr;
    if ((rc = packed_weight(c, w, inCols, outCols, swiglu, bn, &wk))) return rc;
    if (b && (rc = packed_bias(c, b, outCols, swiglu, bn, &bf))) return rc;
    const int epi = swiglu ? EPI_SWIGLU : activation == FLETCHER_ACT_GELU ? EPI_GELU : EPI_STORE;
    return launch_gemm_tc(c, dt, epi, bn, x->ptr, rows, inCols, wk, outCols, y->ptr, ycols, bf, nullptr, 0, nullptr,
                          nullptr, nullptr, 0);
  }
  if (!swiglu && activation != FLETCHER_ACT_SOFTMAX) {
    rc = launch_gemm_simt(c, dt, x->ptr, inCols, w->ptr, outCols, y->ptr, outCols, rows, outCols, inCols,
                          b ? b->ptr : nullptr, act);
    return rc;
  }
  Temp full(c);
  if ((rc = full.alloc(rows * outCols * dtype_size(dt)))) return rc;
  if ((rc = launch_gemm_simt(c, dt, x->ptr, inCols, w->ptr, outCols, full.p, outCols, rows, outCols, inCols,
                             b ? b->ptr : nullptr, FLETCHER_ACT_IDENTITY)))
    return rc;
  if (swiglu) return launch_swiglu(c, dt, full.p, y->ptr, rows, outCols / 2);
  if ((rc = launch_activation(c, dt, full.p, rows, outCols, FLETCHER_ACT_SOFTMAX))) return rc;
  FL_CUDA(c, cudaMemcpyAsync(y->ptr, full.p, rows * outCols * dtype_size(dt), cudaMemcpyDeviceToDevice, c->stream));
  return FLETCHER_OK;
}

int32_t Cuda_LayerNorm(CudaContextRef ctx, CudaBufferRef input, CudaBufferRef gamma, CudaBufferRef beta,
                       CudaBufferRef result, int64_t rows, int64_t cols, float eps) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *x = B(input), *ga = B(gamma), *be = B(beta), *y = B(result);
  FL_CHECK(c, x && ga && be && y, "LayerNorm: null buffer");
  FL_CHECK(c, ga->dtype == FLETCHER_F32 && be->dtype == FLETCHER_F32, "LayerNorm: gamma/beta must be f32");
  FL_CHECK(c, x->dtype == y->dtype, "LayerNorm: dtype mismatch");
  FL_CHECK(c, fits(x, rows * cols) && fits(y, rows * cols) && fits(ga, cols) && fits(be, cols), "LayerNorm: shape");
  touch(y);
  return launch_add_layernorm(c, x->dtype, x->ptr, nullptr, y->ptr, (const float*)ga->ptr, (const float*)be->ptr, rows,
                              cols, eps);
}

int32_t Cuda_AddLayerNorm(CudaContextRef ctx, CudaBufferRef xb, CudaBufferRef residual, CudaBufferRef gamma,
                          CudaBufferRef beta, int64_t rows, int64_t cols, float eps) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *x = B(xb), *r = B(residual), *ga = B(gamma), *be = B(beta);
  FL_CHECK(c, x && r && ga && be, "AddLayerNorm: null buffer");
  FL_CHECK(c, ga->dtype == FLETCHER_F32 && be->dtype == FLETCHER_F32, "AddLayerNorm: gamma/beta must be f32");
  FL_CHECK(c, x->dtype == r->dtype, "AddLayerNorm: dtype mismatch");
  FL_CHECK(c, fits(x, rows * cols) && fits(r, rows * cols) && fits(ga, cols) && fits(be, cols), "AddLayerNorm: shape");
  touch(x);
  return launch_add_layernorm(c, x->dtype, x->ptr, r->ptr, x->ptr, (const float*)ga->ptr, (const float*)be->ptr, rows,
                              cols, eps);
}

int32_t Cuda_Softmax(CudaContextRef ctx, CudaBufferRef input, CudaBufferRef result, int64_t rows, int64_t cols) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *x = B(input), *y = B(result);
  FL_CHECK(c, x && y && x->dtype == y->dtype && fits(x, rows * cols) && fits(y, rows * cols), "Softmax: bad buffers");
  touch(y);
  if (x != y)
    FL_CUDA(c, cudaMemcpyAsync(y->ptr, x->ptr, rows * cols * dtype_size(x->dtype), cudaMemcpyDeviceToDevice, c->stream));
  return launch_activation(c, y->dtype, y->ptr, rows, cols, FLETCHER_ACT_SOFTMAX);
}

int32_t Cuda_Gather(CudaContextRef ctx, CudaBufferRef table, const int32_t* indices, CudaBufferRef output,
                    int64_t count, int64_t cols) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *t = B(table), *o = B(output);
  FL_CHECK(c, t && o && (indices || count == 0), "Gather: null argument");
  FL_CHECK(c, t->dtype == o->dtype && fits(o, count * cols), "Gather: bad output");
  const int64_t rows = cols > 0 ? t->bytes / dtype_size(t->dtype) / cols : 0;
  for (int64_t i = 0; i < count; i++)  // cpu_backend.go:501-502 panics on a bad index
    FL_CHECK(c, indices[i] >= 0 && indices[i] < rows, "Gather index out of bounds: %d", indices[i]);
  if (count == 0) return FLETCHER_OK;
  touch(o);
  Temp idx(c);
  int32_t rc = upload(c, idx, indices, count * 4);
  if (rc) return rc;
  // Gather as f32 rows then convert: one kernel per dtype is not worth it for this op.
  if (t->dtype == FLETCHER_F32)
    return launch_gather_rows_f32(c, FLETCHER_F32, t->ptr, (const int32_t*)idx.p, count, cols, (float*)o->ptr);
  Temp f(c);
  if ((rc = f.alloc(count * cols * 4))) return rc;
  if ((rc = launch_gather_rows_f32(c, t->dtype, t->ptr, (const int32_t*)idx.p, count, cols, (float*)f.p))) return rc;
  return launch_cast(c, FLETCHER_F32, f.p, o->dtype, o->ptr, count * cols);
}

int32_t Cuda_Add(CudaContextRef ctx, CudaBufferRef x, CudaBufferRef other, int64_t count) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *a = B(x), *b = B(other);
  FL_CHECK(c, a && b && a->dtype == b->dtype && fits(a, count) && fits(b, count), "Add: bad buffers");
  touch(a);
  return launch_scale_add(c, a->dtype, a->ptr, b->ptr, 1.0f, 0.0f, count);
}

int32_t Cuda_Scale(CudaContextRef ctx, CudaBufferRef x, float val, int64_t count) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf* a = B(x);
  FL_CHECK(c, a && fits(a, count), "Scale: bad buffer");
  touch(a);
  if (val == 1.0f) return FLETCHER_OK;
  return launch_scale_add(c, a->dtype, a->ptr, nullptr, val, 0.0f, count);
}

int32_t Cuda_AddScalar(CudaContextRef ctx, CudaBufferRef x, float val, int64_t count) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf* a = B(x);
  FL_CHECK(c, a && fits(a, count), "AddScalar: bad buffer");
  touch(a);
  return launch_scale_add(c, a->dtype, a->ptr, nullptr, 1.0f, val, count);
}

int32_t Cuda_AddBias(CudaContextRef ctx, CudaBufferRef x, CudaBufferRef bias, int64_t rows, int64_t cols) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *a = B(x), *b = B(bias);
  FL_CHECK(c, a && b && a->dtype == b->dtype && fits(a, rows * cols) && fits(b, cols), "AddBias: bad buffers");
  touch(a);
  return launch_add_bias(c, a->dtype, a->ptr, b->ptr, rows, cols);
}

int32_t Cuda_Activation(CudaContextRef ctx, CudaBufferRef x, int64_t rows, int64_t cols, int32_t activation) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf* a = B(x);
  FL_CHECK(c, a && fits(a, rows * cols), "Activation: bad buffer");
  touch(a);
  return launch_activation(c, a->dtype, a->ptr, rows, cols, activation);
}

int32_t Cuda_Cast(CudaContextRef ctx, CudaBufferRef src, CudaBufferRef dst, int64_t count) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *s = B(src), *d = B(dst);
  FL_CHECK(c, s && d && fits(s, count) && fits(d, count), "Cast: bad buffers");
  touch(d);
  return launch_cast(c, s->dtype, s->ptr, d->dtype, d->ptr, count, c->half_mode == FLETCHER_HALF_REFERENCE);
}

int32_t Cuda_HasNaN(CudaContextRef ctx, CudaBufferRef x, int64_t count, int32_t* result) {
  Ctx* c = C(ctx);
  if (!c || !result) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf* a = B(x);
  FL_CHECK(c, a && fits(a, count), "HasNaN: bad buffer");
  Temp flag(c);
  int32_t rc = flag.alloc(4);
  if (rc) return rc;
  if ((rc = launch_has_nan(c, a->dtype, a->ptr, count, (int32_t*)flag.p))) return rc;
  int32_t h = 0;
  FL_CUDA(c, cudaMemcpyAsync(&h, flag.p, 4, cudaMemcpyDeviceToHost, c->stream));
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  *result = h != 0;
  return FLETCHER_OK;
}

static int32_t attention_common(Ctx* c, Buf* q, Buf* k, Buf* v, Buf* out, const std::vector<int32_t>& lens,
                                int64_t hidden, int32_t nh, float scale) {
  int64_t T = 0;
  int32_t mx = 0;
  for (int32_t l : lens) {
    FL_CHECK(c, l >= 0, "Attention: negative length");
    T += l;
    mx = std::max(mx, l);
  }
  FL_CHECK(c, q && k && v && out, "Attention: null buffer");
  const int32_t dt = q->dtype;
  FL_CHECK(c, k->dtype == dt && v->dtype == dt && out->dtype == dt, "Attention: dtype mismatch");
  FL_CHECK(c, nh > 0 && hidden % nh == 0, "Attention: hidden %% heads != 0");
  FL_CHECK(c, fits(q, T * hidden) && fits(k, T * hidden) && fits(v, T * hidden) && fits(out, T * hidden),
           "Attention: buffers smaller than the batch");
  const int32_t dh = (int32_t)(hidden / nh);
  const int32_t Bn = (int32_t)lens.size();
  if (T == 0) return FLETCHER_OK;
  touch(out);
  std::vector<int32_t> cu(Bn + 1, 0);
  for (int i = 0; i < Bn; i++) cu[i + 1] = cu[i] + lens[i];
  Temp dcu(c);
  int32_t rc = upload(c, dcu, cu.data(), (Bn + 1) * 4);
  if (rc) return rc;
  if (dt == FLETCHER_F32)
    return launch_attention_f32(c, (const float*)q->ptr, (const float*)k->ptr, (const float*)v->ptr, hidden,
                                (float*)out->ptr, hidden, (const int32_t*)dcu.p, Bn, T, nh, dh, scale, mx);
  FL_CHECK(c, dh == 64, "Attention: 16-bit attention needs head_dim 64 (got %d)", dh);
  FL_CHECK(c, mx <= kAttnMaxLen, "Attention: 16-bit attention takes sequences up to %d rows (got %d)", kAttnMaxLen, mx);
  std::vector<int2> tiles;
  for (int s = 0; s < Bn; s++)
    for (int q0 = 0; q0 < lens[s]; q0 += kAttnTileRows) tiles.push_back(attn_tile(cu[s], lens[s], q0));
  Temp dt_(c);
  if ((rc = upload(c, dt_, tiles.data(), (int64_t)tiles.size() * 8))) return rc;
  return launch_flash_attention_tc(c, dt, q->ptr, k->ptr, v->ptr, hidden, T, hidden, out->ptr, hidden,
                                   (const int32_t*)dcu.p, (const int2*)dt_.p, (int32_t)tiles.size(), nh, scale);
}

int32_t Cuda_Attention_Fused(CudaContextRef ctx, CudaBufferRef q, CudaBufferRef k, CudaBufferRef v,
                             CudaBufferRef result, int64_t batchSize, int64_t seqLen, int64_t hidden, int32_t numHeads,
                             float scale) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  FL_CHECK(c, batchSize >= 0 && seqLen >= 0, "Attention: negative shape");
  std::vector<int32_t> lens((size_t)batchSize, (int32_t)seqLen);
  return attention_common(c, B(q), B(k), B(v), B(result), lens, hidden, numHeads, scale);
}

int32_t Cuda_Attention_VarLen(CudaContextRef ctx, CudaBufferRef q, CudaBufferRef k, CudaBufferRef v,
                              CudaBufferRef result, const int32_t* lengths, int32_t numSeqs, int64_t hidden,
                              int32_t numHeads, float scale) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  FL_CHECK(c, numSeqs >= 0 && (lengths || numSeqs == 0), "AttentionVarLen: bad lengths");
  std::vector<int32_t> lens(lengths, lengths + numSeqs);
  return attention_common(c, B(q), B(k), B(v), B(result), lens, hidden, numHeads, scale);
}

static int32_t rope_common(Ctx* c, Buf* x, const std::vector<int32_t>& pos, int32_t nh, int32_t dh, double base) {
  const int64_t T = (int64_t)pos.size();
  FL_CHECK(c, x && nh > 0 && dh > 0 && dh % 2 == 0, "ApplyRoPE: bad arguments");
  FL_CHECK(c, fits(x, T * nh * dh), "ApplyRoPE: buffer smaller than rows*heads*headDim");
  if (T == 0) return FLETCHER_OK;
  touch(x);
  int32_t mx = 0;
  for (int32_t p : pos) mx = std::max(mx, p);
  Temp dpos(c), tab(c);
  int32_t rc = upload(c, dpos, pos.data(), T * 4);
  if (rc) return rc;
  const int64_t n = (int64_t)(mx + 1) * (dh / 2);
  if ((rc = tab.alloc(2 * n * 4))) return rc;
  float* ct = (float*)tab.p;
  if ((rc = launch_rope_build_table(c, ct, ct + n, mx + 1, dh, base))) return rc;
  return launch_rope_table(c, x->dtype, x->ptr, T, (int64_t)nh * dh, (int64_t)nh * dh, dh, (const int32_t*)dpos.p, ct,
                           ct + n);
}

int32_t Cuda_ApplyRoPE(CudaContextRef ctx, CudaBufferRef data, int64_t batchSize, int64_t seqLen, int32_t numHeads,
                       int32_t headDim) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  FL_CHECK(c, batchSize >= 0 && seqLen > 0, "ApplyRoPE: bad shape");
  std::vector<int32_t> pos((size_t)(batchSize * seqLen));
  for (int64_t r = 0; r < batchSize * seqLen; r++) pos[r] = (int32_t)(r % seqLen);  // cpu_backend.go:783
  return rope_common(c, B(data), pos, numHeads, headDim, 10000.0);
}

int32_t Cuda_ApplyRoPE_VarLen(CudaContextRef ctx, CudaBufferRef data, const int32_t* lengths, int32_t numSeqs,
                              int32_t numHeads, int32_t headDim, float base) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  FL_CHECK(c, numSeqs >= 0 && (lengths || numSeqs == 0), "ApplyRoPE_VarLen: bad lengths");
  std::vector<int32_t> pos;
  for (int s = 0; s < numSeqs; s++) {
    FL_CHECK(c, lengths[s] >= 0, "ApplyRoPE_VarLen: negative length");
    for (int i = 0; i < lengths[s]; i++) pos.push_back(i);
  }
  return rope_common(c, B(data), pos, numHeads, headDim, (double)base);
}

int32_t Cuda_MeanPoolL2(CudaContextRef ctx, CudaBufferRef hidden, const int32_t* lengths, int32_t numSeqs, int64_t cols,
                        CudaBufferRef out) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *h = B(hidden), *o = B(out);
  FL_CHECK(c, h && o && o->dtype == FLETCHER_F32 && numSeqs >= 0 && (lengths || numSeqs == 0), "MeanPoolL2: bad args");
  std::vector<int32_t> cu(numSeqs + 1, 0);
  for (int i = 0; i < numSeqs; i++) {
    FL_CHECK(c, lengths[i] >= 0, "MeanPoolL2: negative length");
    cu[i + 1] = cu[i] + lengths[i];
  }
  FL_CHECK(c, fits(h, (int64_t)cu[numSeqs] * cols) && fits(o, (int64_t)numSeqs * cols), "MeanPoolL2: shape");
  if (numSeqs == 0) return FLETCHER_OK;
  touch(o);
  Temp dcu(c);
  int32_t rc = upload(c, dcu, cu.data(), (numSeqs + 1) * 4);
  if (rc) return rc;
  return launch_mean_pool_l2(c, h->dtype, h->ptr, (const int32_t*)dcu.p, numSeqs, cols, (float*)o->ptr);
}

int32_t Cuda_Copy(CudaContextRef ctx, CudaBufferRef dst, int64_t dstOffset, CudaBufferRef src, int64_t srcOffset,
                  int64_t count) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *d = B(dst), *s = B(src);
  FL_CHECK(c, d && s, "Copy: null buffer");
  FL_CHECK(c, dstOffset >= 0 && srcOffset >= 0 && count >= 0 && fits(d, dstOffset + count) && fits(s, srcOffset + count),
           "Copy: range out of bounds");
  if (count == 0) return FLETCHER_OK;
  touch(d);
  char* dp = (char*)d->ptr + dstOffset * dtype_size(d->dtype);
  const char* sp = (const char*)s->ptr + srcOffset * dtype_size(s->dtype);
  if (d->dtype == s->dtype) {
    FL_CUDA(c, cudaMemcpyAsync(dp, sp, count * dtype_size(d->dtype), cudaMemcpyDeviceToDevice, c->stream));
    return FLETCHER_OK;
  }
  return launch_cast(c, s->dtype, sp, d->dtype, dp, count, c->half_mode == FLETCHER_HALF_REFERENCE);
}

int32_t Cuda_Slice(CudaContextRef ctx, CudaBufferRef src, int64_t i, int64_t k, int64_t j, int64_t l,
                   CudaBufferRef dst) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *s = B(src), *d = B(dst);
  FL_CHECK(c, s && d, "Slice: null buffer");
  FL_CHECK(c, k > i && l > j, "Slice: invalid dimensions");  // cpu_backend.go:292-294
  FL_CHECK(c, i >= 0 && j >= 0 && k <= s->rows && l <= s->cols, "Slice [%lld:%lld, %lld:%lld] outside a %lldx%lld tensor",
           (long long)i, (long long)k, (long long)j, (long long)l, (long long)s->rows, (long long)s->cols);
  FL_CHECK(c, d->dtype == s->dtype && fits(d, (k - i) * (l - j)), "Slice: destination must hold %lldx%lld of the source dtype",
           (long long)(k - i), (long long)(l - j));
  touch(d);
  const int64_t es = dtype_size(s->dtype);
  FL_CUDA(c, cudaMemcpy2DAsync(d->ptr, (size_t)((l - j) * es), (const char*)s->ptr + (i * s->cols + j) * es,
                               (size_t)(s->cols * es), (size_t)((l - j) * es), (size_t)(k - i), cudaMemcpyDeviceToDevice,
                               c->stream));
  return FLETCHER_OK;
}

int32_t Cuda_Mul(CudaContextRef ctx, CudaBufferRef a, int32_t transA, CudaBufferRef b, int32_t transB, CudaBufferRef cb,
                 int64_t m, int64_t n, int64_t k) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Buf *A = B(a), *Bm = B(b), *Cm = B(cb);
  FL_CHECK(c, A && Bm && Cm, "Mul: null buffer");
  FL_CHECK(c, m >= 0 && n >= 0 && k >= 0, "Mul: negative shape");
  const int32_t dt = Cm->dtype;
  FL_CHECK(c, A->dtype == dt && Bm->dtype == dt, "Mul: dtype mismatch");
  FL_CHECK(c, fits(A, m * k) && fits(Bm, k * n) && fits(Cm, m * n), "Mul: buffers smaller than %lldx%lld . %lldx%lld",
           (long long)m, (long long)k, (long long)k, (long long)n);
  if (m == 0 || n == 0) return FLETCHER_OK;
  touch(Cm);
  if (k == 0) {  // beta = 0: an empty product is zero
    FL_CUDA(c, cudaMemsetAsync(Cm->ptr, 0, m * n * dtype_size(dt), c->stream));
    return FLETCHER_OK;
  }
  // 16-bit, A not transposed: tensor cores.  B^T stored [n, k] is already the K-major operand;
  // a plain B [k, n] is packed K-major into a temporary first.
  if (dt != FLETCHER_F32 && !transA && gemm_tc_supported(m, n, k, 128) &&
      ((uintptr_t)A->ptr & 15) == 0 && ((uintptr_t)Bm->ptr & 15) == 0 && n % 8 == 0) {
    if (transB) return launch_gemm_tc(c, dt, EPI_STORE, 128, A->ptr, m, k, Bm->ptr, n, Cm->ptr, n, nullptr, nullptr, 0,
                                      nullptr, nullptr, nullptr, 0);
    Temp wk(c);
    int32_t rc = wk.alloc(k * n * 2);
    if (rc) return rc;
    if ((rc = launch_pack_kmajor_16(c, dt, Bm->ptr, k, n, wk.p, 0, 0))) return rc;
    return launch_gemm_tc(c, dt, EPI_STORE, 128, A->ptr, m, k, wk.p, n, Cm->ptr, n, nullptr, nullptr, 0, nullptr,
                          nullptr, nullptr, 0);
  }
  // SIMT (fp32 accumulation; the fp32 parity path): strides express the T() views.
  const int64_t sam = transA ? 1 : k, sak = transA ? m : 1;
  const int64_t sbk = transB ? 1 : n, sbn = transB ? k : 1;
  return launch_gemm_simt_strided(c, dt, A->ptr, sam, sak, Bm->ptr, sbk, sbn, Cm->ptr, n, m, n, k, nullptr,
                                  FLETCHER_ACT_IDENTITY);
}

}  // extern "C"
