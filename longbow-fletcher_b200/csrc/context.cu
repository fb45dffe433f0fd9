// Context, buffers and host<->device copies of the C ABI (include/fletcher_cuda.h).
// Replaces Cuda_Init / Cuda_Alloc / Cuda_Copy* of the reference (cuda_backend.cu:17-63),
// which bound the device only once and used synchronous cudaMalloc/cudaMemcpy.
#include <cstdarg>
#include <cmath>
#include <cstring>

#include <algorithm>

#include "common.cuh"

namespace fl {

int32_t set_error(Ctx* c, int32_t code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (c) c->last_error = buf;
  return code;
}

int32_t dev_alloc(Ctx* c, void** p, int64_t bytes) {
  *p = nullptr;
  if (bytes <= 0) bytes = 16;
  cudaError_t e = cudaMallocAsync(p, (size_t)bytes, c->stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(c, FLETCHER_ERR_OOM, "cudaMallocAsync(%lld) failed: %s", (long long)bytes,
                     cudaGetErrorString(e));
  }
  e = cudaMemsetAsync(*p, 0, (size_t)bytes, c->stream);
  if (e != cudaSuccess) return set_error(c, FLETCHER_ERR_CUDA, "memset: %s", cudaGetErrorString(e));
  c->allocated += bytes;
  return FLETCHER_OK;
}

void dev_free(Ctx* c, void* p, int64_t bytes) {
  if (!p) return;
  cudaFreeAsync(p, c->stream);
  c->allocated -= bytes <= 0 ? 16 : bytes;  // mirrors the minimum size dev_alloc charges
}

static int32_t init_on_device(Ctx* c, int device) {
  FL_CUDA(c, cudaSetDevice(device));
  c->device = device;
  FL_CUDA(c, cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  // Keep freed pool memory cached instead of returning it to the driver at each sync.
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  void* e = nullptr;
  int32_t rc = dev_alloc(c, &e, 16);
  if (rc) return rc;
  c->d_err = (int32_t*)e;
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  return FLETCHER_OK;
}

// ---- host-side scalar conversions for Cuda_At / Cuda_Set (one element, no kernel).
// The reference's Float32ToFloat16 (utils.go:13-72); same steps as half_bits_ref on the device.
static uint16_t host_f32_to_half_ref(float f) {
  if (std::isnan(f)) return 0x7E00;
  if (std::isinf(f)) return f > 0 ? 0x7C00 : 0xFC00;
  if (f > 65504.0f) f = 65504.0f;
  else if (f < -65504.0f) f = -65504.0f;
  const float a = std::fabs(f);
  if (a < 6.103515625e-05f && a > 0.0f) return f < 0 ? 0x8000 : 0x0000;
  uint32_t bits;
  memcpy(&bits, &f, 4);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const int e = (int)((bits >> 23) & 0xFF) - 127 + 15;
  const uint32_t frac = (bits >> 13) & 0x3FFu;
  if (e >= 0x1F) return (uint16_t)(sign | 0x7BFFu);
  if (e <= 0) return (uint16_t)sign;
  return (uint16_t)(sign | ((uint32_t)e << 10) | frac);
}
// Float16ToFloat32 (utils.go:75-91).
static float host_half_to_f32_ref(uint16_t h) {
  const uint32_t sign = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, frac = h & 0x3FFu;
  if (e == 0) return 0.0f;
  uint32_t bits = e == 31 ? (sign << 31) | (0xFFu << 23) | (frac << 13)
                          : (sign << 31) | ((e - 15 + 127) << 23) | (frac << 13);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
// IEEE conversions (FLETCHER_HALF_RNE, bf16): cuda_fp16.h / cuda_bf16.h are host-callable.
static uint16_t host_f32_to_half_rne(float f) { return __half_as_ushort(__float2half_rn(f)); }
static float host_half_to_f32_ieee(uint16_t r) { return __half2float(__ushort_as_half(r)); }
static uint32_t host_f32_to_bf16_rne(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }

static Ctx* C(CudaContextRef r) { return reinterpret_cast<Ctx*>(r); }
static Buf* B(CudaBufferRef r) { return reinterpret_cast<Buf*>(r); }

// Converts a float32 staging buffer into dst's dtype.
// fp16 follows the context's conversion mode (ref = the reference's utils.go bytes).
template <typename T>
__global__ void k_from_f32(const float* __restrict__ s, T* __restrict__ d, int64_t n, bool ref) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    d[i] = from_f_host<T>(s[i], ref);
}
template <typename T>
__global__ void k_to_f32(const T* __restrict__ s, float* __restrict__ d, int64_t n, bool ref) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    d[i] = to_f_host<T>(s[i], ref);
}

int32_t convert_from_f32(Ctx* c, const float* src, void* dst, int32_t dtype, int64_t n) {
  if (n <= 0) return FLETCHER_OK;
  int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
  if (dtype == FLETCHER_F32)
    FL_CUDA(c, cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, c->stream));
  else if (dtype == FLETCHER_BF16)
    k_from_f32<__nv_bfloat16><<<blocks, 256, 0, c->stream>>>(src, (__nv_bfloat16*)dst, n, false);
  else
    k_from_f32<__half><<<blocks, 256, 0, c->stream>>>(src, (__half*)dst, n, c->half_mode == FLETCHER_HALF_REFERENCE);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

int32_t convert_to_f32(Ctx* c, const void* src, int32_t dtype, float* dst, int64_t n) {
  if (n <= 0) return FLETCHER_OK;
  int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
  if (dtype == FLETCHER_F32)
    FL_CUDA(c, cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, c->stream));
  else if (dtype == FLETCHER_BF16)
    k_to_f32<__nv_bfloat16><<<blocks, 256, 0, c->stream>>>((const __nv_bfloat16*)src, dst, n, false);
  else
    k_to_f32<__half><<<blocks, 256, 0, c->stream>>>((const __half*)src, dst, n, c->half_mode == FLETCHER_HALF_REFERENCE);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

int32_t stage_to_device(Ctx* c, void* d, const void* h, int64_t bytes) {
  if (bytes <= 0) return FLETCHER_OK;
  const int i = c->stage_next;
  c->stage_next = (i + 1) % Ctx::kStageSlots;
  if (!c->stage_ev[i]) FL_CUDA(c, cudaEventCreateWithFlags(&c->stage_ev[i], cudaEventDisableTiming));
  else FL_CUDA(c, cudaEventSynchronize(c->stage_ev[i]));  // this slot's previous copy has read it
  if (bytes > c->h_stage_cap[i]) {
    if (c->h_stage[i]) cudaFreeHost(c->h_stage[i]);
    c->h_stage[i] = nullptr;
    c->h_stage_cap[i] = 0;
    const int64_t cap = std::max<int64_t>(bytes * 2, 1 << 16);
    FL_CUDA(c, cudaHostAlloc((void**)&c->h_stage[i], (size_t)cap, cudaHostAllocPortable));
    c->h_stage_cap[i] = cap;
  }
  memcpy(c->h_stage[i], h, (size_t)bytes);
  FL_CUDA(c, cudaMemcpyAsync(d, c->h_stage[i], (size_t)bytes, cudaMemcpyHostToDevice, c->stream));
  FL_CUDA(c, cudaEventRecord(c->stage_ev[i], c->stream));
  return FLETCHER_OK;
}

// Frees the staging ring (after the stream has drained).
void free_staging(Ctx* c) {
  for (int i = 0; i < Ctx::kStageSlots; i++) {
    if (c->h_stage[i]) cudaFreeHost(c->h_stage[i]);
    if (c->stage_ev[i]) cudaEventDestroy(c->stage_ev[i]);
    c->h_stage[i] = nullptr;
    c->h_stage_cap[i] = 0;
    c->stage_ev[i] = nullptr;
  }
  c->stage_next = 0;
}

// Reads and clears the device error flag (after the stream has been synchronised).
int32_t check_device_flag(Ctx* c) {
  int32_t h = 0;
  FL_CUDA(c, cudaMemcpy(&h, c->d_err, 4, cudaMemcpyDeviceToHost));
  if (h != kDevOk) {
    cudaMemset(c->d_err, 0, 4);
    return set_error(c, FLETCHER_ERR_DEVICE_WAIT,
                     "a kernel's bounded wait expired (device code %d); results are invalid", h);
  }
  return FLETCHER_OK;
}

}  // namespace fl

using namespace fl;

extern "C" {

CudaContextRef Cuda_Init(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return nullptr;
  }
  Ctx* c = new Ctx();
  if (init_on_device(c, 0) != FLETCHER_OK) {
    fprintf(stderr, "Cuda_Init: %s\n", c->last_error.c_str());
    delete c;
    return nullptr;
  }
  return c;
}

int32_t Cuda_GetDeviceCount(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int32_t Cuda_SetDevice(CudaContextRef ctx, int32_t device) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  int n = Cuda_GetDeviceCount();
  FL_CHECK(c, device >= 0 && device < n, "SetDevice: index %d out of range [0,%d)", device, n);
  if (device == c->device) return FLETCHER_OK;
  {
    DeviceGuard g(c);
    cudaStreamSynchronize(c->stream);
    free_staging(c);  // the ring's events belong to the old device
    cudaFree(c->d_err);
    cudaStreamDestroy(c->stream);
  }
  c->allocated -= 16;
  return init_on_device(c, device);
}

void Cuda_FreeContext(CudaContextRef ctx) {
  Ctx* c = C(ctx);
  if (!c) return;
  DeviceGuard g(c);
  cudaStreamSynchronize(c->stream);
  free_staging(c);
  cudaFree(c->d_err);
  cudaStreamDestroy(c->stream);
  delete c;
}

void* Cuda_HostAlloc(CudaContextRef ctx, int64_t bytes) {
  Ctx* c = C(ctx);
  if (!c || bytes <= 0) return nullptr;
  DeviceGuard g(c);
  void* p = nullptr;
  if (cudaHostAlloc(&p, (size_t)bytes, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    set_error(c, FLETCHER_ERR_OOM, "cudaHostAlloc of %lld bytes failed", (long long)bytes);
    return nullptr;
  }
  return p;
}

void Cuda_HostFree(CudaContextRef ctx, void* p) {
  Ctx* c = C(ctx);
  if (!p) return;
  if (c) cudaSetDevice(c->device);
  cudaFreeHost(p);
}

int32_t Cuda_GetLastError(CudaContextRef ctx, char* buf, int32_t len) {
  Ctx* c = C(ctx);
  if (!buf || len <= 0) return FLETCHER_ERR_INVALID;
  const char* s = c ? c->last_error.c_str() : "null context";
  strncpy(buf, s, (size_t)len - 1);
  buf[len - 1] = 0;
  return FLETCHER_OK;
}

int32_t Cuda_Synchronize(CudaContextRef ctx) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  return check_device_flag(c);
}

void* Cuda_GetStream(CudaContextRef ctx) { return ctx ? (void*)C(ctx)->stream : nullptr; }

int64_t Cuda_GetLaunchCount(CudaContextRef ctx) { return ctx ? C(ctx)->launches : -1; }

int32_t Cuda_MemGetInfo(CudaContextRef ctx, int64_t* allocated, int64_t* total) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  size_t fr = 0, tot = 0;
  FL_CUDA(c, cudaMemGetInfo(&fr, &tot));
  if (allocated) *allocated = c->allocated;
  if (total) *total = (int64_t)tot;
  return FLETCHER_OK;
}

CudaBufferRef Cuda_AllocTensor(CudaContextRef ctx, int64_t rows, int64_t cols, int32_t dtype) {
  Ctx* c = C(ctx);
  if (!c || rows < 0 || cols < 0 || dtype < 0 || dtype > 2) return nullptr;
  DeviceGuard g(c);
  Buf* b = new Buf();
  b->ctx = c;
  b->rows = rows;
  b->cols = cols;
  b->dtype = dtype;
  b->bytes = rows * cols * dtype_size(dtype);
  if (dev_alloc(c, &b->ptr, b->bytes) != FLETCHER_OK) {
    delete b;
    return nullptr;
  }
  return b;
}

CudaBufferRef Cuda_Alloc(CudaContextRef ctx, int64_t size) {
  if (size < 0) return nullptr;
  return Cuda_AllocTensor(ctx, 1, (size + 3) / 4, FLETCHER_F32);
}

int32_t Cuda_FreeBuffer(CudaContextRef ctx, CudaBufferRef buf) {
  Buf* b = B(buf);
  if (!b) return FLETCHER_OK;
  Ctx* c = ctx ? C(ctx) : b->ctx;
  DeviceGuard g(c);
  dev_free(c, b->ptr, b->bytes);
  dev_free(c, b->packed, b->packed_bytes);
  dev_free(c, b->bias32, b->bias32_bytes);
  delete b;
  return FLETCHER_OK;
}

int32_t Cuda_CopyToDevice(CudaBufferRef buf, int64_t offset, const void* data, int64_t size) {
  Buf* b = B(buf);
  if (!b) return FLETCHER_ERR_INVALID;
  Ctx* c = b->ctx;
  DeviceGuard g(c);
  FL_CHECK(c, offset >= 0 && size >= 0 && offset + size <= b->bytes, "CopyToDevice: range out of bounds");
  touch(b);
  FL_CUDA(c, cudaMemcpyAsync((char*)b->ptr + offset, data, size, cudaMemcpyHostToDevice, c->stream));
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  return FLETCHER_OK;
}

int32_t Cuda_CopyToHost(CudaBufferRef buf, int64_t offset, void* data, int64_t size) {
  Buf* b = B(buf);
  if (!b) return FLETCHER_ERR_INVALID;
  Ctx* c = b->ctx;
  DeviceGuard g(c);
  FL_CHECK(c, offset >= 0 && size >= 0 && offset + size <= b->bytes, "CopyToHost: range out of bounds");
  FL_CUDA(c, cudaMemcpyAsync(data, (char*)b->ptr + offset, size, cudaMemcpyDeviceToHost, c->stream));
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  return FLETCHER_OK;
}

// Handing out the raw pointer counts as a write: the caller may change the contents behind
// the ABI's back.
void* Cuda_GetBufferContents(CudaBufferRef buf) {
  if (!buf) return nullptr;
  touch(B(buf));
  return B(buf)->ptr;
}

int32_t Cuda_BufferInfo(CudaBufferRef buf, int64_t* rows, int64_t* cols, int32_t* dtype) {
  Buf* b = B(buf);
  if (!b) return FLETCHER_ERR_INVALID;
  if (rows) *rows = b->rows;
  if (cols) *cols = b->cols;
  if (dtype) *dtype = b->dtype;
  return FLETCHER_OK;
}

int32_t Cuda_CopyFromFloat32(CudaBufferRef buf, const float* data, int64_t count) {
  Buf* b = B(buf);
  if (!b) return FLETCHER_ERR_INVALID;
  Ctx* c = b->ctx;
  DeviceGuard g(c);
  FL_CHECK(c, count >= 0 && count * dtype_size(b->dtype) <= b->bytes, "CopyFromFloat32: %lld elements exceed the buffer", (long long)count);
  touch(b);
  if (b->dtype == FLETCHER_F32) {
    FL_CUDA(c, cudaMemcpyAsync(b->ptr, data, count * 4, cudaMemcpyHostToDevice, c->stream));
  } else {
    void* stage = nullptr;
    int32_t rc = dev_alloc(c, &stage, count * 4);
    if (rc) return rc;
    FL_CUDA(c, cudaMemcpyAsync(stage, data, count * 4, cudaMemcpyHostToDevice, c->stream));
    rc = convert_from_f32(c, (const float*)stage, b->ptr, b->dtype, count);
    dev_free(c, stage, count * 4);
    if (rc) return rc;
  }
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  return FLETCHER_OK;
}

int32_t Cuda_ToHostFloat32(CudaBufferRef buf, float* data, int64_t count) {
  Buf* b = B(buf);
  if (!b) return FLETCHER_ERR_INVALID;
  Ctx* c = b->ctx;
  DeviceGuard g(c);
  FL_CHECK(c, count >= 0 && count * dtype_size(b->dtype) <= b->bytes, "ToHostFloat32: %lld elements exceed the buffer", (long long)count);
  if (b->dtype == FLETCHER_F32) {
    FL_CUDA(c, cudaMemcpyAsync(data, b->ptr, count * 4, cudaMemcpyDeviceToHost, c->stream));
  } else {
    void* stage = nullptr;
    int32_t rc = dev_alloc(c, &stage, count * 4);
    if (rc) return rc;
    rc = convert_to_f32(c, b->ptr, b->dtype, (float*)stage, count);
    if (rc) return rc;
    FL_CUDA(c, cudaMemcpyAsync(data, stage, count * 4, cudaMemcpyDeviceToHost, c->stream));
    dev_free(c, stage, count * 4);
  }
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  return FLETCHER_OK;
}

int32_t Cuda_SetHalfConversion(CudaContextRef ctx, int32_t mode) {
  Ctx* c = C(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  FL_CHECK(c, mode == FLETCHER_HALF_REFERENCE || mode == FLETCHER_HALF_RNE, "SetHalfConversion: unknown mode %d", mode);
  c->half_mode = mode;
  return FLETCHER_OK;
}

int32_t Cuda_At(CudaBufferRef buf, int64_t row, int64_t col, float* value) {
  Buf* b = B(buf);
  if (!b || !value) return FLETCHER_ERR_INVALID;
  Ctx* c = b->ctx;
  DeviceGuard g(c);
  FL_CHECK(c, row >= 0 && row < b->rows && col >= 0 && col < b->cols, "At(%lld, %lld) outside a %lldx%lld tensor",
           (long long)row, (long long)col, (long long)b->rows, (long long)b->cols);
  const int64_t off = (row * b->cols + col) * dtype_size(b->dtype);
  uint32_t raw = 0;
  FL_CUDA(c, cudaMemcpyAsync(&raw, (char*)b->ptr + off, dtype_size(b->dtype), cudaMemcpyDeviceToHost, c->stream));
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  if (b->dtype == FLETCHER_F32) memcpy(value, &raw, 4);
  else if (b->dtype == FLETCHER_BF16) {
    const uint32_t w = raw << 16;
    memcpy(value, &w, 4);
  } else {
    *value = c->half_mode == FLETCHER_HALF_REFERENCE ? host_half_to_f32_ref((uint16_t)raw)
                                                     : host_half_to_f32_ieee((uint16_t)raw);
  }
  return FLETCHER_OK;
}

int32_t Cuda_Set(CudaBufferRef buf, int64_t row, int64_t col, float value) {
  Buf* b = B(buf);
  if (!b) return FLETCHER_ERR_INVALID;
  Ctx* c = b->ctx;
  DeviceGuard g(c);
  FL_CHECK(c, row >= 0 && row < b->rows && col >= 0 && col < b->cols, "Set(%lld, %lld) outside a %lldx%lld tensor",
           (long long)row, (long long)col, (long long)b->rows, (long long)b->cols);
  touch(b);
  const int64_t off = (row * b->cols + col) * dtype_size(b->dtype);
  uint32_t raw = 0;
  if (b->dtype == FLETCHER_F32) memcpy(&raw, &value, 4);
  else if (b->dtype == FLETCHER_BF16) raw = host_f32_to_bf16_rne(value);
  else raw = c->half_mode == FLETCHER_HALF_REFERENCE ? host_f32_to_half_ref(value) : host_f32_to_half_rne(value);
  FL_CUDA(c, cudaMemcpyAsync((char*)b->ptr + off, &raw, dtype_size(b->dtype), cudaMemcpyHostToDevice, c->stream));
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  return FLETCHER_OK;
}

}  // extern "C"
