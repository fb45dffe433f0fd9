// Context, buffers and host<->device copies of the C ABI (include/fletcher_cuda.h).
// Replaces Cuda_Init / Cuda_Alloc / Cuda_Copy* of the reference (cuda_backend.cu:17-63),
// which bound the device only once and used synchronous cudaMalloc/cudaMemcpy.
#include <cstdarg>
#include <cstring>

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

static Ctx* C(CudaContextRef r) { return reinterpret_cast<Ctx*>(r); }
static Buf* B(CudaBufferRef r) { return reinterpret_cast<Buf*>(r); }

// Converts a float32 staging buffer into dst's dtype.
template <typename T>
__global__ void k_from_f32(const float* __restrict__ s, T* __restrict__ d, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    d[i] = from_f<T>(s[i]);
}
template <typename T>
__global__ void k_to_f32(const T* __restrict__ s, float* __restrict__ d, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    d[i] = to_f<T>(s[i]);
}

int32_t convert_from_f32(Ctx* c, const float* src, void* dst, int32_t dtype, int64_t n) {
  if (n <= 0) return FLETCHER_OK;
  int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
  if (dtype == FLETCHER_F32)
    FL_CUDA(c, cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, c->stream));
  else if (dtype == FLETCHER_BF16)
    k_from_f32<__nv_bfloat16><<<blocks, 256, 0, c->stream>>>(src, (__nv_bfloat16*)dst, n);
  else
    k_from_f32<__half><<<blocks, 256, 0, c->stream>>>(src, (__half*)dst, n);
  FL_LAUNCH(c);
  return FLETCHER_OK;
}

int32_t convert_to_f32(Ctx* c, const void* src, int32_t dtype, float* dst, int64_t n) {
  if (n <= 0) return FLETCHER_OK;
  int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
  if (dtype == FLETCHER_F32)
    FL_CUDA(c, cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, c->stream));
  else if (dtype == FLETCHER_BF16)
    k_to_f32<__nv_bfloat16><<<blocks, 256, 0, c->stream>>>((const __nv_bfloat16*)src, dst, n);
  else
    k_to_f32<__half><<<blocks, 256, 0, c->stream>>>((const __half*)src, dst, n);
  FL_LAUNCH(c);
  return FLETCHER_OK;
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
  delete b;
  return FLETCHER_OK;
}

int32_t Cuda_CopyToDevice(CudaBufferRef buf, int64_t offset, const void* data, int64_t size) {
  Buf* b = B(buf);
  if (!b) return FLETCHER_ERR_INVALID;
  Ctx* c = b->ctx;
  DeviceGuard g(c);
  FL_CHECK(c, offset >= 0 && size >= 0 && offset + size <= b->bytes, "CopyToDevice: range out of bounds");
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

void* Cuda_GetBufferContents(CudaBufferRef buf) { return buf ? B(buf)->ptr : nullptr; }

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

}  // extern "C"
