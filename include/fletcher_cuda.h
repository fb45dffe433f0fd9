/*
 * fletcher_cuda.h — C ABI of libcuda_fletcher.so, the B200 (sm_100a) backend for the
 * embedding forward pass of longbow-fletcher.
 *
 * The library replaces the reference's CUDA shim (internal/device/cuda_bridge.h:17-53 +
 * internal/device/cuda_backend.cu) behind the Go device.Backend / device.Tensor interface
 * (internal/device/device.go:5-162).  The style of the reference bridge is kept: C linkage,
 * opaque context and buffer handles, row-major (rows, cols) tensors, Linear weights stored
 * (in, out), activation codes equal to device.ActivationType.  Differences:
 *   - every call returns an int32 status (FLETCHER_OK = 0); Cuda_GetLastError gives the text,
 *   - sizes are 64-bit,
 *   - buffers carry a dtype (device.DataType plus BFloat16 = 2),
 *   - variable-length attention, RoPE and pooling take per-sequence lengths,
 *   - a whole-model entry point (Cuda_Model_*) runs BertModel.ForwardBatch
 *     (internal/embeddings/model/bert.go:149-169) with fused kernels.
 * Every call binds the context's device first, so calls may come from any host thread
 * (goroutines migrate between OS threads).  Calls on one context are ordered on that
 * context's stream; a context must not be used from two threads at the same time.
 */
#ifndef FLETCHER_CUDA_H
#define FLETCHER_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with -fvisibility=hidden; everything declared here is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef void* CudaContextRef; /* cuda_bridge.h:14 */
typedef void* CudaBufferRef;  /* cuda_bridge.h:15 */
typedef void* CudaModelRef;

/* ---- status codes */
enum {
  FLETCHER_OK = 0,
  FLETCHER_ERR_INVALID = 1,     /* bad argument, shape or dtype */
  FLETCHER_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  FLETCHER_ERR_OOM = 3,         /* device allocation failed */
  FLETCHER_ERR_UNSUPPORTED = 4, /* shape/dtype combination this build does not handle */
  FLETCHER_ERR_DEVICE_WAIT = 5  /* a kernel's bounded wait expired; the result is invalid */
};

/* ---- device.DataType (device.go:119-124) + BFloat16 */
enum { FLETCHER_F32 = 0, FLETCHER_F16 = 1, FLETCHER_BF16 = 2 };

/* ---- fp32 <-> fp16 conversion of host-facing copies (Cuda_SetHalfConversion).
 * REFERENCE (the default) reproduces the reference's Float32ToFloat16 / Float16ToFloat32
 * (internal/device/utils.go:13-91), which its fp16 CUDA backend applies to CopyFromFloat32,
 * Set and ToHost (cuda_linux.go:128,148,163): mantissa truncated, |x| < 2^-14 flushed to a
 * signed zero, finite values saturated to +-65504 (0x7BFF), NaN -> 0x7E00, and fp16
 * subnormals read back as +0.  RNE is IEEE round-to-nearest-even with gradual underflow. */
enum { FLETCHER_HALF_REFERENCE = 0, FLETCHER_HALF_RNE = 1 };

/* ---- device.ActivationType (device.go:126-134) */
enum {
  FLETCHER_ACT_IDENTITY = 0,
  FLETCHER_ACT_GELU = 1, /* GeluFast: tanh-GELU with the Pade tanh (simd.go:66-75) */
  FLETCHER_ACT_TANH = 2, /* TanhFast (simd.go:49-63) */
  FLETCHER_ACT_SOFTMAX = 3,
  FLETCHER_ACT_SWIGLU = 4 /* silu(first half) * second half (cpu_backend.go:636-654) */
};

/* ---- pooling heads */
enum {
  FLETCHER_POOL_CLS_TANH = 0, /* BertPooler: CLS row -> Dense -> TanhFast (bert.go:441-488) */
  FLETCHER_POOL_MEAN_L2 = 1   /* mean over each sequence's rows, then L2 normalisation */
};

/* BertConfig (bert.go:20-30) plus the RoPE base, which the reference hard-codes to 10000
 * (cpu_backend.go:790).  position_type: 0 absolute (learned table), 1 RoPE. */
typedef struct FletcherBertConfig {
  int32_t vocab_size;
  int32_t hidden;
  int32_t num_layers;
  int32_t num_heads;
  int32_t intermediate;
  int32_t max_positions;
  int32_t activation;    /* FLETCHER_ACT_GELU or FLETCHER_ACT_SWIGLU */
  int32_t position_type; /* 0 absolute, 1 RoPE */
  float layer_norm_eps;
  float rope_base;
} FletcherBertConfig;

/* ================================================================ context
 * Cuda_Init: cuda_bridge.h:19.  Creates a context on device 0 with its own stream.
 * Returns NULL when no CUDA device is usable. */
CudaContextRef Cuda_Init(void);
/* cuda_bridge.h:20; 0 when CUDA is unavailable. */
int32_t Cuda_GetDeviceCount(void);
/* cuda_bridge.h:21 (device.Backend.SetDevice, device.go:155).  Re-creates the stream on the
 * new device; buffers made earlier stay on their device. */
int32_t Cuda_SetDevice(CudaContextRef ctx, int32_t device);
/* cuda_bridge.h:22 */
void Cuda_FreeContext(CudaContextRef ctx);
/* Copies the last error message of this context (NUL-terminated) into buf. */
int32_t Cuda_GetLastError(CudaContextRef ctx, char* buf, int32_t len);
/* cuda_bridge.h:51 (device.Backend.Synchronize, device.go:149).  Also reports a bounded
 * device wait that expired since the last check (FLETCHER_ERR_DEVICE_WAIT). */
int32_t Cuda_Synchronize(CudaContextRef ctx);
/* The context's cudaStream_t, for callers that time or order work around it. */
void* Cuda_GetStream(CudaContextRef ctx);
/* Number of kernels this context has launched so far (for launch accounting). */
int64_t Cuda_GetLaunchCount(CudaContextRef ctx);
/* Test hook without a counterpart in the reference: runs the bounded device wait that every
 * tensor-core kernel uses on an mbarrier that nothing completes, with a limit of limit_cycles
 * (0 < limit <= the production limit of about 2 s); sleeping selects the sleeping wait, else the
 * spinning one.  Expected result: FLETCHER_ERR_DEVICE_WAIT, with the context still usable. */
int32_t Cuda_Debug_WaitTimeoutProbe(CudaContextRef ctx, int64_t limit_cycles, int32_t sleeping);
/* device.Backend.GetVRAMUsage (device.go:161): bytes held by this context's buffers, and
 * the device's total memory. */
int32_t Cuda_MemGetInfo(CudaContextRef ctx, int64_t* allocated, int64_t* total);
/* Selects the fp16 conversion (FLETCHER_HALF_REFERENCE or FLETCHER_HALF_RNE) used from now on
 * by this context's Cuda_CopyFromFloat32, Cuda_ToHostFloat32, Cuda_At, Cuda_Set, Cuda_Cast,
 * the fp16 output of Cuda_Model_ForwardBatchEx/Async and the fp16 packing of Cuda_Model_LoadRaw.
 * The reference's backend has only its own conversion (utils.go:13-91); RNE has no
 * counterpart there. */
int32_t Cuda_SetHalfConversion(CudaContextRef ctx, int32_t mode);

/* ================================================================ buffers
 * Cuda_Alloc: cuda_bridge.h:25 (size in bytes, dtype f32).  Cuda_AllocTensor allocates
 * rows*cols elements of dtype (device.Backend.NewTensorWithType, device.go:140).
 * Memory comes from a stream-ordered pool and is zero-filled. */
CudaBufferRef Cuda_Alloc(CudaContextRef ctx, int64_t size);
CudaBufferRef Cuda_AllocTensor(CudaContextRef ctx, int64_t rows, int64_t cols, int32_t dtype);
/* cuda_bridge.h:26 */
int32_t Cuda_FreeBuffer(CudaContextRef ctx, CudaBufferRef buf);
/* cuda_bridge.h:27-29: raw byte copies (synchronous with respect to the host). */
int32_t Cuda_CopyToDevice(CudaBufferRef buf, int64_t offset, const void* data, int64_t size);
int32_t Cuda_CopyToHost(CudaBufferRef buf, int64_t offset, void* data, int64_t size);
/* cuda_bridge.h:30: the device pointer. */
void* Cuda_GetBufferContents(CudaBufferRef buf);
int32_t Cuda_BufferInfo(CudaBufferRef buf, int64_t* rows, int64_t* cols, int32_t* dtype);
/* device.Tensor.CopyFromFloat32 / ToHost (device.go:24-27): float32 host data converted to
 * or from the buffer's dtype on the device (cuda_linux.go:139-169 converts on the host). */
int32_t Cuda_CopyFromFloat32(CudaBufferRef buf, const float* data, int64_t count);
int32_t Cuda_ToHostFloat32(CudaBufferRef buf, float* data, int64_t count);
/* device.Tensor.At / Set (device.go:14-15; cuda_linux.go:119-133): one element (row, col) of a
 * (rows, cols) buffer, read into or written from a float32, fp16 with the context's
 * conversion.  Synchronous. */
int32_t Cuda_At(CudaBufferRef buf, int64_t row, int64_t col, float* value);
int32_t Cuda_Set(CudaBufferRef buf, int64_t row, int64_t col, float value);
/* device.Tensor.Copy (cpu_backend.go:259-286, cuda_linux.go:171-174): count elements from
 * src[srcOffset..] to dst[dstOffset..] on the device, converted to dst's dtype when the
 * dtypes differ.  Offsets and count are in elements. */
int32_t Cuda_Copy(CudaContextRef ctx, CudaBufferRef dst, int64_t dstOffset, CudaBufferRef src,
                  int64_t srcOffset, int64_t count);
/* device.Tensor.Slice(i, k, j, l) (cpu_backend.go:288-303): dst (a dense (k-i, l-j) buffer of
 * src's dtype) receives a COPY of src[i:k, j:l], as the reference's CPU backend returns a copy,
 * not a view.  k > i and l > j, as the reference panics otherwise. */
int32_t Cuda_Slice(CudaContextRef ctx, CudaBufferRef src, int64_t i, int64_t k, int64_t j, int64_t l,
                   CudaBufferRef dst);

/* ================================================================ tensor ops
 * All tensors are row-major and dense.  Buffers of one op share a dtype except where noted
 * (LayerNorm gamma/beta are always f32, as in bert.go:279-280). */

/* cuda_bridge.h:33-36 (device.Tensor.Linear / LinearActivation, cpu_backend.go:612-660):
 * result = act(input[rows,inCols] . weight[inCols,outCols] + bias).  For SwiGLU the
 * result has outCols/2 columns.  bias may be NULL.  For 16-bit buffers the tensor-core layout
 * of the weight (K-major, SwiGLU-interleaved) and the fp32 bias are built on the first call
 * and kept with the weight / bias buffer until that buffer is written through this ABI
 * (any call that outputs to it, Cuda_CopyToDevice, Cuda_CopyFromFloat32, Cuda_Set) or its
 * device pointer is handed out by Cuda_GetBufferContents, which invalidate them. */
int32_t Cuda_Linear_Fused(CudaContextRef ctx, CudaBufferRef input, int64_t rows, int64_t inCols,
                          CudaBufferRef weight, int64_t outCols, CudaBufferRef bias,
                          CudaBufferRef result, int32_t activation);
/* device.Tensor.Mul(a, b) with the T() view flag of each operand (cpu_backend.go:306-372):
 * c[m, n] = op(a) . op(b), alpha 1 / beta 0, fp32 accumulation.  a is stored dense as [m, k]
 * (transA = 0) or [k, m] (transA = 1); b as [k, n] (transB = 0) or [n, k] (transB = 1); all
 * three share one dtype.  16-bit products with transA = 0 run on the tensor cores. */
int32_t Cuda_Mul(CudaContextRef ctx, CudaBufferRef a, int32_t transA, CudaBufferRef b, int32_t transB,
                 CudaBufferRef c, int64_t m, int64_t n, int64_t k);
/* cuda_bridge.h:38-40 (cpu_backend.go:541-601).  input may equal result. */
int32_t Cuda_LayerNorm(CudaContextRef ctx, CudaBufferRef input, CudaBufferRef gamma,
                       CudaBufferRef beta, CudaBufferRef result, int64_t rows, int64_t cols,
                       float eps);
/* device.Tensor.AddLayerNorm (cpu_backend.go:603-610): x = LayerNorm(x + residual). */
int32_t Cuda_AddLayerNorm(CudaContextRef ctx, CudaBufferRef x, CudaBufferRef residual,
                          CudaBufferRef gamma, CudaBufferRef beta, int64_t rows, int64_t cols,
                          float eps);
/* cuda_bridge.h:42-43: SoftmaxFast per row (simd.go:78-99). */
int32_t Cuda_Softmax(CudaContextRef ctx, CudaBufferRef input, CudaBufferRef result, int64_t rows,
                     int64_t cols);
/* cuda_bridge.h:45-46 (cpu_backend.go:496-510): output[i] = table[indices[i]].  indices is
 * a host int32 array here (the Go caller holds []int). */
int32_t Cuda_Gather(CudaContextRef ctx, CudaBufferRef table, const int32_t* indices,
                    CudaBufferRef output, int64_t indicesCount, int64_t cols);
/* Elementwise ops of device.Tensor (device.go:42-60), in place on x. */
int32_t Cuda_Add(CudaContextRef ctx, CudaBufferRef x, CudaBufferRef other, int64_t count);
int32_t Cuda_Scale(CudaContextRef ctx, CudaBufferRef x, float val, int64_t count);
int32_t Cuda_AddScalar(CudaContextRef ctx, CudaBufferRef x, float val, int64_t count);
int32_t Cuda_AddBias(CudaContextRef ctx, CudaBufferRef x, CudaBufferRef bias, int64_t rows,
                     int64_t cols);
int32_t Cuda_Activation(CudaContextRef ctx, CudaBufferRef x, int64_t rows, int64_t cols,
                        int32_t activation);
/* device.Tensor.Cast (device.go:111): dst = src converted to dst's dtype. */
int32_t Cuda_Cast(CudaContextRef ctx, CudaBufferRef src, CudaBufferRef dst, int64_t count);
/* device.Tensor.HasNaN (device.go:116): *result = 1 if any NaN or Inf. */
int32_t Cuda_HasNaN(CudaContextRef ctx, CudaBufferRef x, int64_t count, int32_t* result);

/* cuda_bridge.h:48-49 (device.Tensor.Attention, cpu_backend.go:662-758): uniform batches,
 * q/k/v/result [batch*seqLen, hidden], numHeads heads, softmax(scale * Q K^T) V. */
int32_t Cuda_Attention_Fused(CudaContextRef ctx, CudaBufferRef q, CudaBufferRef k,
                             CudaBufferRef v, CudaBufferRef result, int64_t batchSize,
                             int64_t seqLen, int64_t hidden, int32_t numHeads, float scale);
/* device.Tensor.AttentionVarLen (device.go:92, cpu_backend.go:66-132): packed sequences
 * of the given lengths (host array), per-sequence multi-head attention. */
int32_t Cuda_Attention_VarLen(CudaContextRef ctx, CudaBufferRef q, CudaBufferRef k,
                              CudaBufferRef v, CudaBufferRef result, const int32_t* lengths,
                              int32_t numSeqs, int64_t hidden, int32_t numHeads, float scale);
/* No counterpart in the reference.  Cuda_Attention_VarLen for callers that must not allocate
 * device memory during the call (memory fully reserved by admission control, or an allocator
 * owned by a host framework): the per-call metadata lives in one fixed device array per GPU
 * of FLETCHER_NOALLOC_SCRATCH_INTS int32 (1 MiB, held until the process exits) instead of a
 * per-call allocation.  A call needs numSeqs+1 ints (f32) or about numSeqs+1 + 2 per 128-row
 * query tile (16-bit); larger batches return FLETCHER_ERR_INVALID.  All calls on a device
 * share the array: calls that overlap on the GPU (two contexts or streams) race; calls on one
 * context are ordered.  The first call on each device resolves the array's address
 * (cudaGetSymbolAddress); make it before any stream capture. */
#define FLETCHER_NOALLOC_SCRATCH_INTS (1 << 18)
int32_t Cuda_Attention_VarLen_NoAlloc(CudaContextRef ctx, CudaBufferRef q, CudaBufferRef k,
                                      CudaBufferRef v, CudaBufferRef result,
                                      const int32_t* lengths, int32_t numSeqs, int64_t hidden,
                                      int32_t numHeads, float scale);
/* cuda_bridge.h:51-52 (cpu_backend.go:760-805): rotate-half RoPE in place, base 10000,
 * position = row % seqLen. */
int32_t Cuda_ApplyRoPE(CudaContextRef ctx, CudaBufferRef data, int64_t batchSize, int64_t seqLen,
                       int32_t numHeads, int32_t headDim);
/* RoPE over packed sequences: position = row index within its own sequence. */
int32_t Cuda_ApplyRoPE_VarLen(CudaContextRef ctx, CudaBufferRef data, const int32_t* lengths,
                              int32_t numSeqs, int32_t numHeads, int32_t headDim, float base);
/* Mean pooling + L2 normalisation: hidden [sum(lengths), cols] -> out [numSeqs, cols] f32.
 * (No counterpart in the reference; the spec's pooling head.) */
int32_t Cuda_MeanPoolL2(CudaContextRef ctx, CudaBufferRef hidden, const int32_t* lengths,
                        int32_t numSeqs, int64_t cols, CudaBufferRef out);

/* ================================================================ whole model
 * BertModel (bert.go:77-169) on the device, with fused kernels: tcgen05 GEMMs with fused
 * epilogues (bias, RoPE, GELU/SwiGLU, residual) and flash attention for bf16/f16;
 * fp32 SIMT kernels with the reference's fast-math formulas for f32. */
int32_t Cuda_Model_Create(CudaContextRef ctx, const FletcherBertConfig* cfg, int32_t dtype,
                          CudaModelRef* out);
/* Loads weights from one host float32 blob in LoadFromRawBinary order
 * (internal/embeddings/weights/loader.go:29-90); count must equal Cuda_Model_WeightCount. */
int32_t Cuda_Model_LoadRaw(CudaModelRef model, const float* blob, int64_t count);
int64_t Cuda_Model_WeightCount(const FletcherBertConfig* cfg);
/* One checkpoint tensor, by its name in the reference's SafeTensors loader (LoadFromSafeTensors,
 * internal/embeddings/weights/loader.go:155-296: "embeddings.word_embeddings.weight",
 * "encoder.layer.3.attention.self.query.weight", "pooler.dense.bias", ...), straight from host
 * memory in its stored dtype (FLETCHER_F32, F16 or BF16) into the model's device layout: no
 * host fp32 copy of the model is made (the reference widens on the host and rejects F16,
 * loader.go:210-215).  rows x cols is the tensor as given; transposed = 1 marks a Linear weight
 * stored (out, in), the PyTorch layout that loader.go:229-251 transposes; 0 means (in, out).
 * Only Linear weights (2-D ".weight" outside the embeddings and LayerNorms) may be transposed.
 * Errors follow the loader: unknown name, size or shape mismatch -> FLETCHER_ERR_INVALID.
 * fp32 data becomes fp16 with the context's conversion (the reference's CopyFromFloat32 bytes
 * by default).  Synchronous: `data` may be freed on return.  The model can run once every
 * tensor of Cuda_Model_TensorCount has been loaded (Cuda_Model_IsLoaded). */
int32_t Cuda_Model_LoadTensor(CudaModelRef model, const char* name, int32_t dtype, const void* data, int64_t rows,
                              int64_t cols, int32_t transposed);
/* Number of checkpoint tensors of a config, and the name of tensor `index` in LoadFromSafeTensors
 * order (loader.go:257-293). */
int32_t Cuda_Model_TensorCount(const FletcherBertConfig* cfg);
int32_t Cuda_Model_TensorName(const FletcherBertConfig* cfg, int32_t index, char* buf, int32_t len);
/* 1 once the model holds a full set of weights (Cuda_Model_LoadRaw, or every LoadTensor). */
int32_t Cuda_Model_IsLoaded(CudaModelRef model);
/* BertModel.ForwardBatch(ids, lengths) (bert.go:149): host ids (packed, sum(lengths)
 * entries) and lengths in, host float32 out[numSeqs, hidden].  Synchronous. */
int32_t Cuda_Model_ForwardBatch(CudaModelRef model, const int32_t* ids, const int32_t* lengths,
                                int32_t numSeqs, int32_t pooling, float* out);
/* Cuda_Model_ForwardBatch with the vectors returned as out_dtype (FLETCHER_F32, F16 or BF16;
 * converted on the device, so half the bytes cross PCIe; fp16 with the context's conversion,
 * the reference's bytes by default, bf16 rounded to nearest even): the reference's fp16
 * transport, Cast(Float16) + ExtractBytes (embeddings.go:256-288). */
int32_t Cuda_Model_ForwardBatchEx(CudaModelRef model, const int32_t* ids, const int32_t* lengths,
                                  int32_t numSeqs, int32_t pooling, int32_t out_dtype, void* out);
/* Asynchronous Cuda_Model_ForwardBatchEx for a batcher's double buffering (the reference's
 * per-device loop, embeddings.go:678-815, waits for each batch before forming the next).  It
 * enqueues the H2D copy of ids, the pass and the D2H copy of the vectors into `out` on the
 * context's stream and returns without waiting; *ticket identifies the batch.  lengths are
 * consumed before the call returns.  ids and out must stay valid until Cuda_Model_Wait(ticket)
 * returns; with pinned buffers (Cuda_HostAlloc) the copies overlap other batches' compute.  At
 * most 8 batches are in flight: a ninth call first waits for the oldest. */
int32_t Cuda_Model_ForwardBatchAsync(CudaModelRef model, const int32_t* ids, const int32_t* lengths,
                                     int32_t numSeqs, int32_t pooling, int32_t out_dtype, void* out,
                                     int64_t* ticket);
/* Waits until batch `ticket` has finished and its vectors are in host memory; reports a
 * device-side error of any batch up to it. */
int32_t Cuda_Model_Wait(CudaModelRef model, int64_t ticket);
/* Page-locked host memory for the asynchronous copies (cudaHostAlloc / cudaFreeHost). */
void* Cuda_HostAlloc(CudaContextRef ctx, int64_t bytes);
void Cuda_HostFree(CudaContextRef ctx, void* p);
/* Same pass with device-resident ids (int32, packed) and a device float32 output; lengths
 * stay on the host (they shape the launch).  Asynchronous on the context's stream. */
int32_t Cuda_Model_ForwardBatchDevice(CudaModelRef model, const int32_t* d_ids,
                                      const int32_t* lengths, int32_t numSeqs, int32_t pooling,
                                      float* d_out);
/* CUDA-graph replay of repeated batch shapes (on by default): a shape (lengths, pooling,
 * buffers) runs eagerly the first time, is captured the second time and replayed after that,
 * which removes per-kernel host launch cost.  Disabling also drops the cached graphs. */
int32_t Cuda_Model_SetGraphs(CudaModelRef model, int32_t enable);
/* Stage timing: when enabled, every stage of the forward pass is bracketed by CUDA events on
 * the context's stream.  Cuda_Model_StageTimes synchronises, writes the summed milliseconds
 * (and the number of timed calls) per stage since the last read into ms[n] / launches[n]
 * (launches may be NULL), then resets.  Stage indices: */
enum {
  FLETCHER_STAGE_EMBED = 0,
  FLETCHER_STAGE_GEMM_QKV = 1,
  FLETCHER_STAGE_ROPE = 2,
  FLETCHER_STAGE_ATTENTION = 3,
  FLETCHER_STAGE_GEMM_O = 4,
  FLETCHER_STAGE_LAYERNORM = 5,
  FLETCHER_STAGE_GEMM_UP = 6,
  FLETCHER_STAGE_ACTIVATION = 7,
  FLETCHER_STAGE_GEMM_DOWN = 8,
  FLETCHER_STAGE_POOL = 9,
  FLETCHER_NUM_STAGES = 10
};
int32_t Cuda_Model_SetStageTiming(CudaModelRef model, int32_t enable);
int32_t Cuda_Model_StageTimes(CudaModelRef model, float* ms, int64_t* launches, int32_t n);
/* Copies the last hidden state [sum(lengths), hidden] of the previous forward as float32.  A
 * mean-pooled forward of a 16-bit model normalises its final rows inside the pooling kernel and
 * does not store them: LastHidden then fails unless Cuda_Model_SetKeepHidden(model, 1) was set
 * before that forward (which keeps the separate final LayerNorm pass). */
int32_t Cuda_Model_LastHidden(CudaModelRef model, float* host_out, int64_t count);
int32_t Cuda_Model_SetKeepHidden(CudaModelRef model, int32_t enable);
int32_t Cuda_Model_Free(CudaModelRef model);

/* ---- Host runtime: multi-GPU embedder and request server (internal/embeddings/embeddings.go)
 *
 * Native restatement of the reference's Embedder: one model replica per device, each driven by
 * its own host thread that keeps two device batches in flight (Cuda_Model_ForwardBatchAsync into
 * pinned buffers), requests split across replicas by token count weighted by each replica's
 * measured throughput (embeddings.go:436-501) and cut into dynamic batches of at most max_batch
 * sequences / max_tokens tokens (embeddings.go:704-731); and of its server front end: a request
 * queue whose batcher keeps at most max_in_flight sequences handed to the replicas (server.go:101,
 * the sequence semaphore) and dispatches batches round-robin to replicas holding fewer than
 * jobs_per_replica batches.  Packing ([CLS] ids [SEP] per text, embeddings.go:742-749) and
 * tokenisation stay with the caller. */
typedef void* CudaEmbedderRef;
typedef void* CudaServerRef;

/* Replicas over existing models, one per element of models[] (each on its own context; two
 * models may share a device).  The embedder drives the models from its own threads: do not call
 * them elsewhere while it runs.  pooling: FLETCHER_POOL_*.  max_tokens <= 0: 65536 tokens per
 * batch on devices with >= 64 GB, else 16384 (the reference's VRAM-dependent default,
 * embeddings.go:177-190). */
int32_t Cuda_Embedder_Create(const CudaModelRef* models, int32_t n, int32_t pooling, int32_t max_batch,
                             int64_t max_tokens, CudaEmbedderRef* out);
/* Test double with no GPU: n replicas that return, for sequence i of a batch, the vector
 * (first id, length, replica index, 0, ...) of width `hidden`, after sleeping delay_us per batch. */
int32_t Cuda_Embedder_CreateFake(int32_t n, int32_t hidden, int64_t delay_us, int32_t max_batch,
                                 int64_t max_tokens, CudaEmbedderRef* out);
/* Embeds packed ids / lengths (numSeqs sequences) into out[numSeqs, hidden] (float32, request
 * order).  Synchronous; may run concurrently with a server on the same embedder. */
int32_t Cuda_Embedder_Embed(CudaEmbedderRef e, const int32_t* ids, const int32_t* lengths, int32_t numSeqs,
                            float* out);
/* Per-replica throughput in sequences/s: 1.0 until the first batch finishes, then that batch's
 * rate, then an exponential average with weight 0.3 on each new batch (embeddings.go:197,
 * 795-804).  Read into tput[n], or set from tput[n] when set != 0. */
int32_t Cuda_Embedder_Throughput(CudaEmbedderRef e, double* tput, int32_t n, int32_t set);
/* Per-replica counters since creation: batches handed to the replica (jobs) and their sequences. */
int32_t Cuda_Embedder_Counts(CudaEmbedderRef e, int64_t* jobs, int64_t* seqs, int32_t n);
int32_t Cuda_Embedder_Hidden(CudaEmbedderRef e);
int32_t Cuda_Embedder_MaxBatch(CudaEmbedderRef e, int32_t* max_batch, int64_t* max_tokens);
/* Text of the last failed call on this embedder (or of a failed request of its servers). */
int32_t Cuda_Embedder_LastError(CudaEmbedderRef e, char* buf, int32_t len);
/* Stops the replica threads (after their queued work).  Does not free the models.  Destroy the
 * embedder's servers first. */
void Cuda_Embedder_Destroy(CudaEmbedderRef e);

/* Request server over an embedder.  max_in_flight <= 0: 16384; jobs_per_replica <= 0: 2. */
int32_t Cuda_Server_Create(CudaEmbedderRef e, int32_t max_in_flight, int32_t jobs_per_replica, CudaServerRef* out);
/* Enqueues n requests.  Request r holds the sequences seq_off[r] .. seq_off[r+1]-1 of
 * lengths[] (seq_off has n+1 entries, seq_off[0] = 0), whose ids lie packed in ids[] in that
 * order; its vectors go to out + seq_off[r] * hidden.  ids and lengths are copied before the call
 * returns; out must stay valid until the request completes.  arrival_ns (may be NULL): each
 * request's arrival on Cuda_Server_Clock's clock, from which its latency counts (an open-loop
 * load schedule); otherwise latency counts from this call.  The requests get consecutive
 * tickets starting at *first_ticket (>= 1).  A request's ids are freed once its batch completes;
 * its completion record (arrival, completion time, status: about 100 bytes) stays until
 * Cuda_Server_Destroy, so a long-running server holds about 100 MB per million requests. */
int32_t Cuda_Server_Submit(CudaServerRef s, int32_t n, const int32_t* ids, const int32_t* lengths,
                           const int64_t* seq_off, const int64_t* arrival_ns, float* out, int64_t* first_ticket);
/* Monotonic clock of the server, nanoseconds. */
int64_t Cuda_Server_Clock(void);
/* Waits up to timeout_s seconds (< 0: no limit) for request `ticket`.  Returns its status
 * (FLETCHER_OK, an error of its batch, or FLETCHER_ERR_INVALID for an unknown ticket); a wait
 * that times out returns -1.  *latency_ns (may be NULL) receives the request's latency. */
int32_t Cuda_Server_Wait(CudaServerRef s, int64_t ticket, double timeout_s, int64_t* latency_ns);
/* Latencies of tickets first .. first+n-1 (-1: not complete, -2: failed). */
int32_t Cuda_Server_Latencies(CudaServerRef s, int64_t first, int64_t n, int64_t* latency_ns);
/* Waits until every submitted request has completed. */
int32_t Cuda_Server_Drain(CudaServerRef s);
typedef struct FletcherServerStats {
  int64_t requests;        /* submitted */
  int64_t completed;
  int64_t batches;         /* batches handed to replicas */
  int64_t max_batch_seqs;  /* largest batch made of two or more requests */
  int64_t max_request_seqs;/* largest single request */
  int64_t max_busy;        /* most sequences in flight at once */
} FletcherServerStats;
int32_t Cuda_Server_Stats(CudaServerRef s, FletcherServerStats* st);
/* Completes every submitted request, then stops the batcher. */
void Cuda_Server_Destroy(CudaServerRef s);
/* The reference's split and batching rules, exported for callers and tests.  SplitByWeight:
 * contiguous [ranges[2d], ranges[2d+1]) of the numSeqs sequences per replica d (n replicas,
 * weights = throughputs, all 0 = equal shares); returns the number of replicas that got a range.
 * DynamicBatches: [start, end) pairs into ranges (capacity cap pairs); returns the count. */
int32_t Cuda_Runtime_SplitByWeight(const int32_t* lengths, int32_t numSeqs, const double* weights, int32_t n,
                                   int32_t* ranges);
int32_t Cuda_Runtime_DynamicBatches(const int32_t* lengths, int32_t numSeqs, int32_t max_batch, int64_t max_tokens,
                                    int32_t* ranges, int32_t cap);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* FLETCHER_CUDA_H */
