// Whole-model forward on the device: BertModel.ForwardBatch (bert.go:149-169) with fused
// kernels, behind Cuda_Model_* of include/fletcher_cuda.h.
//
// Per layer (16-bit mode), 7 launches:
//   QKV   = X . Wqkv^T (+b), RoPE on Q|K in the epilogue          (tcgen05 GEMM, EPI_ROPE)
//   CTX   = flash-attention(QKV) over packed sequences            (tcgen05 attention)
//   S     = CTX . Wo^T + bo + X                                   (tcgen05 GEMM, EPI_RESIDUAL)
//   X     = LayerNorm(S)                                          (warp-per-row LN)
//   ACT   = SwiGLU / GeluFast(X . Wi^T + bi)                      (tcgen05 GEMM, EPI_SWIGLU/GELU)
//   S     = ACT . Wd^T + bd + X                                   (tcgen05 GEMM, EPI_RESIDUAL)
//   X     = LayerNorm(S)
// fp32 mode runs the same graph with the SIMT GEMM, a RoPE kernel and the fp32 attention
// kernel, using the reference's fast-math formulas, for parity with its CPU path.
// The residual stream X stays in the model dtype; LayerNorm statistics are fp32.  The kernel
// sequence is captured into a CUDA graph for repeated batch shapes.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <vector>

#include "gemm.cuh"

namespace fl {

struct Layer {
  void* wqkv = nullptr;  // f32: (in,out) [H, 3H]; 16-bit: K-major [3H, H]
  float* bqkv = nullptr;
  void* wo = nullptr;
  float* bo = nullptr;
  float *ln1g = nullptr, *ln1b = nullptr;
  void* wi = nullptr;  // f32: [H, Iup]; 16-bit: K-major [Iup, H] (SwiGLU gate/up interleaved)
  float* bi = nullptr;
  void* wd = nullptr;  // f32: [I, H]; 16-bit: K-major [H, I]
  float* bd = nullptr;
  float *ln2g = nullptr, *ln2b = nullptr;
};

struct Model {
  Ctx* c = nullptr;
  FletcherBertConfig cfg{};
  int32_t dtype = FLETCHER_F32;
  bool loaded = false;
  int64_t H = 0, I = 0, Iup = 0, nh = 0, dh = 0;
  int bn_qkv = 256, bn_o = 128, bn_up = 256, bn_d = 128;
  std::vector<std::pair<void*, int64_t>> allocs;  // everything owned, freed at destroy
  std::vector<uint8_t> tensor_loaded;              // Cuda_Model_LoadTensor: which checkpoint tensors arrived
  void* word = nullptr;
  void* ptab = nullptr;
  void* type0 = nullptr;
  float *eln_g = nullptr, *eln_b = nullptr;
  std::vector<Layer> layers;
  float *wp = nullptr, *bp = nullptr;  // pooler in fp32 (bert.go:459-477 forces fp32)
  float *cos_t = nullptr, *sin_t = nullptr;
  int rope_len = 0;
  // workspace
  int64_t ws_T = 0;
  int32_t ws_B = 0;
  void *X = nullptr, *S = nullptr, *QKV = nullptr, *CTX = nullptr, *ACT = nullptr, *INTER = nullptr;
  int32_t *d_ids = nullptr, *d_cu = nullptr, *d_pos = nullptr;
  int2* d_tiles = nullptr;
  int64_t tiles_cap = 0;
  float* d_out = nullptr;
  float* d_cls = nullptr;
  float* splitk = nullptr;  // split-K partial sums of the GEMMs of small batches
  int64_t splitk_bytes = 0;
  float* lnpool = nullptr;  // chunk sums of the last LayerNorm fused into mean pooling
  int64_t lnpool_bytes = 0;
  bool keep_hidden = false;  // Cuda_Model_SetKeepHidden: store the final hidden state
  bool last_fused = false;   // the previous forward fused its final LayerNorm into the pool
  std::vector<std::pair<void*, int64_t>> ws;
  // pinned staging for per-batch metadata
  uint8_t* h_meta = nullptr;
  int64_t h_meta_cap = 0;
  cudaEvent_t meta_done = nullptr;
  // CUDA graphs of the kernel sequence, per batch shape
  struct GraphEntry {
    std::vector<int32_t> key;
    cudaGraphExec_t exec;
    uint64_t last_use;
    int64_t kernels;
  };
  bool use_graphs = true;
  std::vector<GraphEntry> graphs;
  std::vector<std::vector<int32_t>> graph_seen;
  uint64_t graph_tick = 0;
  int64_t last_T = 0;
  // stage timing
  bool timing = false;
  std::vector<cudaEvent_t> ev_pool;
  // Asynchronous batches (Cuda_Model_ForwardBatchAsync): a completion event per in-flight slot.
  static constexpr int kAsyncSlots = 8;
  cudaEvent_t async_ev[kAsyncSlots] = {};
  int64_t async_issued = 0, async_done = 0;  // tickets issued / known complete
  size_t ev_used = 0;
  struct StageRec {
    int cat;
    cudaEvent_t a, b;
  };
  std::vector<StageRec> stage_recs;
};

static int32_t own(Model* m, void** p, int64_t bytes) {
  int32_t rc = dev_alloc(m->c, p, bytes);
  if (rc == FLETCHER_OK) m->allocs.push_back({*p, bytes});
  return rc;
}

void clear_graphs(Model* m);

static void free_ws(Model* m) {
  clear_graphs(m);  // captured graphs hold the old workspace pointers
  if (m->splitk && m->c->splitk == m->splitk) {  // stop lending the split-K workspace
    m->c->splitk = nullptr;
    m->c->splitk_bytes = 0;
  }
  for (auto& a : m->ws) dev_free(m->c, a.first, a.second);
  m->ws.clear();
  m->ws_T = 0;
  m->ws_B = 0;
}

static int32_t ws_alloc(Model* m, void** p, int64_t bytes) {
  int32_t rc = dev_alloc(m->c, p, bytes);
  if (rc == FLETCHER_OK) m->ws.push_back({*p, bytes});
  return rc;
}

static int32_t ensure_ws(Model* m, int64_t T, int32_t B) {
  if (T <= m->ws_T && B <= m->ws_B) return FLETCHER_OK;
  free_ws(m);
  const int64_t Tc = std::max<int64_t>(T, 128), Bc = std::max<int32_t>(B, 64);
  const int64_t es = dtype_size(m->dtype);
  int32_t rc = 0;
  if ((rc = ws_alloc(m, &m->X, Tc * m->H * es))) return rc;
  if ((rc = ws_alloc(m, &m->S, Tc * m->H * es))) return rc;
  if ((rc = ws_alloc(m, &m->QKV, Tc * 3 * m->H * es))) return rc;
  if ((rc = ws_alloc(m, &m->CTX, Tc * m->H * es))) return rc;
  if ((rc = ws_alloc(m, &m->ACT, Tc * m->I * es))) return rc;
  if (m->dtype == FLETCHER_F32 && (rc = ws_alloc(m, &m->INTER, Tc * m->Iup * es))) return rc;
  if ((rc = ws_alloc(m, (void**)&m->d_ids, Tc * 4))) return rc;
  if ((rc = ws_alloc(m, (void**)&m->d_pos, Tc * 4))) return rc;
  if ((rc = ws_alloc(m, (void**)&m->d_cu, (Bc + 1) * 4))) return rc;
  m->tiles_cap = Tc / 64 + Bc + 1;
  if ((rc = ws_alloc(m, (void**)&m->d_tiles, m->tiles_cap * 8))) return rc;
  if ((rc = ws_alloc(m, (void**)&m->d_out, Bc * m->H * 4))) return rc;
  if ((rc = ws_alloc(m, (void**)&m->d_cls, Bc * m->H * 4))) return rc;
  // Split-K workspace: the largest plan of the four GEMM shapes for batches of up to 1024 tokens.
  m->splitk = nullptr;
  m->splitk_bytes = 0;
  if (m->dtype != FLETCHER_F32) {
    const int64_t shapes[4][2] = {{3 * m->H, m->H}, {m->H, m->H}, {m->Iup, m->H}, {m->H, m->I}};  // N, K
    int64_t need = 0;
    for (int64_t M = 128; M <= std::min<int64_t>(Tc, 1024); M += 128)
      for (const auto& sh : shapes) {
        int sp = 0, per = 0;
        need = std::max(need, gemm_splitk_plan(m->c, M, sh[0], sh[1], &sp, &per));
      }
    if (need > 0) {
      if ((rc = ws_alloc(m, (void**)&m->splitk, need))) return rc;
      m->splitk_bytes = need;
    }
  }
  m->ws_T = Tc;
  m->ws_B = (int32_t)Bc;
  return FLETCHER_OK;
}

static int32_t ensure_rope(Model* m, int32_t need) {
  if (m->cfg.position_type != 1 || need <= m->rope_len) return FLETCHER_OK;
  int32_t len = std::max<int32_t>(need, m->cfg.max_positions);
  if (m->cos_t) {
    dev_free(m->c, m->cos_t, (int64_t)m->rope_len * (m->dh / 2) * 4);
    dev_free(m->c, m->sin_t, (int64_t)m->rope_len * (m->dh / 2) * 4);
    m->cos_t = m->sin_t = nullptr;
  }
  int32_t rc;
  if ((rc = dev_alloc(m->c, (void**)&m->cos_t, (int64_t)len * (m->dh / 2) * 4))) return rc;
  if ((rc = dev_alloc(m->c, (void**)&m->sin_t, (int64_t)len * (m->dh / 2) * 4))) return rc;
  m->rope_len = len;
  clear_graphs(m);  // captured graphs hold the old table pointers
  return launch_rope_build_table(m->c, m->cos_t, m->sin_t, len, (int32_t)m->dh, (double)m->cfg.rope_base);
}

int64_t weight_count(const FletcherBertConfig* c) {
  const int64_t H = c->hidden, I = c->intermediate, Iup = c->activation == FLETCHER_ACT_SWIGLU ? 2 * I : I;
  int64_t n = (int64_t)c->vocab_size * H + (int64_t)c->max_positions * H + 2 * H + 2 * H;
  const int64_t per = 3 * (H * H + H) + (H * H + H) + 2 * H + (H * Iup + Iup) + (I * H + H) + 2 * H;
  return n + per * c->num_layers + H * H + H;
}

// Uploads n fp32 host values to a fresh device array.
static int32_t up_f32(Model* m, float** d, const float* h, int64_t n) {
  int32_t rc = own(m, (void**)d, n * 4);
  if (rc) return rc;
  FL_CUDA(m->c, cudaMemcpyAsync(*d, h, n * 4, cudaMemcpyHostToDevice, m->c->stream));
  return FLETCHER_OK;
}

static bool all_zero(const float* p, int64_t n) {
  for (int64_t i = 0; i < n; i++)
    if (p[i] != 0.0f) return false;
  return true;
}

// A Linear weight (in,out) = [K, N] fp32 on the host -> the layout the GEMM of this dtype
// reads: fp32 (in,out) as is; 16-bit K-major [N, K] (optionally SwiGLU-interleaved).
static int32_t up_weight(Model* m, void** d, const float* h, int64_t K, int64_t N, int perm, int bn, float* staging) {
  Ctx* c = m->c;
  if (m->dtype == FLETCHER_F32) return up_f32(m, (float**)d, h, K * N);
  int32_t rc = own(m, d, K * N * 2);
  if (rc) return rc;
  FL_CUDA(c, cudaMemcpyAsync(staging, h, K * N * 4, cudaMemcpyHostToDevice, c->stream));
  rc = launch_pack_weight_kmajor(c, staging, K, N, *d, m->dtype, perm, bn);
  if (rc) return rc;
  FL_CUDA(c, cudaStreamSynchronize(c->stream));  // staging is reused by the next weight
  return FLETCHER_OK;
}

static int32_t up_table(Model* m, void** d, const float* h, int64_t n, float* staging) {
  Ctx* c = m->c;
  if (m->dtype == FLETCHER_F32) return up_f32(m, (float**)d, h, n);
  int32_t rc = own(m, d, n * 2);
  if (rc) return rc;
  const int64_t chunk = 64ll << 20;  // staging holds at most `chunk` floats
  for (int64_t o = 0; o < n; o += chunk) {
    const int64_t k = std::min(chunk, n - o);
    FL_CUDA(c, cudaMemcpyAsync(staging, h + o, k * 4, cudaMemcpyHostToDevice, c->stream));
    rc = convert_from_f32(c, staging, (uint8_t*)*d + o * 2, m->dtype, k);
    if (rc) return rc;
    FL_CUDA(c, cudaStreamSynchronize(c->stream));
  }
  return FLETCHER_OK;
}

// Frees every weight buffer (a second LoadRaw, or LoadRaw after LoadTensor, starts afresh).
static void release_weights(Model* m) {
  cudaStreamSynchronize(m->c->stream);
  clear_graphs(m);  // captured graphs hold the old weight pointers
  for (auto& a : m->allocs) dev_free(m->c, a.first, a.second);
  m->allocs.clear();
  m->word = m->ptab = m->type0 = nullptr;
  m->eln_g = m->eln_b = nullptr;
  m->layers.clear();
  m->wp = m->bp = nullptr;
  m->loaded = false;
  m->tensor_loaded.clear();
}

static int32_t load_raw(Model* m, const float* blob, int64_t count) {
  Ctx* c = m->c;
  const FletcherBertConfig& cf = m->cfg;
  FL_CHECK(c, count == weight_count(&cf), "LoadRaw: %lld values, expected %lld", (long long)count,
           (long long)weight_count(&cf));
  release_weights(m);
  const int64_t H = m->H, I = m->I, Iup = m->Iup;
  const float* p = blob;
  auto take = [&](int64_t n) {
    const float* r = p;
    p += n;
    return r;
  };
  float* staging = nullptr;
  const int64_t stage_n = std::max<int64_t>({H * 3 * H, H * Iup, I * H, 64ll << 20});
  int32_t rc = dev_alloc(c, (void**)&staging, stage_n * 4);
  if (rc) return rc;
  struct StageFree {
    Ctx* c;
    float* p;
    int64_t n;
    ~StageFree() { dev_free(c, p, n * 4); }
  } sf{c, staging, stage_n};

  const float* word = take((int64_t)cf.vocab_size * H);
  const float* pos = take((int64_t)cf.max_positions * H);
  const float* type = take(2 * H);
  const float* eg = take(H);
  const float* eb = take(H);
  if ((rc = up_table(m, &m->word, word, (int64_t)cf.vocab_size * H, staging))) return rc;
  if (cf.position_type == 0 && (rc = up_table(m, &m->ptab, pos, (int64_t)cf.max_positions * H, staging))) return rc;
  if ((rc = up_table(m, &m->type0, type, H, staging))) return rc;  // token type 0 only (bert.go:242-245)
  if ((rc = up_f32(m, &m->eln_g, eg, H))) return rc;
  if ((rc = up_f32(m, &m->eln_b, eb, H))) return rc;

  std::vector<float> cat((size_t)(H * 3 * H));
  std::vector<float> bcat((size_t)(3 * H));
  std::vector<float> bip((size_t)Iup);
  m->layers.assign(cf.num_layers, Layer());
  for (int l = 0; l < cf.num_layers; l++) {
    Layer& L = m->layers[l];
    const float* wq = take(H * H); const float* bq = take(H);
    const float* wk = take(H * H); const float* bk = take(H);
    const float* wv = take(H * H); const float* bv = take(H);
    const float* wo = take(H * H); const float* bo = take(H);
    const float* l1g = take(H);    const float* l1b = take(H);
    const float* wi = take(H * Iup); const float* bi = take(Iup);
    const float* wd = take(I * H);   const float* bd = take(H);
    const float* l2g = take(H);    const float* l2b = take(H);
    // [Wq | Wk | Wv] as one (in,out) [H, 3H] matrix: the three Linear calls of bert.go:614-616
    // become one GEMM with identical per-column dot products.
    for (int64_t k = 0; k < H; k++) {
      memcpy(&cat[k * 3 * H], wq + k * H, H * 4);
      memcpy(&cat[k * 3 * H + H], wk + k * H, H * 4);
      memcpy(&cat[k * 3 * H + 2 * H], wv + k * H, H * 4);
    }
    memcpy(&bcat[0], bq, H * 4);
    memcpy(&bcat[H], bk, H * 4);
    memcpy(&bcat[2 * H], bv, H * 4);
    if ((rc = up_weight(m, &L.wqkv, cat.data(), H, 3 * H, 0, 0, staging))) return rc;
    if (!all_zero(bcat.data(), 3 * H) && (rc = up_f32(m, &L.bqkv, bcat.data(), 3 * H))) return rc;
    if ((rc = up_weight(m, &L.wo, wo, H, H, 0, 0, staging))) return rc;
    if (!all_zero(bo, H) && (rc = up_f32(m, &L.bo, bo, H))) return rc;
    if ((rc = up_f32(m, &L.ln1g, l1g, H))) return rc;
    if ((rc = up_f32(m, &L.ln1b, l1b, H))) return rc;
    const bool swiglu = cf.activation == FLETCHER_ACT_SWIGLU;
    const bool interleave = swiglu && m->dtype != FLETCHER_F32;
    if ((rc = up_weight(m, &L.wi, wi, H, Iup, interleave ? 1 : 0, m->bn_up, staging))) return rc;
    if (!all_zero(bi, Iup)) {
      if (interleave) {  // same interleave as the weight rows
        const int64_t half = m->bn_up / 2;
        for (int64_t n = 0; n < Iup; n++) {
          const int64_t j = n / m->bn_up, r = n % m->bn_up;
          bip[n] = bi[r < half ? j * half + r : I + j * half + (r - half)];
        }
        if ((rc = up_f32(m, &L.bi, bip.data(), Iup))) return rc;
      } else if ((rc = up_f32(m, &L.bi, bi, Iup))) {
        return rc;
      }
    }
    if ((rc = up_weight(m, &L.wd, wd, I, H, 0, 0, staging))) return rc;
    if (!all_zero(bd, H) && (rc = up_f32(m, &L.bd, bd, H))) return rc;
    if ((rc = up_f32(m, &L.ln2g, l2g, H))) return rc;
    if ((rc = up_f32(m, &L.ln2b, l2b, H))) return rc;
  }
  const float* wp = take(H * H);
  const float* bp = take(H);
  if ((rc = up_f32(m, &m->wp, wp, H * H))) return rc;
  if ((rc = up_f32(m, &m->bp, bp, H))) return rc;
  if ((rc = ensure_rope(m, cf.max_positions))) return rc;
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  m->loaded = true;
  return FLETCHER_OK;
}

// ---- Cuda_Model_LoadTensor: one checkpoint tensor by its reference name, any dtype, placed
// straight into the model's device layout (no host fp32 copy of the model).

// Checkpoint tensor names in LoadFromSafeTensors order (weights/loader.go:257-293).
static const char* kLayerSuffix[16] = {
    "attention.self.query.weight", "attention.self.query.bias", "attention.self.key.weight",
    "attention.self.key.bias", "attention.self.value.weight", "attention.self.value.bias",
    "attention.output.dense.weight", "attention.output.dense.bias", "attention.output.LayerNorm.weight",
    "attention.output.LayerNorm.bias", "intermediate.dense.weight", "intermediate.dense.bias",
    "output.dense.weight", "output.dense.bias", "output.LayerNorm.weight", "output.LayerNorm.bias"};
static const char* kHeadNames[5] = {"embeddings.word_embeddings.weight", "embeddings.position_embeddings.weight",
                                     "embeddings.token_type_embeddings.weight", "embeddings.LayerNorm.weight",
                                     "embeddings.LayerNorm.bias"};

int64_t tensor_count(const FletcherBertConfig* c) { return 5 + 16ll * c->num_layers + 2; }

// name -> index in raw order (-1 if unknown).
static int64_t tensor_index(const FletcherBertConfig* cf, const char* name) {
  for (int i = 0; i < 5; i++)
    if (!strcmp(name, kHeadNames[i])) return i;
  if (!strcmp(name, "pooler.dense.weight")) return 5 + 16ll * cf->num_layers;
  if (!strcmp(name, "pooler.dense.bias")) return 5 + 16ll * cf->num_layers + 1;
  int layer = -1, used = 0;
  if (sscanf(name, "encoder.layer.%d.%n", &layer, &used) == 1 && used > 0 && layer >= 0 && layer < cf->num_layers)
    for (int j = 0; j < 16; j++)
      if (!strcmp(name + used, kLayerSuffix[j])) return 5 + 16ll * layer + j;
  return -1;
}

// Expected (rows, cols) of tensor `idx` as the raw order stores it ((in,out) for Linear weights;
// vectors as (1, n)), and whether it is a Linear weight (loader.go:231-234).
static void tensor_shape(const Model* m, int64_t idx, int64_t* rows, int64_t* cols, bool* linear) {
  const FletcherBertConfig& cf = m->cfg;
  const int64_t H = m->H, I = m->I, Iup = m->Iup;
  *linear = false;
  if (idx < 5) {
    const int64_t r[5] = {cf.vocab_size, cf.max_positions, 2, 1, 1};
    *rows = r[idx];
    *cols = H;
    return;
  }
  const int64_t L = cf.num_layers;
  if (idx >= 5 + 16 * L) {
    *linear = idx == 5 + 16 * L;
    *rows = *linear ? H : 1;
    *cols = H;
    return;
  }
  const int j = (int)((idx - 5) % 16);
  const int64_t shapes[16][2] = {{H, H}, {1, H}, {H, H}, {1, H}, {H, H}, {1, H}, {H, H}, {1, H}, {1, H}, {1, H},
                                 {H, Iup}, {1, Iup}, {I, H}, {1, H}, {1, H}, {1, H}};
  *rows = shapes[j][0];
  *cols = shapes[j][1];
  *linear = j == 0 || j == 2 || j == 4 || j == 6 || j == 10 || j == 12;
}

static bool host_all_zero(const void* p, int32_t dt, int64_t n) {
  const int64_t bytes = n * dtype_size(dt);
  const uint8_t* b = (const uint8_t*)p;
  for (int64_t i = 0; i < bytes; i++)  // +0 only; a -0 bias is kept (it is a no-op either way)
    if (b[i]) return false;
  return true;
}

// A vector (bias, LayerNorm parameter) into an fp32 device array, allocated on first use.
static int32_t place_vec_f32(Model* m, float** d, int64_t total, int64_t off, const void* src_dev, int32_t sdt,
                             int64_t n) {
  int32_t rc;
  if (!*d && (rc = own(m, (void**)d, total * 4))) return rc;
  return launch_cast(m->c, sdt, src_dev, FLETCHER_F32, *d + off, n);
}

static int32_t load_tensor(Model* m, const char* name, int32_t sdt, const void* data, int64_t rows, int64_t cols,
                           int32_t transposed) {
  Ctx* c = m->c;
  const FletcherBertConfig& cf = m->cfg;
  FL_CHECK(c, name && data, "LoadTensor: null argument");
  FL_CHECK(c, sdt >= 0 && sdt <= 2, "LoadTensor %s: bad dtype %d", name, sdt);
  const int64_t idx = tensor_index(&cf, name);
  FL_CHECK(c, idx >= 0, "LoadTensor: tensor %s is not part of this model", name);  // loader.go:187-190
  int64_t er = 0, ec = 0;
  bool linear = false;
  tensor_shape(m, idx, &er, &ec, &linear);
  FL_CHECK(c, rows * cols == er * ec, "LoadTensor %s: size mismatch: expected %lld, got %lldx%lld", name,
           (long long)(er * ec), (long long)rows, (long long)cols);  // loader.go:200-202
  FL_CHECK(c, !transposed || linear, "LoadTensor %s: only Linear weights may be given transposed", name);
  if (linear)
    FL_CHECK(c, transposed ? (rows == ec && cols == er) : (rows == er && cols == ec),
             "LoadTensor %s: shape mismatch: got (%lld, %lld), expected %s (%lld, %lld)", name, (long long)rows,
             (long long)cols, transposed ? "(out, in)" : "(in, out)", (long long)(transposed ? ec : er),
             (long long)(transposed ? er : ec));
  const int64_t n = er * ec;
  const bool zero = !linear && er == 1 && host_all_zero(data, sdt, n);
  const int64_t H = m->H, L = cf.num_layers;
  if ((int64_t)m->layers.size() != L) m->layers.assign(L, Layer());
  if ((int64_t)m->tensor_loaded.size() != tensor_count(&cf)) m->tensor_loaded.assign(tensor_count(&cf), 0);
  clear_graphs(m);  // captured graphs may hold a pointer this load allocates
  m->loaded = false;

  // Stage the host tensor on the device as it is (sdt, given layout).
  void* stage = nullptr;
  int32_t rc = dev_alloc(c, &stage, n * dtype_size(sdt));
  if (rc) return rc;
  struct StageFree {
    Ctx* c;
    void* p;
    int64_t b;
    ~StageFree() { dev_free(c, p, b); }
  } sf{c, stage, n * dtype_size(sdt)};
  FL_CUDA(c, cudaMemcpyAsync(stage, data, n * dtype_size(sdt), cudaMemcpyHostToDevice, c->stream));

  const bool sixteen = m->dtype != FLETCHER_F32;
  const bool hf = sdt == FLETCHER_F32 && c->half_mode == FLETCHER_HALF_REFERENCE;
  auto table = [&](void** d, int64_t elems) -> int32_t {  // model-dtype table, first `elems` values
    int32_t r;
    if (!*d && (r = own(m, d, elems * dtype_size(m->dtype)))) return r;
    return launch_cast(c, sdt, stage, m->dtype, *d, elems, hf);
  };
  // Linear weight of (in,out) [K, N] into `d` (allocated [Ntot, K] K-major for 16-bit models,
  // or (in,out) [K, Ntot] for fp32) at output offset `off`.
  auto weight = [&](void** d, int64_t K, int64_t N, int64_t Ntot, int64_t off, int perm, int bn) -> int32_t {
    int32_t r;
    if (!*d && (r = own(m, d, K * Ntot * dtype_size(m->dtype)))) return r;
    return launch_place_weight(c, sdt, stage, K, N, transposed, m->dtype, *d, sixteen ? 1 : 0, Ntot, off, perm, bn);
  };
  auto bias = [&](float** d, int64_t total, int64_t off, int64_t len) -> int32_t {
    if (zero) {  // an all-zero bias adds nothing; keep it absent (or clear a loaded one)
      if (*d) FL_CUDA(c, cudaMemsetAsync(*d + off, 0, len * 4, c->stream));
      return FLETCHER_OK;
    }
    return place_vec_f32(m, d, total, off, stage, sdt, len);
  };

  if (idx == 0) {
    rc = table(&m->word, (int64_t)cf.vocab_size * H);
  } else if (idx == 1) {
    rc = cf.position_type == 0 ? table(&m->ptab, (int64_t)cf.max_positions * H) : FLETCHER_OK;  // RoPE: unused
  } else if (idx == 2) {
    rc = table(&m->type0, H);  // token type 0 only (bert.go:242-245)
  } else if (idx == 3 || idx == 4) {
    rc = place_vec_f32(m, idx == 3 ? &m->eln_g : &m->eln_b, H, 0, stage, sdt, H);
  } else if (idx >= 5 + 16 * L) {
    if (idx == 5 + 16 * L) {  // the pooler stays fp32 (in,out) in every mode (bert.go:459-477)
      if (!m->wp && (rc = own(m, (void**)&m->wp, H * H * 4))) return rc;
      rc = launch_place_weight(c, sdt, stage, H, H, transposed, FLETCHER_F32, m->wp, 0, H, 0, 0, 0);
    } else {
      rc = place_vec_f32(m, &m->bp, H, 0, stage, sdt, H);
    }
  } else {
    Layer& Ly = m->layers[(idx - 5) / 16];
    const int j = (int)((idx - 5) % 16);
    const bool swiglu = cf.activation == FLETCHER_ACT_SWIGLU;
    const int perm = swiglu && sixteen ? 1 : 0;
    switch (j) {
      case 0: case 2: case 4: rc = weight(&Ly.wqkv, H, H, 3 * H, (j / 2) * H, 0, 0); break;
      case 1: case 3: case 5: rc = bias(&Ly.bqkv, 3 * H, (j / 2) * H, H); break;
      case 6: rc = weight(&Ly.wo, H, H, H, 0, 0, 0); break;
      case 7: rc = bias(&Ly.bo, H, 0, H); break;
      case 8: rc = place_vec_f32(m, &Ly.ln1g, H, 0, stage, sdt, H); break;
      case 9: rc = place_vec_f32(m, &Ly.ln1b, H, 0, stage, sdt, H); break;
      case 10: rc = weight(&Ly.wi, H, m->Iup, m->Iup, 0, perm, m->bn_up); break;
      case 11:
        if (perm && !zero) {  // interleave like the weight rows: place the [1, Iup] row as K = 1
          if (!Ly.bi && (rc = own(m, (void**)&Ly.bi, m->Iup * 4))) return rc;
          rc = launch_place_weight(c, sdt, stage, 1, m->Iup, 0, FLETCHER_F32, Ly.bi, 1, 0, 0, perm, m->bn_up);
        } else {
          rc = bias(&Ly.bi, m->Iup, 0, m->Iup);
        }
        break;
      case 12: rc = weight(&Ly.wd, m->I, H, H, 0, 0, 0); break;
      case 13: rc = bias(&Ly.bd, H, 0, H); break;
      case 14: rc = place_vec_f32(m, &Ly.ln2g, H, 0, stage, sdt, H); break;
      default: rc = place_vec_f32(m, &Ly.ln2b, H, 0, stage, sdt, H); break;
    }
  }
  if (rc) return rc;
  FL_CUDA(c, cudaStreamSynchronize(c->stream));  // the caller may free `data` on return
  m->tensor_loaded[idx] = 1;
  bool all = true;
  for (uint8_t v : m->tensor_loaded) all = all && v;
  if (all) {
    if ((rc = ensure_rope(m, cf.max_positions))) return rc;
    m->loaded = true;
  }
  return FLETCHER_OK;
}

// Per-batch metadata -> device: cu_seqlens [B+1] and the attention tile list, through one
// pinned staging buffer and one copy.
static int32_t upload_meta(Model* m, const int32_t* lengths, int32_t B, int64_t T, int32_t* n_tiles, int32_t* max_len) {
  Ctx* c = m->c;
  std::vector<int32_t> order(B);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return lengths[a] > lengths[b]; });
  int64_t nt = 0;
  int32_t mx = 0;
  for (int i = 0; i < B; i++) {
    nt += (lengths[i] + kAttnTileRows - 1) / kAttnTileRows;
    mx = std::max(mx, lengths[i]);
  }
  FL_CHECK(c, nt <= m->tiles_cap, "internal: tile list overflow");
  FL_CHECK(c, mx <= kAttnMaxLen, "ForwardBatch: sequences are limited to %d tokens (got %d)", kAttnMaxLen, mx);
  const int64_t bytes = (int64_t)(B + 1) * 4 + nt * 8 + 16;
  if (bytes > m->h_meta_cap) {
    if (m->h_meta) {
      cudaEventSynchronize(m->meta_done);
      cudaFreeHost(m->h_meta);
    }
    const int64_t cap = std::max<int64_t>(bytes * 2, 1 << 16);
    FL_CUDA(c, cudaMallocHost((void**)&m->h_meta, cap));
    m->h_meta_cap = cap;
  } else {
    FL_CUDA(c, cudaEventSynchronize(m->meta_done));  // previous batch's copy has consumed it
  }
  int32_t* cu = reinterpret_cast<int32_t*>(m->h_meta);
  cu[0] = 0;
  for (int i = 0; i < B; i++) cu[i + 1] = cu[i] + lengths[i];
  const int64_t tiles_off = ((int64_t)(B + 1) * 4 + 15) / 16 * 16;
  int2* tl = reinterpret_cast<int2*>(m->h_meta + tiles_off);
  int64_t k = 0;
  for (int oi = 0; oi < B; oi++) {
    const int s = order[oi];
    for (int q0 = 0; q0 < lengths[s]; q0 += kAttnTileRows) tl[k++] = attn_tile(cu[s], lengths[s], q0);
  }
  FL_CUDA(c, cudaMemcpyAsync(m->d_cu, cu, (B + 1) * 4, cudaMemcpyHostToDevice, c->stream));
  if (nt) FL_CUDA(c, cudaMemcpyAsync(m->d_tiles, tl, nt * 8, cudaMemcpyHostToDevice, c->stream));
  FL_CUDA(c, cudaEventRecord(m->meta_done, c->stream));
  *n_tiles = (int32_t)nt;
  *max_len = mx;
  (void)T;
  return FLETCHER_OK;
}

// ---- optional per-stage timing with CUDA events on the context's stream
static cudaEvent_t next_event(Model* m) {
  if (m->ev_used == m->ev_pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    m->ev_pool.push_back(e);
  }
  return m->ev_pool[m->ev_used++];
}

static cudaEvent_t stage_begin(Model* m) {
  if (!m->timing) return nullptr;
  cudaEvent_t e = next_event(m);
  if (e) cudaEventRecord(e, m->c->stream);
  return e;
}

static int32_t stage_end(Model* m, int cat, cudaEvent_t e0) {
  if (!m->timing || !e0) return FLETCHER_OK;
  cudaEvent_t e1 = next_event(m);
  if (!e1) return set_error(m->c, FLETCHER_ERR_CUDA, "cudaEventCreate failed");
  FL_CUDA(m->c, cudaEventRecord(e1, m->c->stream));
  m->stage_recs.push_back({cat, e0, e1});
  return FLETCHER_OK;
}

static int32_t launch_or_replay(Model* m, const int32_t* d_ids, const int32_t* lengths, int32_t B, int32_t pooling,
                                float* d_out, int64_t T, int32_t n_tiles, int32_t max_len);

static int32_t forward_device(Model* m, const int32_t* d_ids, const int32_t* lengths, int32_t B, int32_t pooling,
                              float* d_out) {
  Ctx* c = m->c;
  FL_CHECK(c, m->loaded, "model weights are not loaded");
  FL_CHECK(c, B > 0 && lengths != nullptr, "ForwardBatch: empty batch");
  FL_CHECK(c, pooling == FLETCHER_POOL_CLS_TANH || pooling == FLETCHER_POOL_MEAN_L2, "unknown pooling %d", pooling);
  int64_t T = 0;
  for (int i = 0; i < B; i++) {
    FL_CHECK(c, lengths[i] >= 0, "negative length");
    T += lengths[i];
  }
  FL_CHECK(c, T > 0, "ForwardBatch: no tokens");
  if (pooling == FLETCHER_POOL_CLS_TANH) FL_CHECK(c, lengths[B - 1] > 0, "CLS pooling of an empty last sequence");
  int32_t rc = ensure_ws(m, T, B);
  if (rc) return rc;
  int32_t n_tiles = 0, max_len = 0;
  if ((rc = upload_meta(m, lengths, B, T, &n_tiles, &max_len))) return rc;
  if ((rc = ensure_rope(m, max_len))) return rc;
  if (m->dtype != FLETCHER_F32 && ln_pool_supported(m->dtype, m->H)) {
    const int64_t need = ln_pool_workspace_bytes(B, max_len, m->H);
    if (need > m->lnpool_bytes) {
      clear_graphs(m);  // captured graphs hold the old pointer
      if (m->lnpool) dev_free(c, m->lnpool, m->lnpool_bytes);
      m->lnpool = nullptr;
      m->lnpool_bytes = 0;
      const int64_t cap = std::max<int64_t>(need, 1 << 20);
      if ((rc = dev_alloc(c, (void**)&m->lnpool, cap))) return rc;
      m->lnpool_bytes = cap;
    }
  }
  m->last_T = T;
  c->splitk = m->splitk;  // this model's split-K workspace for its GEMM launches
  c->splitk_bytes = m->splitk_bytes;
  return launch_or_replay(m, d_ids, lengths, B, pooling, d_out, T, n_tiles, max_len);
}

// The kernel sequence of one forward pass (everything after the metadata upload).
static int32_t run_layers(Model* m, const int32_t* d_ids, int32_t B, int32_t pooling, float* d_out, int64_t T,
                          int32_t n_tiles, int32_t max_len) {
  Ctx* c = m->c;
  int32_t rc = 0;
  const int64_t H = m->H, I = m->I, Iup = m->Iup;
  const int32_t dt = m->dtype;
  const float eps = m->cfg.layer_norm_eps;
  const bool rope = m->cfg.position_type == 1;
  // Each stage is optionally bracketed by CUDA events on the context's stream
  // (Cuda_Model_SetStageTiming / Cuda_Model_StageTimes).
#define FL_STAGE(cat, call)                  \
  do {                                       \
    cudaEvent_t e0_ = stage_begin(m);        \
    if ((rc = (call))) return rc;            \
    if ((rc = stage_end(m, (cat), e0_))) return rc; \
  } while (0)
  FL_STAGE(FLETCHER_STAGE_EMBED, launch_positions(c, m->d_cu, B, m->d_pos, max_len));
  FL_STAGE(FLETCHER_STAGE_EMBED, launch_embed(c, dt, d_ids, m->d_pos, m->word, rope ? nullptr : m->ptab,
                                              m->cfg.max_positions, m->type0, m->eln_g, m->eln_b, m->X, T, H, eps));
  const int64_t es = dtype_size(dt);
  const float scale = 1.0f / (float)std::sqrt((double)m->dh);
  const bool swiglu = m->cfg.activation == FLETCHER_ACT_SWIGLU;
  // Mean pooling of a 16-bit model: the last LayerNorm is fused into the pool, so the final
  // normalised rows are never written (unless the caller keeps the last hidden state).
  const bool fuse_last = pooling == FLETCHER_POOL_MEAN_L2 && dt != FLETCHER_F32 && ln_pool_supported(dt, H) &&
                         !m->keep_hidden && m->lnpool && !m->layers.empty();
  m->last_fused = fuse_last;
  for (size_t li = 0; li < m->layers.size(); li++) {
    auto& L = m->layers[li];
    const bool last = li + 1 == m->layers.size();
    if (dt == FLETCHER_F32) {
      FL_STAGE(FLETCHER_STAGE_GEMM_QKV, launch_sgemm(c, (float*)m->X, H, (float*)L.wqkv, 3 * H, (float*)m->QKV, 3 * H, T,
                                                     3 * H, H, L.bqkv, FLETCHER_ACT_IDENTITY));
      if (rope)
        FL_STAGE(FLETCHER_STAGE_ROPE, launch_rope_table(c, dt, m->QKV, T, 3 * H, 2 * H, (int32_t)m->dh, m->d_pos,
                                                        m->cos_t, m->sin_t));
      float* qkv = (float*)m->QKV;
      FL_STAGE(FLETCHER_STAGE_ATTENTION, launch_attention_f32(c, qkv, qkv + H, qkv + 2 * H, 3 * H, (float*)m->CTX, H,
                                                              m->d_cu, B, T, (int32_t)m->nh, (int32_t)m->dh, scale,
                                                              max_len));
      FL_STAGE(FLETCHER_STAGE_GEMM_O, launch_sgemm(c, (float*)m->CTX, H, (float*)L.wo, H, (float*)m->S, H, T, H, H, L.bo,
                                                   FLETCHER_ACT_IDENTITY));
      FL_STAGE(FLETCHER_STAGE_LAYERNORM, launch_add_layernorm(c, dt, m->X, m->S, m->X, L.ln1g, L.ln1b, T, H, eps));
      FL_STAGE(FLETCHER_STAGE_GEMM_UP, launch_sgemm(c, (float*)m->X, H, (float*)L.wi, Iup, (float*)m->INTER, Iup, T, Iup,
                                                    H, L.bi, swiglu ? FLETCHER_ACT_IDENTITY : FLETCHER_ACT_GELU));
      const float* a_in = (float*)m->INTER;
      if (swiglu) {
        FL_STAGE(FLETCHER_STAGE_ACTIVATION, launch_swiglu(c, dt, m->INTER, m->ACT, T, I));
        a_in = (float*)m->ACT;
      }
      FL_STAGE(FLETCHER_STAGE_GEMM_DOWN, launch_sgemm(c, a_in, I, (float*)L.wd, H, (float*)m->S, H, T, H, I, L.bd,
                                                      FLETCHER_ACT_IDENTITY));
      FL_STAGE(FLETCHER_STAGE_LAYERNORM, launch_add_layernorm(c, dt, m->X, m->S, m->X, L.ln2g, L.ln2b, T, H, eps));
    } else {
      const bool fuse_rope = rope && m->dh == 64;
      FL_STAGE(FLETCHER_STAGE_GEMM_QKV,
               launch_gemm_tc(c, dt, fuse_rope ? EPI_ROPE : EPI_STORE, m->bn_qkv, m->X, T, H, L.wqkv, 3 * H, m->QKV,
                              3 * H, L.bqkv, nullptr, 0, m->d_pos, m->cos_t, m->sin_t, rope ? 2 * H : 0));
      if (rope && !fuse_rope)
        FL_STAGE(FLETCHER_STAGE_ROPE, launch_rope_table(c, dt, m->QKV, T, 3 * H, 2 * H, (int32_t)m->dh, m->d_pos,
                                                        m->cos_t, m->sin_t));
      const uint8_t* qkv = (const uint8_t*)m->QKV;
      FL_STAGE(FLETCHER_STAGE_ATTENTION,
               launch_flash_attention_tc(c, dt, qkv, qkv + H * es, qkv + 2 * H * es, 3 * H, T, H, m->CTX, H,
                                         m->d_cu, m->d_tiles, n_tiles, (int32_t)m->nh, scale));
      FL_STAGE(FLETCHER_STAGE_GEMM_O, launch_gemm_tc(c, dt, EPI_RESIDUAL, m->bn_o, m->CTX, T, H, L.wo, H, m->S, H, L.bo,
                                                     m->X, H, nullptr, nullptr, nullptr, 0));
      FL_STAGE(FLETCHER_STAGE_LAYERNORM, launch_add_layernorm(c, dt, m->S, nullptr, m->X, L.ln1g, L.ln1b, T, H, eps));
      FL_STAGE(FLETCHER_STAGE_GEMM_UP, launch_gemm_tc(c, dt, swiglu ? EPI_SWIGLU : EPI_GELU, m->bn_up, m->X, T, H, L.wi,
                                                      Iup, m->ACT, I, L.bi, nullptr, 0, nullptr, nullptr, nullptr, 0));
      FL_STAGE(FLETCHER_STAGE_GEMM_DOWN, launch_gemm_tc(c, dt, EPI_RESIDUAL, m->bn_d, m->ACT, T, I, L.wd, H, m->S, H,
                                                        L.bd, m->X, H, nullptr, nullptr, nullptr, 0));
      if (last && fuse_last) {
        FL_STAGE(FLETCHER_STAGE_POOL, launch_ln_mean_pool_l2(c, dt, m->S, m->d_cu, L.ln2g, L.ln2b, eps, B, max_len, H,
                                                             m->lnpool, d_out));
        return FLETCHER_OK;
      }
      FL_STAGE(FLETCHER_STAGE_LAYERNORM, launch_add_layernorm(c, dt, m->S, nullptr, m->X, L.ln2g, L.ln2b, T, H, eps));
    }
  }
  if (pooling == FLETCHER_POOL_MEAN_L2) {
    FL_STAGE(FLETCHER_STAGE_POOL, launch_mean_pool_l2(c, dt, m->X, m->d_cu, B, H, d_out));
    return FLETCHER_OK;
  }
  // BertPooler.ForwardBatch (bert.go:441-488): CLS rows at cu_seqlens[i] -> fp32 Dense -> TanhFast.
  FL_STAGE(FLETCHER_STAGE_POOL, launch_gather_rows_f32(c, dt, m->X, m->d_cu, B, H, m->d_cls));
  FL_STAGE(FLETCHER_STAGE_POOL, launch_sgemm(c, m->d_cls, H, m->wp, H, d_out, H, B, H, H, m->bp, FLETCHER_ACT_TANH));
#undef FL_STAGE
  return FLETCHER_OK;
}

// CUDA-graph replay of the kernel sequence for repeated batch shapes.  A shape (lengths,
// pooling, input/output pointers) seen for the first time runs eagerly; the second time it is
// captured; later calls replay the graph, which removes the per-kernel launch and tensor-map
// encoding cost on the host (what dominates single-request latency).  The metadata upload
// stays outside the graph, so replays read the freshly uploaded cu_seqlens / tile list.
void clear_graphs(Model* m) {
  for (auto& g : m->graphs) cudaGraphExecDestroy(g.exec);
  m->graphs.clear();
  m->graph_seen.clear();
}

static int32_t launch_or_replay(Model* m, const int32_t* d_ids, const int32_t* lengths, int32_t B, int32_t pooling,
                                float* d_out, int64_t T, int32_t n_tiles, int32_t max_len) {
  Ctx* c = m->c;
  if (!m->use_graphs || m->timing) return run_layers(m, d_ids, B, pooling, d_out, T, n_tiles, max_len);
  std::vector<int32_t> key;
  key.reserve(B + 6);
  const uint64_t pi = (uint64_t)(uintptr_t)d_ids, po = (uint64_t)(uintptr_t)d_out;
  key.insert(key.end(), {pooling, B, (int32_t)pi, (int32_t)(pi >> 32), (int32_t)po, (int32_t)(po >> 32)});
  key.insert(key.end(), lengths, lengths + B);
  ++m->graph_tick;
  for (auto& g : m->graphs)
    if (g.key == key) {
      g.last_use = m->graph_tick;
      FL_CUDA(c, cudaGraphLaunch(g.exec, c->stream));
      c->launches += g.kernels;
      return FLETCHER_OK;
    }
  bool seen = false;
  for (auto& k : m->graph_seen) seen |= k == key;
  if (!seen) {
    if (m->graph_seen.size() >= 64) m->graph_seen.erase(m->graph_seen.begin());
    m->graph_seen.push_back(key);
    return run_layers(m, d_ids, B, pooling, d_out, T, n_tiles, max_len);
  }
  const int64_t l0 = c->launches;
  FL_CUDA(c, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  int32_t rc = run_layers(m, d_ids, B, pooling, d_out, T, n_tiles, max_len);
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  cudaGraphExec_t exec = nullptr;
  if (e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
  if (graph) cudaGraphDestroy(graph);
  if (e != cudaSuccess) {  // capture unavailable here: keep running eagerly
    cudaGetLastError();
    m->use_graphs = false;
    c->launches = l0;
    return run_layers(m, d_ids, B, pooling, d_out, T, n_tiles, max_len);
  }
  const int64_t kernels = c->launches - l0;
  if (m->graphs.size() >= 16) {  // evict the least recently used
    auto lru = std::min_element(m->graphs.begin(), m->graphs.end(),
                                [](const Model::GraphEntry& a, const Model::GraphEntry& b) { return a.last_use < b.last_use; });
    cudaGraphExecDestroy(lru->exec);
    m->graphs.erase(lru);
  }
  m->graphs.push_back({key, exec, m->graph_tick, kernels});
  FL_CUDA(c, cudaGraphLaunch(exec, c->stream));
  return FLETCHER_OK;
}

static int32_t create(Ctx* c, const FletcherBertConfig* cfg, int32_t dtype, Model** out) {
  FL_CHECK(c, cfg && out, "Model_Create: null argument");
  FL_CHECK(c, dtype >= 0 && dtype <= 2, "Model_Create: bad dtype %d", dtype);
  FL_CHECK(c, cfg->hidden > 0 && cfg->num_heads > 0 && cfg->hidden % cfg->num_heads == 0, "bad hidden/heads");
  FL_CHECK(c, cfg->activation == FLETCHER_ACT_GELU || cfg->activation == FLETCHER_ACT_SWIGLU,
           "activation must be GELU or SwiGLU");
  FL_CHECK(c, cfg->vocab_size > 0 && cfg->max_positions > 0 && cfg->num_layers >= 0, "bad config");
  const int64_t dh = cfg->hidden / cfg->num_heads;
  if (dtype != FLETCHER_F32) {
    if (dh != 64 || cfg->hidden % 64 != 0 || cfg->intermediate % 128 != 0)
      return set_error(c, FLETCHER_ERR_UNSUPPORTED,
                       "16-bit model path needs head_dim 64, hidden %% 64 == 0, intermediate %% 128 == 0");
  }
  Model* m = new Model();
  m->c = c;
  m->cfg = *cfg;
  m->dtype = dtype;
  m->H = cfg->hidden;
  m->I = cfg->intermediate;
  m->Iup = cfg->activation == FLETCHER_ACT_SWIGLU ? 2 * m->I : m->I;
  m->nh = cfg->num_heads;
  m->dh = dh;
  // Tile widths: 256-wide tiles for the wide GEMMs, 128 where N is small.
  // (SwiGLU needs 256 so that a tile holds 128 gate and 128 up columns.)
  m->bn_qkv = (3 * m->H) % 256 == 0 && 3 * m->H >= 1024 ? 256 : 128;
  m->bn_o = m->H % 256 == 0 ? 256 : 128;
  m->bn_d = m->bn_o;
  m->bn_up = cfg->activation == FLETCHER_ACT_SWIGLU || (m->Iup % 256 == 0 && m->Iup >= 1024) ? 256 : 128;
  if (cudaEventCreateWithFlags(&m->meta_done, cudaEventDisableTiming) != cudaSuccess) {
    delete m;
    return set_error(c, FLETCHER_ERR_CUDA, "cudaEventCreate failed");
  }
  cudaEventRecord(m->meta_done, c->stream);
  *out = m;
  return FLETCHER_OK;
}

static void destroy(Model* m) {
  Ctx* c = m->c;
  cudaStreamSynchronize(c->stream);
  free_ws(m);
  for (auto& a : m->allocs) dev_free(c, a.first, a.second);
  if (m->cos_t) dev_free(c, m->cos_t, (int64_t)m->rope_len * (m->dh / 2) * 4);
  if (m->sin_t) dev_free(c, m->sin_t, (int64_t)m->rope_len * (m->dh / 2) * 4);
  if (m->lnpool) dev_free(c, m->lnpool, m->lnpool_bytes);
  cudaStreamSynchronize(c->stream);
  if (m->h_meta) cudaFreeHost(m->h_meta);
  if (m->meta_done) cudaEventDestroy(m->meta_done);
  for (cudaEvent_t e : m->ev_pool) cudaEventDestroy(e);
  for (cudaEvent_t e : m->async_ev)
    if (e) cudaEventDestroy(e);
  delete m;
}

}  // namespace fl

using namespace fl;

extern "C" {

int64_t Cuda_Model_WeightCount(const FletcherBertConfig* cfg) { return cfg ? weight_count(cfg) : -1; }

int32_t Cuda_Model_Create(CudaContextRef ctx, const FletcherBertConfig* cfg, int32_t dtype, CudaModelRef* out) {
  Ctx* c = reinterpret_cast<Ctx*>(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  Model* m = nullptr;
  int32_t rc = create(c, cfg, dtype, &m);
  if (rc == FLETCHER_OK) *out = m;
  return rc;
}

int32_t Cuda_Model_LoadRaw(CudaModelRef model, const float* blob, int64_t count) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m || !blob) return FLETCHER_ERR_INVALID;
  DeviceGuard g(m->c);
  return load_raw(m, blob, count);
}

int32_t Cuda_Model_LoadTensor(CudaModelRef model, const char* name, int32_t dtype, const void* data, int64_t rows,
                              int64_t cols, int32_t transposed) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m) return FLETCHER_ERR_INVALID;
  DeviceGuard g(m->c);
  return load_tensor(m, name, dtype, data, rows, cols, transposed);
}

int32_t Cuda_Model_TensorCount(const FletcherBertConfig* cfg) { return cfg ? (int32_t)tensor_count(cfg) : -1; }

int32_t Cuda_Model_TensorName(const FletcherBertConfig* cfg, int32_t index, char* buf, int32_t len) {
  if (!cfg || !buf || len <= 0 || index < 0 || index >= tensor_count(cfg)) return FLETCHER_ERR_INVALID;
  const int64_t L = cfg->num_layers;
  if (index < 5) snprintf(buf, len, "%s", kHeadNames[index]);
  else if (index == 5 + 16 * L) snprintf(buf, len, "pooler.dense.weight");
  else if (index == 5 + 16 * L + 1) snprintf(buf, len, "pooler.dense.bias");
  else snprintf(buf, len, "encoder.layer.%d.%s", (int)((index - 5) / 16), kLayerSuffix[(index - 5) % 16]);
  return FLETCHER_OK;
}

int32_t Cuda_Model_IsLoaded(CudaModelRef model) {
  Model* m = reinterpret_cast<Model*>(model);
  return m && m->loaded ? 1 : 0;
}

int32_t Cuda_Model_ForwardBatchDevice(CudaModelRef model, const int32_t* d_ids, const int32_t* lengths, int32_t B,
                                      int32_t pooling, float* d_out) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m) return FLETCHER_ERR_INVALID;
  DeviceGuard g(m->c);
  return forward_device(m, d_ids, lengths, B, pooling, d_out);
}

int32_t Cuda_Model_ForwardBatch(CudaModelRef model, const int32_t* ids, const int32_t* lengths, int32_t B,
                                int32_t pooling, float* out) {
  return Cuda_Model_ForwardBatchEx(model, ids, lengths, B, pooling, FLETCHER_F32, out);
}

int32_t Cuda_Model_ForwardBatchEx(CudaModelRef model, const int32_t* ids, const int32_t* lengths, int32_t B,
                                  int32_t pooling, int32_t out_dtype, void* out) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m || !ids || !lengths || !out) return FLETCHER_ERR_INVALID;
  Ctx* c = m->c;
  DeviceGuard g(c);
  FL_CHECK(c, out_dtype >= FLETCHER_F32 && out_dtype <= FLETCHER_BF16, "ForwardBatchEx: bad output dtype %d", out_dtype);
  FL_CHECK(c, B > 0, "ForwardBatch: empty batch");
  int64_t T = 0;
  for (int i = 0; i < B; i++) T += lengths[i] > 0 ? lengths[i] : 0;
  for (int64_t t = 0; t < T; t++)
    FL_CHECK(c, ids[t] >= 0 && ids[t] < m->cfg.vocab_size, "Gather index out of bounds: ids[%lld]=%d",
             (long long)t, ids[t]);
  int32_t rc = ensure_ws(m, T, B);
  if (rc) return rc;
  FL_CUDA(c, cudaMemcpyAsync(m->d_ids, ids, T * 4, cudaMemcpyHostToDevice, c->stream));
  if ((rc = forward_device(m, m->d_ids, lengths, B, pooling, m->d_out))) return rc;
  const int64_t n = (int64_t)B * m->H;
  if (out_dtype == FLETCHER_F32) {
    FL_CUDA(c, cudaMemcpyAsync(out, m->d_out, n * 4, cudaMemcpyDeviceToHost, c->stream));
  } else {  // cast on the device (fp16 with the context's conversion, bf16 RNE), copy half the bytes
    if ((rc = launch_cast(c, FLETCHER_F32, m->d_out, out_dtype, m->d_cls, n, c->half_mode == FLETCHER_HALF_REFERENCE)))
      return rc;
    FL_CUDA(c, cudaMemcpyAsync(out, m->d_cls, n * 2, cudaMemcpyDeviceToHost, c->stream));
  }
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  return check_device_flag(c);
}

// Waits for tickets up to `ticket` (slots are reused every kAsyncSlots tickets).
static int32_t wait_ticket(Model* m, int64_t ticket) {
  Ctx* c = m->c;
  FL_CHECK(c, ticket >= 1 && ticket <= m->async_issued, "Wait: unknown ticket %lld", (long long)ticket);
  if (ticket <= m->async_done) return FLETCHER_OK;
  FL_CUDA(c, cudaEventSynchronize(m->async_ev[(ticket - 1) % Model::kAsyncSlots]));
  m->async_done = ticket;
  return check_device_flag(c);
}

int32_t Cuda_Model_ForwardBatchAsync(CudaModelRef model, const int32_t* ids, const int32_t* lengths, int32_t B,
                                     int32_t pooling, int32_t out_dtype, void* out, int64_t* ticket) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m || !ids || !lengths || !out || !ticket) return FLETCHER_ERR_INVALID;
  Ctx* c = m->c;
  DeviceGuard g(c);
  FL_CHECK(c, out_dtype >= FLETCHER_F32 && out_dtype <= FLETCHER_BF16, "ForwardBatchAsync: bad output dtype %d",
           out_dtype);
  FL_CHECK(c, B > 0, "ForwardBatch: empty batch");
  int32_t rc;
  // A free slot: the ticket issued kAsyncSlots ago must be complete.
  if (m->async_issued - m->async_done >= Model::kAsyncSlots &&
      (rc = wait_ticket(m, m->async_issued - Model::kAsyncSlots + 1)))
    return rc;
  int64_t T = 0;
  for (int i = 0; i < B; i++) T += lengths[i] > 0 ? lengths[i] : 0;
  for (int64_t t = 0; t < T; t++)
    FL_CHECK(c, ids[t] >= 0 && ids[t] < m->cfg.vocab_size, "Gather index out of bounds: ids[%lld]=%d",
             (long long)t, ids[t]);
  // A larger batch reallocates the workspace and drops the captured graphs: let the batches in
  // flight finish first.
  if ((T > m->ws_T || B > m->ws_B) && m->async_issued > m->async_done && (rc = wait_ticket(m, m->async_issued)))
    return rc;
  if ((rc = ensure_ws(m, T, B))) return rc;
  FL_CUDA(c, cudaMemcpyAsync(m->d_ids, ids, T * 4, cudaMemcpyHostToDevice, c->stream));
  if ((rc = forward_device(m, m->d_ids, lengths, B, pooling, m->d_out))) return rc;
  const int64_t n = (int64_t)B * m->H;
  if (out_dtype == FLETCHER_F32) {
    FL_CUDA(c, cudaMemcpyAsync(out, m->d_out, n * 4, cudaMemcpyDeviceToHost, c->stream));
  } else {
    if ((rc = launch_cast(c, FLETCHER_F32, m->d_out, out_dtype, m->d_cls, n, c->half_mode == FLETCHER_HALF_REFERENCE)))
      return rc;
    FL_CUDA(c, cudaMemcpyAsync(out, m->d_cls, n * 2, cudaMemcpyDeviceToHost, c->stream));
  }
  const int slot = (int)(m->async_issued % Model::kAsyncSlots);
  if (!m->async_ev[slot]) FL_CUDA(c, cudaEventCreateWithFlags(&m->async_ev[slot], cudaEventDisableTiming));
  FL_CUDA(c, cudaEventRecord(m->async_ev[slot], c->stream));
  *ticket = ++m->async_issued;
  return FLETCHER_OK;
}

int32_t Cuda_Model_Wait(CudaModelRef model, int64_t ticket) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m) return FLETCHER_ERR_INVALID;
  DeviceGuard g(m->c);
  return wait_ticket(m, ticket);
}

int32_t Cuda_Model_LastHidden(CudaModelRef model, float* host_out, int64_t count) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m || !host_out) return FLETCHER_ERR_INVALID;
  Ctx* c = m->c;
  DeviceGuard g(c);
  FL_CHECK(c, count <= m->last_T * m->H, "LastHidden: count exceeds the last batch");
  FL_CHECK(c, !m->last_fused,
           "LastHidden: the previous mean-pooled forward fused its final LayerNorm into the pool and did not store "
           "the hidden state (enable Cuda_Model_SetKeepHidden first)");
  float* tmp = nullptr;
  int32_t rc = dev_alloc(c, (void**)&tmp, count * 4);
  if (rc) return rc;
  rc = convert_to_f32(c, m->X, m->dtype, tmp, count);
  if (rc == FLETCHER_OK) {
    cudaMemcpyAsync(host_out, tmp, count * 4, cudaMemcpyDeviceToHost, c->stream);
    cudaStreamSynchronize(c->stream);
  }
  dev_free(c, tmp, count * 4);
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  return rc;
}

int32_t Cuda_Model_SetKeepHidden(CudaModelRef model, int32_t enable) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m) return FLETCHER_ERR_INVALID;
  DeviceGuard g(m->c);
  FL_CUDA(m->c, cudaStreamSynchronize(m->c->stream));
  m->keep_hidden = enable != 0;
  clear_graphs(m);  // the kernel sequence changes
  return FLETCHER_OK;
}

int32_t Cuda_Model_SetGraphs(CudaModelRef model, int32_t enable) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m) return FLETCHER_ERR_INVALID;
  DeviceGuard g(m->c);
  FL_CUDA(m->c, cudaStreamSynchronize(m->c->stream));
  m->use_graphs = enable != 0;
  clear_graphs(m);
  return FLETCHER_OK;
}

int32_t Cuda_Model_SetStageTiming(CudaModelRef model, int32_t enable) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m) return FLETCHER_ERR_INVALID;
  DeviceGuard g(m->c);
  FL_CUDA(m->c, cudaStreamSynchronize(m->c->stream));
  m->timing = enable != 0;
  m->stage_recs.clear();
  m->ev_used = 0;
  return FLETCHER_OK;
}

int32_t Cuda_Model_StageTimes(CudaModelRef model, float* ms, int64_t* launches, int32_t n) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m || !ms || n <= 0) return FLETCHER_ERR_INVALID;
  DeviceGuard g(m->c);
  FL_CUDA(m->c, cudaStreamSynchronize(m->c->stream));
  for (int i = 0; i < n; i++) {
    ms[i] = 0.f;
    if (launches) launches[i] = 0;
  }
  for (auto& r : m->stage_recs) {
    if (r.cat >= n) continue;
    float t = 0.f;
    FL_CUDA(m->c, cudaEventElapsedTime(&t, r.a, r.b));
    ms[r.cat] += t;
    if (launches) launches[r.cat]++;
  }
  m->stage_recs.clear();
  m->ev_used = 0;
  return FLETCHER_OK;
}

}  // extern "C"

// The host runtime (runtime.cu) reads a model's width and context through these.
int64_t model_hidden(CudaModelRef model) { return model ? reinterpret_cast<Model*>(model)->H : 0; }
CudaContextRef model_context(CudaModelRef model) { return model ? reinterpret_cast<Model*>(model)->c : nullptr; }

extern "C" {

int32_t Cuda_Model_Free(CudaModelRef model) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m) return FLETCHER_OK;
  DeviceGuard g(m->c);
  destroy(m);
  return FLETCHER_OK;
}

}  // extern "C"
