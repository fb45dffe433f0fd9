// TEST INFRASTRUCTURE ONLY — the CPU oracle for the embedding forward pass.
//
// This file restates, in C++, the reference's fp32 CPU path for
// BertModel.ForwardBatch (internal/embeddings/model/bert.go:149-169) as it runs
// on the CPU backend (internal/device/cpu_backend.go) with the fast-math
// helpers of internal/simd/simd.go.  It is used only by the tests, by
// __graft_entry__.smoke() as a checker, and by bench.py's CPU-baseline leg.
// Nothing in the product (the CUDA library) links or calls it.
//
// Parity pin: the reference's own Go code cannot be compiled here (no Go
// toolchain, modules not vendored), so this restatement is pinned against the
// reference's known-answer tests (device_test.go LayerNorm/Mul, simd_test.go
// fast-math bounds, cast_test.go fp16 bytes, rope_test.go formula) — see
// tests/test_oracle.py.
//
// Two modes:
//   MODE_LITERAL (0): the reference as written, including
//     - LayerNorm eps hard-coded to 1e-7 for every LayerNorm (bert.go:281),
//     - RoPE base 10000 (cpu_backend.go:790) and position = row % lengths[0]
//       (bert.go:619-624, cpu_backend.go:783),
//     - for batches whose lengths differ, a self-attention context of ZEROS:
//       the per-sequence fallback (bert.go:653-716) writes its result through
//       output.Slice(...).Copy(res), and CPUTensor.Slice returns a copy
//       (cpu_backend.go:288-303), so `output` keeps its zero initialisation.
//   MODE_SPEC (1): identical formulas, but eps / RoPE base from the config,
//     per-sequence RoPE positions and per-sequence multi-head attention for
//     every batch.  On uniform-length batches with eps=1e-7 and base=10000 the
//     two modes are bit-identical (tests check this).
//
// Both modes also emit the spec's mean-pool + L2 head (no reference code).
//
// GEMMs go through OpenBLAS sgemm (the reference's Mul -> blas32.Gemm ->
// cblas_sgemm, cpu_backend.go:350-372); the OpenBLAS used is the one numpy
// ships (ILP64 symbol names with the 64_ suffix), loaded with dlopen.
//
// Build: oracle/Makefile (-O2 -ffp-contract=off: Go on amd64 does not fuse
// multiply-adds, so neither may we).

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <dlfcn.h>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------- OpenBLAS
typedef void (*sgemm64_fn)(int order, int ta, int tb, int64_t m, int64_t n, int64_t k,
                           float alpha, const float* a, int64_t lda, const float* b,
                           int64_t ldb, float beta, float* c, int64_t ldc);
typedef void (*setthreads64_fn)(int);

sgemm64_fn g_sgemm = nullptr;
setthreads64_fn g_set_threads = nullptr;
int g_threads = 1;

constexpr int kRowMajor = 101, kNoTrans = 111, kTrans = 112;

void sgemm(bool ta, bool tb, int64_t m, int64_t n, int64_t k, float alpha, const float* a,
           int64_t lda, const float* b, int64_t ldb, float* c, int64_t ldc) {
  g_sgemm(kRowMajor, ta ? kTrans : kNoTrans, tb ? kTrans : kNoTrans, m, n, k, alpha, a, lda, b,
          ldb, 0.0f, c, ldc);
}

// ---------------------------------------------------------------- simd.go
// ExpFast, simd.go:7-46.  Every operation is a float32 operation, in the
// order Go evaluates it.
inline float exp_fast(float x) {
  if (x > 88.0f) return 1e38f;
  if (x < -88.0f) return 0.0f;
  const float log2e = 1.442695f;
  float t = x * log2e;
  int k = (int)t;  // Go int(t): truncation toward zero
  if (t < 0) k--;
  float f = t - (float)k;
  float p = 1.0f + f * (0.6931472f + f * (0.2402265f + f * 0.0555041f));
  return p * (float)std::pow(2.0, (double)k);
}

// TanhFast, simd.go:49-63 (Pade approximation, clamped beyond |x|>4).
inline float tanh_fast(float x) {
  if (x > 4.0f) return 1.0f;
  if (x < -4.0f) return -1.0f;
  float x2 = x * x;
  return x * (27.0f + x2) / (27.0f + 9.0f * x2);
}

// GeluFast, simd.go:66-75.
inline float gelu_fast(float x) {
  const float sqrt2overPi = 0.7978846f, coeff = 0.044715f;
  return 0.5f * x * (1.0f + tanh_fast(sqrt2overPi * (x + coeff * x * x * x)));
}

// SoftmaxFast, simd.go:78-99: max, ExpFast(v-max) with a sequential float32
// sum, then a multiply by 1/sum.
void softmax_fast(float* row, int64_t n) {
  float mx = row[0];
  for (int64_t i = 0; i < n; i++)
    if (row[i] > mx) mx = row[i];
  float sum = 0.0f;
  for (int64_t i = 0; i < n; i++) {
    row[i] = exp_fast(row[i] - mx);
    sum += row[i];
  }
  float inv = 1.0f / sum;
  for (int64_t i = 0; i < n; i++) row[i] *= inv;
}

// ---------------------------------------------------------------- cpu_backend.go
// CPUTensor.LayerNorm, cpu_backend.go:541-601 (two-pass, biased variance,
// invStd = 1/float32(sqrt(float64(var+eps)))).
void layer_norm_rows(float* x, int64_t rows, int64_t c, const float* g, const float* b, float eps) {
  for (int64_t i = 0; i < rows; i++) {
    float* row = x + i * c;
    float sum = 0.0f;
    for (int64_t j = 0; j < c; j++) sum += row[j];
    float mean = sum / (float)c;
    float var_sum = 0.0f;
    for (int64_t j = 0; j < c; j++) {
      float d = row[j] - mean;
      var_sum += d * d;
    }
    float variance = var_sum / (float)c;
    float inv_std = 1.0f / (float)std::sqrt((double)(variance + eps));
    for (int64_t j = 0; j < c; j++) row[j] = (row[j] - mean) * inv_std * g[j] + b[j];
  }
}

// AddBias (cpu_backend.go:448-488) = VecAdd of the bias into every row.
void add_bias(float* y, int64_t rows, int64_t c, const float* b) {
  for (int64_t i = 0; i < rows; i++)
    for (int64_t j = 0; j < c; j++) y[i * c + j] += b[j];
}

// Linear (cpu_backend.go:612-624): Y = X.W (W stored (in,out)), then AddBias.
void linear(const float* x, int64_t rows, int64_t k, const float* w, int64_t n, const float* b,
            float* y) {
  sgemm(false, false, rows, n, k, 1.0f, x, k, w, n, y, n);
  if (b) add_bias(y, rows, n, b);
}

// ApplyRoPE, cpu_backend.go:760-805: rotate-half with float64 trig.  `pos`
// gives the position of every row (literal mode passes row % lengths[0]).
void apply_rope(float* t, int64_t rows, int nh, int dh, const int32_t* pos, double base) {
  auto work = [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; r++) {
      int64_t row_off = r * (int64_t)nh * dh;
      for (int h = 0; h < nh; h++) {
        float* p = t + row_off + (int64_t)h * dh;
        for (int i = 0; i < dh / 2; i++) {
          double theta = (double)pos[r] * std::pow(base, -2.0 * (double)i / (double)dh);
          float c = (float)std::cos(theta), s = (float)std::sin(theta);
          float x1 = p[i], x2 = p[dh / 2 + i];
          p[i] = x1 * c - x2 * s;
          p[dh / 2 + i] = x1 * s + x2 * c;
        }
      }
    }
  };
  int nw = g_threads;
  int64_t per = (rows + nw - 1) / nw;
  std::vector<std::thread> ws;
  for (int w = 0; w < nw; w++) {
    int64_t a = w * per, b = a + per;
    if (a >= rows) break;
    if (b > rows) b = rows;
    ws.emplace_back(work, a, b);
  }
  for (auto& th : ws) th.join();
}

// CPUTensor.Attention (cpu_backend.go:662-758), generalised to packed
// sequences: per sequence, per head, scores = scale * Q_h K_h^T (sgemm with
// alpha=scale), SoftmaxFast per row, O_h = P V_h (sgemm, strided into the
// output).  Sequences are split into contiguous chunks over worker threads,
// like the reference's per-batch-chunk goroutines.
void attention(const float* q, const float* k, const float* v, float* out, int64_t c, int nh,
               const int64_t* starts, const int32_t* lens, int B, float scale) {
  int dh = (int)(c / nh);
  int workers = g_threads < B ? g_threads : B;
  if (workers < 1) workers = 1;
  int per = (B + workers - 1) / workers;
  auto work = [&](int b0, int b1) {
    int maxl = 0;
    for (int i = b0; i < b1; i++) maxl = lens[i] > maxl ? lens[i] : maxl;
    std::vector<float> scores((size_t)maxl * maxl);
    for (int i = b0; i < b1; i++) {
      int64_t l = lens[i];
      if (l == 0) continue;
      int64_t off = starts[i] * c;
      for (int h = 0; h < nh; h++) {
        int64_t ho = (int64_t)h * dh;
        sgemm(false, true, l, l, dh, scale, q + off + ho, c, k + off + ho, c, scores.data(), l);
        for (int64_t r = 0; r < l; r++) softmax_fast(scores.data() + r * l, l);
        sgemm(false, false, l, dh, l, 1.0f, scores.data(), l, v + off + ho, c, out + off + ho, c);
      }
    }
  };
  std::vector<std::thread> ws;
  for (int w = 0; w < workers; w++) {
    int a = w * per, b = a + per;
    if (a >= B) break;
    if (b > B) b = B;
    ws.emplace_back(work, a, b);
  }
  for (auto& th : ws) th.join();
}

struct Cfg {
  int32_t vocab_size, hidden, num_layers, num_heads, intermediate, max_positions;
  int32_t activation;     // device.ActivationType: 1 = GELU, 4 = SwiGLU
  int32_t position_type;  // 0 = absolute, 1 = RoPE
  float layer_norm_eps;
  float rope_base;
};

}  // namespace

extern "C" {

// Must match FletcherBertConfig in include/fletcher_cuda.h (same field order).
typedef Cfg RefConfig;

int ref_init(const char* openblas_path, int nthreads) {
  if (!g_sgemm) {
    void* h = dlopen(openblas_path, RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      fprintf(stderr, "ref_init: dlopen(%s) failed: %s\n", openblas_path, dlerror());
      return -1;
    }
    g_sgemm = (sgemm64_fn)dlsym(h, "scipy_cblas_sgemm64_");
    g_set_threads = (setthreads64_fn)dlsym(h, "scipy_openblas_set_num_threads64_");
    if (!g_sgemm) return -2;
  }
  g_threads = nthreads > 0 ? nthreads : 1;
  if (g_set_threads) g_set_threads(g_threads);
  return 0;
}

// Number of fp32 values in the raw weight blob, in the order of
// LoadFromRawBinary (internal/embeddings/weights/loader.go:29-90).
int64_t ref_weight_count(const RefConfig* c) {
  int64_t H = c->hidden, I = c->intermediate;
  int64_t Iup = c->activation == 4 ? 2 * I : I;
  int64_t n = (int64_t)c->vocab_size * H + (int64_t)c->max_positions * H + 2 * H + 2 * H;
  int64_t per_layer = 3 * (H * H + H) + (H * H + H) + 2 * H + (H * Iup + Iup) + (I * H + H) + 2 * H;
  n += per_layer * c->num_layers;
  n += H * H + H;
  return n;
}

// Scalar fast-math entry points (for the known-answer tests).
float ref_exp_fast(float x) { return exp_fast(x); }
float ref_tanh_fast(float x) { return tanh_fast(x); }
float ref_gelu_fast(float x) { return gelu_fast(x); }
void ref_softmax_fast(float* row, int64_t n) { softmax_fast(row, n); }
void ref_layer_norm(float* x, int64_t rows, int64_t cols, const float* g, const float* b, float eps) {
  layer_norm_rows(x, rows, cols, g, b, eps);
}
void ref_sgemm(int ta, int tb, int64_t m, int64_t n, int64_t k, float alpha, const float* a,
               int64_t lda, const float* b, int64_t ldb, float* c, int64_t ldc) {
  sgemm(ta != 0, tb != 0, m, n, k, alpha, a, lda, b, ldb, c, ldc);
}
// LinearActivation (cpu_backend.go:626-660): y = act(x . w + b); for SwiGLU (act 4) y has n/2
// columns, silu(first half) * second half with float64 exp; GELU (1) / Tanh (2) the fast forms.
void ref_linear_activation(const float* x, int64_t rows, int64_t k, const float* w, int64_t n, const float* b,
                           int act, float* y) {
  std::vector<float> full((size_t)(rows * n));
  linear(x, rows, k, w, n, b, full.data());
  if (act == 4) {
    const int64_t I = n / 2;
    for (int64_t r = 0; r < rows; r++)
      for (int64_t i = 0; i < I; i++) {
        float xx = full[r * n + i], yy = full[r * n + i + I];
        float sw = xx / (1.0f + (float)std::exp((double)(-xx)));
        y[r * I + i] = sw * yy;
      }
    return;
  }
  for (int64_t i = 0; i < rows * n; i++)
    y[i] = act == 1 ? gelu_fast(full[i]) : act == 2 ? tanh_fast(full[i]) : full[i];
}

// CPUTensor.Attention over packed sequences of the given lengths (cpu_backend.go:662-758).
void ref_attention(const float* q, const float* k, const float* v, float* out, int64_t c, int nh,
                   const int32_t* lens, int B, float scale) {
  std::vector<int64_t> starts(B);
  int64_t t = 0;
  for (int i = 0; i < B; i++) {
    starts[i] = t;
    t += lens[i];
  }
  attention(q, k, v, out, c, nh, starts.data(), lens, B, scale);
}

void ref_rope(float* t, int64_t rows, int nh, int dh, const int32_t* pos, double base) {
  apply_rope(t, rows, nh, dh, pos, base);
}

// The full forward pass.  ids: packed [T] int32 (each sequence already framed
// by [CLS] ... [SEP]); lengths: [B].  Outputs (any may be null):
//   out_cls    [B,H] — the reference's pooler output (CLS -> Dense -> TanhFast)
//   out_mean   [B,H] — mean over each sequence's rows, then L2-normalised
//   out_hidden [T,H] — last hidden state
int ref_forward(const RefConfig* cfg, const float* w, int64_t nweights, const int32_t* ids,
                const int32_t* lengths, int32_t B, int32_t mode, float* out_cls, float* out_mean,
                float* out_hidden) {
  if (!g_sgemm) return -1;
  if (nweights != ref_weight_count(cfg)) return -2;
  const bool literal = mode == 0;
  const int64_t H = cfg->hidden, I = cfg->intermediate, nh = cfg->num_heads, dh = H / nh;
  const int64_t Iup = cfg->activation == 4 ? 2 * I : I;
  const float eps = literal ? 1e-7f : cfg->layer_norm_eps;
  const double base = literal ? 10000.0 : (double)cfg->rope_base;
  std::vector<int64_t> starts(B);
  int64_t T = 0;
  for (int i = 0; i < B; i++) {
    starts[i] = T;
    T += lengths[i];
  }
  for (int64_t t = 0; t < T; t++)
    if (ids[t] < 0 || ids[t] >= cfg->vocab_size) return -3;  // Gather: index out of bounds

  // ---- weight views in raw order (loader.go:29-90)
  const float* p = w;
  auto take = [&](int64_t n) { const float* r = p; p += n; return r; };
  const float* word = take((int64_t)cfg->vocab_size * H);
  const float* posw = take((int64_t)cfg->max_positions * H);
  const float* typew = take(2 * H);
  const float* eln_g = take(H);
  const float* eln_b = take(H);

  // ---- BertEmbeddings.ForwardBatch (bert.go:215-261)
  std::vector<float> x((size_t)(T * H));
  for (int64_t t = 0; t < T; t++) memcpy(&x[t * H], word + (int64_t)ids[t] * H, H * 4);
  if (cfg->position_type == 0) {
    int64_t idx = 0;
    for (int i = 0; i < B; i++)
      for (int j = 0; j < lengths[i]; j++, idx++) {
        int pi = j >= cfg->max_positions ? cfg->max_positions - 1 : j;
        for (int64_t c = 0; c < H; c++) x[idx * H + c] += posw[(int64_t)pi * H + c];
      }
  }
  for (int64_t t = 0; t < T; t++)
    for (int64_t c = 0; c < H; c++) x[t * H + c] += typew[c];  // token type 0
  layer_norm_rows(x.data(), T, H, eln_g, eln_b, eps);

  bool uniform = true;
  for (int i = 0; i < B; i++) uniform &= lengths[i] == lengths[0];

  std::vector<int32_t> pos(T);
  {
    int64_t idx = 0;
    for (int i = 0; i < B; i++)
      for (int j = 0; j < lengths[i]; j++, idx++)
        pos[idx] = literal ? (int32_t)(idx % lengths[0]) : j;
  }

  // The reference rotates batchSize*lengths[0] rows (cpu_backend.go:765); when
  // that exceeds the packed row count its goroutines index past the slice and
  // the Go runtime panics.  Literal mode reports that case as error -4.
  int64_t rope_rows = T;
  if (literal && cfg->position_type == 1 && B > 0) {
    rope_rows = (int64_t)B * lengths[0];
    if (rope_rows > T) return -4;
  }

  std::vector<float> q(T * H), k(T * H), v(T * H), ctx(T * H), proj(T * H), inter(T * Iup),
      act(T * I);
  const float scale = 1.0f / (float)std::sqrt((double)dh);
  for (int l = 0; l < cfg->num_layers; l++) {
    const float* wq = take(H * H); const float* bq = take(H);
    const float* wk = take(H * H); const float* bk = take(H);
    const float* wv = take(H * H); const float* bv = take(H);
    const float* wo = take(H * H); const float* bo = take(H);
    const float* ln1g = take(H);   const float* ln1b = take(H);
    const float* wi = take(H * Iup); const float* bi = take(Iup);
    const float* wd = take(I * H);   const float* bd = take(H);
    const float* ln2g = take(H);   const float* ln2b = take(H);

    // BertSelfAttention.ForwardBatch (bert.go:610-728)
    linear(x.data(), T, H, wq, H, bq, q.data());
    linear(x.data(), T, H, wk, H, bk, k.data());
    linear(x.data(), T, H, wv, H, bv, v.data());
    if (cfg->position_type == 1) {
      apply_rope(q.data(), rope_rows, (int)nh, (int)dh, pos.data(), base);
      apply_rope(k.data(), rope_rows, (int)nh, (int)dh, pos.data(), base);
    }
    std::fill(ctx.begin(), ctx.end(), 0.0f);
    if (uniform || !literal)
      attention(q.data(), k.data(), v.data(), ctx.data(), H, (int)nh, starts.data(), lengths, B,
                scale);
    // (literal, non-uniform: ctx stays zero — see the header comment)

    // BertSelfOutput.Forward (bert.go:748-755): x = LN(x + (ctx.Wo + bo))
    linear(ctx.data(), T, H, wo, H, bo, proj.data());
    for (int64_t i = 0; i < T * H; i++) x[i] += proj[i];
    layer_norm_rows(x.data(), T, H, ln1g, ln1b, eps);

    // BertIntermediate.Forward (bert.go:781-787) -> LinearActivation
    // (cpu_backend.go:626-660)
    linear(x.data(), T, H, wi, Iup, bi, inter.data());
    const float* a_in;
    if (cfg->activation == 4) {
      for (int64_t t = 0; t < T; t++)
        for (int64_t i = 0; i < I; i++) {
          float xx = inter[t * Iup + i], yy = inter[t * Iup + i + I];
          float sw = xx / (1.0f + (float)std::exp((double)(-xx)));
          act[t * I + i] = sw * yy;
        }
      a_in = act.data();
    } else {
      for (int64_t i = 0; i < T * I; i++) inter[i] = gelu_fast(inter[i]);
      a_in = inter.data();
    }
    // BertOutput.Forward (bert.go:813-820)
    linear(a_in, T, I, wd, H, bd, proj.data());
    for (int64_t i = 0; i < T * H; i++) x[i] += proj[i];
    layer_norm_rows(x.data(), T, H, ln2g, ln2b, eps);
  }
  const float* wp = take(H * H);
  const float* bp = take(H);

  if (out_hidden) memcpy(out_hidden, x.data(), T * H * 4);
  // BertPooler.ForwardBatch (bert.go:441-488)
  if (out_cls) {
    std::vector<float> cls((size_t)B * H), y((size_t)B * H);
    for (int i = 0; i < B; i++) memcpy(&cls[i * H], &x[starts[i] * H], H * 4);
    linear(cls.data(), B, H, wp, H, bp, y.data());
    for (int64_t i = 0; i < B * H; i++) out_cls[i] = tanh_fast(y[i]);
  }
  // Mean pooling + L2 normalisation (spec extension; float64 accumulation).
  if (out_mean) {
    std::vector<double> acc(H);
    for (int i = 0; i < B; i++) {
      std::fill(acc.begin(), acc.end(), 0.0);
      for (int64_t t = starts[i]; t < starts[i] + lengths[i]; t++)
        for (int64_t c = 0; c < H; c++) acc[c] += x[t * H + c];
      double nrm = 0.0;
      for (int64_t c = 0; c < H; c++) {
        acc[c] /= (double)(lengths[i] > 0 ? lengths[i] : 1);
        nrm += acc[c] * acc[c];
      }
      nrm = std::sqrt(nrm);
      double inv = nrm > 0 ? 1.0 / nrm : 0.0;
      for (int64_t c = 0; c < H; c++) out_mean[(int64_t)i * H + c] = (float)(acc[c] * inv);
    }
  }
  return 0;
}

}  // extern "C"
