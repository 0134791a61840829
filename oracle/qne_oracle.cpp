// qne_oracle - CPU restatement of the reference decoder's arithmetic. TEST INFRASTRUCTURE ONLY:
// the parity tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg call it as the
// checker; the engine never links or calls it.
//
// Reference (arlinamid/qwen-native-engine, read at its `kernels` crate):
//   dequant_row        kernels/src/lib.rs:484-497      (int4 block-32 unpack, QMat layout)
//   f16_to_f32         kernels/src/lib.rs:473-482
//   gemv epilogues     kernels/src/shaders.rs:36-43, CPU form kernels/src/lib.rs:528-535
//   rmsnorm            kernels/src/shaders.rs:380-403
//   embed              kernels/src/shaders.rs:409-434
//   gdn                kernels/src/shaders.rs:445-520, CPU form kernels/src/lib.rs:590-622
//   attention          kernels/src/shaders.rs:531-633, CPU form kernels/src/lib.rs:647-674
//   argmax             kernels/src/shaders.rs:636-699 (here: lowest index among equal maxima,
//                      the host greedy rule of src/sampling.rs:86-94)
//   per-token graph    kernels/src/model.rs:220-269
// Deliberate differences, each switchable where the reference behaviour is wanted:
//   * weights may also be f16 or group-64 int4 with f16 zero points (benchmark configs);
//   * the KV cache may hold f16-rounded keys/values, the current token included (kv_f16 = 1);
//   * RoPE angles come from a double-precision table (rope_table) instead of f32 pow/sin/cos.
// All accumulation is f32; transcendental functions are the host libm's. Work is spread over a
// pool of host threads (ORACLE_THREADS, default: all cores).
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdlib>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#define API extern "C" __attribute__((visibility("default")))

namespace {

constexpr int kMaxCtx = 4096;
constexpr int kGdnProj = 8224, kAttnProj = 5120, kMixerOut = 2048;

// Persistent worker pool: parallel_for(n, f) runs f(i) for i in [0, n) on all workers.
class Pool {
 public:
  Pool() {
    int n = (int)std::thread::hardware_concurrency();
    if (const char* e = getenv("ORACLE_THREADS")) n = atoi(e);
    if (n < 1) n = 1;
    nthreads_ = n;
    for (int i = 1; i < n; ++i) workers_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> l(mu_);
      stop_ = true;
      ++gen_;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int threads() const { return nthreads_; }
  void run(long n, const std::function<void(long)>& f) {
    if (n <= 0) return;
    if (nthreads_ == 1 || n == 1) {
      for (long i = 0; i < n; ++i) f(i);
      return;
    }
    std::unique_lock<std::mutex> l(mu_);
    fn_ = &f;
    total_ = n;
    next_.store(0);
    busy_ = (int)workers_.size();
    ++gen_;
    l.unlock();
    cv_.notify_all();
    work();
    l.lock();
    done_cv_.wait(l, [this] { return busy_ == 0; });
    fn_ = nullptr;
  }

 private:
  void work() {
    const long chunk = total_ / (8 * nthreads_) + 1;
    for (;;) {
      const long i0 = next_.fetch_add(chunk);
      if (i0 >= total_) break;
      const long i1 = i0 + chunk < total_ ? i0 + chunk : total_;
      for (long i = i0; i < i1; ++i) (*fn_)(i);
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> l(mu_);
      cv_.wait(l, [&] { return gen_ != seen; });
      seen = gen_;
      if (stop_) return;
      l.unlock();
      work();
      l.lock();
      if (--busy_ == 0) done_cv_.notify_all();
    }
  }
  int nthreads_ = 1;
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(long)>* fn_ = nullptr;
  long total_ = 0;
  std::atomic<long> next_{0};
  int busy_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

Pool& pool() {
  static Pool p;
  return p;
}

template <typename F>
void parallel_for(long n, F&& f) {
  std::function<void(long)> fn = f;
  pool().run(n, fn);
}

inline float h2f(uint16_t h) { return _cvtsh_ss(h); }
inline uint16_t f2h(float f) { return _cvtss_sh(f, _MM_FROUND_TO_NEAREST_INT); }
inline float silu(float x) { return x / (1.0f + expf(-x)); }

struct Mat {
  int kind;  // 0 f16, 1 q4 (block 32), 2 q4g64
  int rows, k;
  const void* w;
  const void* s;
  const void* z;
};

// Dequantized element (row, c), the arithmetic of dequant_row.
inline float deq(const Mat& m, long row, int c) {
  if (m.kind == 0) return h2f(((const uint16_t*)m.w)[row * m.k + c]);
  const uint32_t word = ((const uint32_t*)m.w)[row * (m.k / 8) + c / 8];
  const uint32_t q = (word >> (4 * (c % 8))) & 15u;
  float scale, zp;
  if (m.kind == 1) {
    const int blk = c / 32;
    const uint32_t sw = ((const uint32_t*)m.s)[row * (m.k / 64) + blk / 2];
    scale = h2f((uint16_t)(blk % 2 == 0 ? (sw & 0xFFFF) : (sw >> 16)));
    zp = (float)((((const uint32_t*)m.z)[row * (m.k / 256) + blk / 8] >> (4 * (blk % 8))) & 15u);
  } else {
    const int g = c / 64;
    scale = h2f(((const uint16_t*)m.s)[row * (m.k / 64) + g]);
    zp = h2f(((const uint16_t*)m.z)[row * (m.k / 64) + g]);
  }
  return ((float)q - zp) * scale;
}

// sum_c deq(row, c) * x[c] in f32 (16 interleaved partial sums).
float row_dot(const Mat& m, long row, const float* x) {
  const int k = m.k;
  if (m.kind == 0) {
    const uint16_t* w = (const uint16_t*)m.w + row * k;
    __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
    int c = 0;
    for (; c + 16 <= k; c += 16) {
      const __m256 w0 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(w + c)));
      const __m256 w1 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(w + c + 8)));
      a0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(x + c), a0);
      a1 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(x + c + 8), a1);
    }
    float t[8];
    _mm256_storeu_ps(t, _mm256_add_ps(a0, a1));
    float s = ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
    for (; c < k; ++c) s += h2f(w[c]) * x[c];
    return s;
  }
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int c = 0; c < k; c += 8) {
    for (int j = 0; j < 8; ++j) acc[j] += deq(m, row, c + j) * x[c + j];
  }
  return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

// epilogue 0 store, 1 accumulate, 2 swiglu (rows = physical; y has rows/2 entries)
void gemv(const Mat& m, const float* x, float* y, int epi) {
  const int out = epi == 2 ? m.rows / 2 : m.rows;
  const long blocks = (out + 63) / 64;
  parallel_for(blocks, [&](long b) {
    const int r1 = (int)(b * 64 + 64 < out ? b * 64 + 64 : out);
    for (int r = (int)(b * 64); r < r1; ++r) {
      const float a = row_dot(m, r, x);
      if (epi == 0) y[r] = a;
      else if (epi == 1) y[r] = y[r] + a;
      else {
        const float u = row_dot(m, (long)r + out, x);
        y[r] = silu(a) * u;
      }
    }
  });
}

void rmsnorm(const float* x, const float* g, int n, float* y) {
  float ss = 0;
  for (int i = 0; i < n; ++i) ss += x[i] * x[i];
  const float inv = 1.0f / sqrtf(ss / (float)n + 1e-6f);
  for (int i = 0; i < n; ++i) y[i] = x[i] * inv * g[i];
}

// gdn step on the reference layouts: conv_state[c*3 + 0..2] (oldest first), state[h][j][t].
void gdn(const float* proj, float* conv_state, const float* conv_w, float* state, const float* prm, float* o) {
  static thread_local std::vector<float> cv;
  cv.resize(6144);
  for (int c = 0; c < 6144; ++c) {
    const float y = conv_state[c * 3] * conv_w[c * 4] + conv_state[c * 3 + 1] * conv_w[c * 4 + 1] +
                    conv_state[c * 3 + 2] * conv_w[c * 4 + 2] + proj[c] * conv_w[c * 4 + 3];
    cv[c] = silu(y);
    conv_state[c * 3] = conv_state[c * 3 + 1];
    conv_state[c * 3 + 1] = conv_state[c * 3 + 2];
    conv_state[c * 3 + 2] = proj[c];
  }
  const float* cvp = cv.data();
  parallel_for(16, [&](long hl) {
    const int h = (int)hl;
    const float* q = cvp + h * 128;
    const float* k = cvp + 2048 + h * 128;
    const float* v = cvp + 4096 + h * 128;
    float qs[128], ks[128], out[128];
    float nq = 0, nk = 0;
    for (int t = 0; t < 128; ++t) {
      nq += q[t] * q[t];
      nk += k[t] * k[t];
    }
    nq = 1.0f / sqrtf(nq + 1e-6f);
    nk = 1.0f / sqrtf(nk + 1e-6f);
    for (int t = 0; t < 128; ++t) {
      qs[t] = q[t] * nq * 0.08838834764f;
      ks[t] = k[t] * nk;
    }
    const float g = expf(prm[16 + h] * logf(1.0f + expf(proj[8192 + h] + prm[h])));
    const float beta = 1.0f / (1.0f + expf(-proj[8208 + h]));
    float kq = 0;
    for (int j = 0; j < 128; ++j) kq += ks[j] * qs[j];
    float* S = state + (size_t)h * 16384;
    float sk[128], sq[128];
    for (int t = 0; t < 128; ++t) sk[t] = sq[t] = 0;
    for (int j = 0; j < 128; ++j)
      for (int t = 0; t < 128; ++t) {
        sk[t] += S[j * 128 + t] * ks[j];
        sq[t] += S[j * 128 + t] * qs[j];
      }
    for (int t = 0; t < 128; ++t) {
      const float dv = beta * (v[t] - g * sk[t]);
      for (int j = 0; j < 128; ++j) S[j * 128 + t] = g * S[j * 128 + t] + dv * ks[j];
      out[t] = g * sq[t] + dv * kq;
    }
    float ss = 0;
    for (int t = 0; t < 128; ++t) ss += out[t] * out[t];
    const float inv = 1.0f / sqrtf(ss / 128.0f + 1e-6f);
    for (int t = 0; t < 128; ++t) o[h * 128 + t] = out[t] * inv * silu(proj[6144 + h * 128 + t]) * prm[32 + t];
  });
}

// norm + rope of one 256-vector at `pos` (rope: [2][4096][32] cos, sin).
void norm_rope(const float* x, const float* w, const float* rope, int pos, float* y) {
  rmsnorm(x, w, 256, y);
  for (int i = 0; i < 32; ++i) {
    const float c = rope[pos * 32 + i], s = rope[kMaxCtx * 32 + pos * 32 + i];
    const float a = y[i], b = y[i + 32];
    y[i] = a * c - b * s;
    y[i + 32] = b * c + a * s;
  }
}

// attention step; kc/vc: [2][4096][256] f32 caches (reference contiguous layout, untransposed).
// Writes the current key/value into the caches (rounded to f16 when kv_f16) before attending.
void attention(const float* proj, float* kc, float* vc, int pos, const float* prm, const float* rope, int kv_f16,
               float* o) {
  for (int kvh = 0; kvh < 2; ++kvh) {
    float kcur[256];
    norm_rope(proj + 4096 + kvh * 256, prm + 256, rope, pos, kcur);
    for (int j = 0; j < 256; ++j) {
      float kv = kcur[j], vv = proj[4608 + kvh * 256 + j];
      if (kv_f16) {
        kv = h2f(f2h(kv));
        vv = h2f(f2h(vv));
      }
      kc[((size_t)kvh * kMaxCtx + pos) * 256 + j] = kv;
      vc[((size_t)kvh * kMaxCtx + pos) * 256 + j] = vv;
    }
  }
  parallel_for(8, [&](long hl) {
    const int h = (int)hl;
    const int kvh = h / 4;
    float q[256];
    norm_rope(proj + h * 256, prm, rope, pos, q);
    std::vector<float> e(pos + 1);
    float m = -3.0e38f;
    for (int l = 0; l <= pos; ++l) {
      const float* kr = kc + ((size_t)kvh * kMaxCtx + l) * 256;
      float d = 0;
      for (int j = 0; j < 256; ++j) d += q[j] * kr[j];
      e[l] = d * 0.0625f;
      m = e[l] > m ? e[l] : m;
    }
    float total = 0;
    for (int l = 0; l <= pos; ++l) {
      e[l] = expf(e[l] - m);
      total += e[l];
    }
    for (int t = 0; t < 256; ++t) {
      float acc = 0;
      for (int l = 0; l <= pos; ++l) acc += e[l] * vc[((size_t)kvh * kMaxCtx + l) * 256 + t];
      o[h * 256 + t] = acc / total / (1.0f + expf(-proj[2048 + h * 256 + t]));
    }
  });
}

uint32_t argmax(const float* x, long n) {
  uint32_t best = 0;
  float bv = -INFINITY;
  for (long i = 0; i < n; ++i)
    if (x[i] > bv) {
      bv = x[i];
      best = (uint32_t)i;
    }
  return best;
}

struct Layer {
  int attn;
  Mat in, out, gate_up, down;
  const float *input_norm, *post_norm, *attn_norms, *conv_w, *gdn_params;
};

struct Model {
  int layers, every, hidden, inter, vocab, kv_f16;
  Mat embed, lm_head;
  const float* final_norm;
  std::vector<Layer> L;
  std::vector<float> rope;
  // state
  std::vector<std::vector<float>> conv, rec, kc, vc;
  std::vector<float> h, xn, proj, mixed, act, logits;
};


// ------------------------------------------------------------------------------------------
// Batched prompt processing on the CPU: the same per-token arithmetic as oracle_model_step for n
// consecutive tokens, restructured so a 4000-token prompt takes seconds. The reference's batched
// prefill (kernels/src/batch.rs:16-371, driven by kernels/src/model.rs:222-259) runs the token
// graph's operators over chunks of tokens; here every operator runs over all n tokens at once.
// Differences from n calls of oracle_model_step: only the f32 summation order of the matrix
// products (blocked over rows and tokens instead of one row_dot per output). RMSNorm, the GDN
// conv/recurrence/gated norm and attention use the per-token functions' loops in the same order,
// so for equal inputs they give equal bits.
// ------------------------------------------------------------------------------------------

inline float hsum8(__m256 v) {
  float t[8];
  _mm256_storeu_ps(t, v);
  return ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
}

// out[r][t] = sum_c W[r][c] * X[t][c] for 4 rows of W (f32, row stride k) and NT token rows of X.
template <int NT>
void micro4(const float* W, const float* const* X, int k, float out[4][3]) {
  __m256 acc[4][NT];
  for (int r = 0; r < 4; ++r)
    for (int t = 0; t < NT; ++t) acc[r][t] = _mm256_setzero_ps();
  int c = 0;
  for (; c + 8 <= k; c += 8) {
    __m256 x[NT];
    for (int t = 0; t < NT; ++t) x[t] = _mm256_loadu_ps(X[t] + c);
    for (int r = 0; r < 4; ++r) {
      const __m256 w = _mm256_loadu_ps(W + (size_t)r * k + c);
      for (int t = 0; t < NT; ++t) acc[r][t] = _mm256_fmadd_ps(w, x[t], acc[r][t]);
    }
  }
  for (int r = 0; r < 4; ++r)
    for (int t = 0; t < NT; ++t) {
      float v = hsum8(acc[r][t]);
      for (int cc = c; cc < k; ++cc) v += W[(size_t)r * k + cc] * X[t][cc];
      out[r][t] = v;
    }
}

// Y[t][r] (=, +=, SwiGLU) for the n token rows X[t][0..k) against matrix m (epilogues as gemv;
// for SwiGLU Y has rows/2 columns). Work is tiled as (16 output rows) x (96 tokens), with the
// tiles of one token block running together so that block stays in the shared cache.
void gemm_tokens(const Mat& m, const float* X, int n, float* Y, int ldy, int epi) {
  const int k = m.k;
  const int out = epi == 2 ? m.rows / 2 : m.rows;
  constexpr int kRowBlk = 16, kTokBlk = 96;
  const int rb_count = (out + kRowBlk - 1) / kRowBlk;
  const int tb_count = (n + kTokBlk - 1) / kTokBlk;
  parallel_for((long)rb_count * tb_count, [&](long task) {
    const int tb = (int)(task / rb_count), rb = (int)(task % rb_count);
    const int r0 = rb * kRowBlk, r1 = std::min(out, r0 + kRowBlk);
    const int t0 = tb * kTokBlk, t1 = std::min(n, t0 + kTokBlk);
    const int nr = r1 - r0;
    // dequantized rows: [gate rows][up rows] for SwiGLU, padded to whole groups of 4
    const int groups = epi == 2 ? 2 : 1;
    static thread_local std::vector<float> wbuf;
    const int pad_rows = (nr + 3) / 4 * 4;
    wbuf.assign((size_t)groups * pad_rows * k, 0.f);
    for (int g = 0; g < groups; ++g)
      for (int r = 0; r < nr; ++r) {
        float* dst = wbuf.data() + ((size_t)g * pad_rows + r) * k;
        const long row = (long)r0 + r + (g ? out : 0);
        if (m.kind == 0) {
          const uint16_t* src = (const uint16_t*)m.w + (size_t)row * k;
          int c = 0;
          for (; c + 8 <= k; c += 8)
            _mm256_storeu_ps(dst + c, _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(src + c))));
          for (; c < k; ++c) dst[c] = h2f(src[c]);
        } else {
          for (int c = 0; c < k; ++c) dst[c] = deq(m, row, c);
        }
      }
    float res[2][kRowBlk][3];
    for (int t = t0; t < t1; t += 3) {
      const int nt = std::min(3, t1 - t);
      const float* xs[3] = {X + (size_t)t * k, X + (size_t)(t + (nt > 1)) * k, X + (size_t)(t + 2 * (nt > 2)) * k};
      for (int g = 0; g < groups; ++g)
        for (int r = 0; r < pad_rows; r += 4) {
          float o[4][3];
          const float* wr = wbuf.data() + ((size_t)g * pad_rows + r) * k;
          if (nt == 3) micro4<3>(wr, xs, k, o);
          else if (nt == 2) micro4<2>(wr, xs, k, o);
          else micro4<1>(wr, xs, k, o);
          for (int i = 0; i < 4 && r + i < kRowBlk; ++i)
            for (int j = 0; j < nt; ++j) res[g][r + i][j] = o[i][j];
        }
      for (int j = 0; j < nt; ++j) {
        float* y = Y + (size_t)(t + j) * ldy;
        for (int r = 0; r < nr; ++r) {
          const float a = res[0][r][j];
          if (epi == 0) y[r0 + r] = a;
          else if (epi == 1) y[r0 + r] = y[r0 + r] + a;
          else y[r0 + r] = silu(a) * res[1][r][j];
        }
      }
    }
  });
}

// gdn for n consecutive tokens: P[n][8224] projections, O[n][2048] gated outputs; conv_state and
// state are updated as n calls of gdn() would. Each (head, 8 value columns) recurrence runs
// sequentially over the tokens with its 128 x 8 state slice in registers/L1.
void gdn_tokens(const float* P, int n, float* conv_state, const float* conv_w, float* state, const float* prm,
                float* O) {
  std::vector<float> cv((size_t)n * 6144);
  parallel_for(6144 / 64, [&](long blk) {
    for (int c = (int)blk * 64; c < (int)blk * 64 + 64; ++c) {
      float w0 = conv_state[c * 3], w1 = conv_state[c * 3 + 1], w2 = conv_state[c * 3 + 2];
      for (int t = 0; t < n; ++t) {
        const float x = P[(size_t)t * kGdnProj + c];
        const float y = w0 * conv_w[c * 4] + w1 * conv_w[c * 4 + 1] + w2 * conv_w[c * 4 + 2] + x * conv_w[c * 4 + 3];
        cv[(size_t)t * 6144 + c] = silu(y);
        w0 = w1;
        w1 = w2;
        w2 = x;
      }
      conv_state[c * 3] = w0;
      conv_state[c * 3 + 1] = w1;
      conv_state[c * 3 + 2] = w2;
    }
  });
  // per (token, head): scaled unit q, unit k, decay g, beta, k.q
  std::vector<float> qs((size_t)n * 2048), ks((size_t)n * 2048), gb((size_t)n * 48);
  parallel_for((long)n * 16, [&](long i) {
    const int t = (int)(i / 16), h = (int)(i % 16);
    const float* q = cv.data() + (size_t)t * 6144 + h * 128;
    const float* k = q + 2048;
    const float* proj = P + (size_t)t * kGdnProj;
    float nq = 0, nk = 0;
    for (int j = 0; j < 128; ++j) {
      nq += q[j] * q[j];
      nk += k[j] * k[j];
    }
    nq = 1.0f / sqrtf(nq + 1e-6f);
    nk = 1.0f / sqrtf(nk + 1e-6f);
    float* qo = qs.data() + (size_t)t * 2048 + h * 128;
    float* ko = ks.data() + (size_t)t * 2048 + h * 128;
    for (int j = 0; j < 128; ++j) {
      qo[j] = q[j] * nq * 0.08838834764f;
      ko[j] = k[j] * nk;
    }
    float kq = 0;
    for (int j = 0; j < 128; ++j) kq += ko[j] * qo[j];
    float* o = gb.data() + (size_t)t * 48 + h * 3;
    o[0] = expf(prm[16 + h] * logf(1.0f + expf(proj[8192 + h] + prm[h])));
    o[1] = 1.0f / (1.0f + expf(-proj[8208 + h]));
    o[2] = kq;
  });
  std::vector<float> raw((size_t)n * 2048);
  parallel_for(16 * 16, [&](long i) {
    const int h = (int)(i / 16), c0 = (int)(i % 16) * 8;
    float S[128][8];
    for (int j = 0; j < 128; ++j)
      for (int c = 0; c < 8; ++c) S[j][c] = state[(size_t)h * 16384 + j * 128 + c0 + c];
    for (int t = 0; t < n; ++t) {
      const float* kv = ks.data() + (size_t)t * 2048 + h * 128;
      const float* qv = qs.data() + (size_t)t * 2048 + h * 128;
      const float* v = cv.data() + (size_t)t * 6144 + 4096 + h * 128;
      const float g = gb[(size_t)t * 48 + h * 3], beta = gb[(size_t)t * 48 + h * 3 + 1],
                  kq = gb[(size_t)t * 48 + h * 3 + 2];
      float sk[8] = {0, 0, 0, 0, 0, 0, 0, 0}, sq[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int j = 0; j < 128; ++j)
        for (int c = 0; c < 8; ++c) {
          sk[c] += S[j][c] * kv[j];
          sq[c] += S[j][c] * qv[j];
        }
      for (int c = 0; c < 8; ++c) {
        const float dv = beta * (v[c0 + c] - g * sk[c]);
        for (int j = 0; j < 128; ++j) S[j][c] = g * S[j][c] + dv * kv[j];
        raw[(size_t)t * 2048 + h * 128 + c0 + c] = g * sq[c] + dv * kq;
      }
    }
    for (int j = 0; j < 128; ++j)
      for (int c = 0; c < 8; ++c) state[(size_t)h * 16384 + j * 128 + c0 + c] = S[j][c];
  });
  parallel_for((long)n * 16, [&](long i) {
    const int t = (int)(i / 16), h = (int)(i % 16);
    const float* out = raw.data() + (size_t)t * 2048 + h * 128;
    const float* proj = P + (size_t)t * kGdnProj;
    float ss = 0;
    for (int c = 0; c < 128; ++c) ss += out[c] * out[c];
    const float inv = 1.0f / sqrtf(ss / 128.0f + 1e-6f);
    for (int c = 0; c < 128; ++c)
      O[(size_t)t * 2048 + h * 128 + c] = out[c] * inv * silu(proj[6144 + h * 128 + c]) * prm[32 + c];
  });
}

// attention for n consecutive tokens at positions start..start+n-1 (P[n][8224] rows hold the
// 5120 attention projections): every key/value is appended first, then each (token, head) attends
// over positions 0..its own, as attention() does for one token.
void attention_tokens(const float* P, int n, int start, float* kc, float* vc, const float* prm, const float* rope,
                      int kv_f16, float* O) {
  parallel_for((long)n * 2, [&](long i) {
    const int t = (int)(i / 2), kvh = (int)(i % 2), pos = start + t;
    const float* proj = P + (size_t)t * kGdnProj;
    float kcur[256];
    norm_rope(proj + 4096 + kvh * 256, prm + 256, rope, pos, kcur);
    for (int j = 0; j < 256; ++j) {
      float kv = kcur[j], vv = proj[4608 + kvh * 256 + j];
      if (kv_f16) {
        kv = h2f(f2h(kv));
        vv = h2f(f2h(vv));
      }
      kc[((size_t)kvh * kMaxCtx + pos) * 256 + j] = kv;
      vc[((size_t)kvh * kMaxCtx + pos) * 256 + j] = vv;
    }
  });
  parallel_for((long)n * 8, [&](long i) {
    const int t = (int)(i / 8), h = (int)(i % 8), kvh = h / 4, pos = start + t;
    const float* proj = P + (size_t)t * kGdnProj;
    float q[256];
    norm_rope(proj + h * 256, prm, rope, pos, q);
    std::vector<float> e(pos + 1);
    float m = -3.0e38f;
    for (int l = 0; l <= pos; ++l) {
      const float* kr = kc + ((size_t)kvh * kMaxCtx + l) * 256;
      float d = 0;
      for (int j = 0; j < 256; ++j) d += q[j] * kr[j];
      e[l] = d * 0.0625f;
      m = e[l] > m ? e[l] : m;
    }
    float total = 0;
    for (int l = 0; l <= pos; ++l) {
      e[l] = expf(e[l] - m);
      total += e[l];
    }
    float acc[256];
    for (int c = 0; c < 256; ++c) acc[c] = 0;
    for (int l = 0; l <= pos; ++l) {
      const float* vr = vc + ((size_t)kvh * kMaxCtx + l) * 256;
      const float el = e[l];
      for (int c = 0; c < 256; ++c) acc[c] += el * vr[c];
    }
    for (int c = 0; c < 256; ++c)
      O[(size_t)t * 2048 + h * 256 + c] = acc[c] / total / (1.0f + expf(-proj[2048 + h * 256 + c]));
  });
}

}  // namespace

// ------------------------------------------------------------------------------------------
// C ABI for the Python tests
// ------------------------------------------------------------------------------------------
API float oracle_f16_to_f32_ref(uint16_t h) {
  // kernels/src/lib.rs:473-482 verbatim semantics (exponent 31 -> NaN).
  const float sign = (h & 0x8000) ? -1.0f : 1.0f;
  const int e = (h >> 10) & 0x1f;
  const float frac = (float)(h & 0x3ff);
  if (e == 0) return sign * frac * ldexpf(1.0f, -24);
  if (e == 31) return NAN;
  return sign * (1.0f + frac / 1024.0f) * ldexpf(1.0f, e - 15);
}

API void oracle_dequant_rows(int kind, const void* w, const void* s, const void* z, int rows, int k, int row0,
                             int nrows, float* out) {
  Mat m{kind, rows, k, w, s, z};
  for (long r = 0; r < nrows; ++r)
    for (int c = 0; c < k; ++c) out[r * k + c] = deq(m, row0 + r, c);
}

API void oracle_gemv(int kind, const void* w, const void* s, const void* z, int rows, int k, const float* x,
                     float* y, int epilogue) {
  gemv(Mat{kind, rows, k, w, s, z}, x, y, epilogue);
}

API void oracle_rmsnorm(const float* x, const float* g, int n, float* y) { rmsnorm(x, g, n, y); }

API void oracle_gdn_step(const float* proj, float* conv_state, const float* conv_w, float* state,
                         const float* params, float* out) {
  gdn(proj, conv_state, conv_w, state, params, out);
}

API void oracle_rope_table(double theta, float* table) {
  for (int p = 0; p < kMaxCtx; ++p)
    for (int i = 0; i < 32; ++i) {
      const double a = (double)p * pow(theta, -(2.0 * i) / 64.0);
      table[p * 32 + i] = (float)cos(a);
      table[kMaxCtx * 32 + p * 32 + i] = (float)sin(a);
    }
}

API void oracle_attention_step(const float* proj, float* kc, float* vc, int pos, const float* norms,
                               const float* rope, int kv_f16, float* out) {
  attention(proj, kc, vc, pos, norms, rope, kv_f16, out);
}

API uint32_t oracle_argmax(const float* x, long n) { return argmax(x, n); }

API float oracle_round_f16(float x) { return h2f(f2h(x)); }

API int oracle_threads(void) { return pool().threads(); }

// Model: `ptrs` lists, in order, embed (w, s, z), lm_head (w, s, z), final_norm, then per layer
// input_norm, post_norm, mixer_in (w, s, z), mixer_out (w, s, z), gate_up (w, s, z),
// down (w, s, z), attn_norms or conv_w, gdn_params (NULL for attention layers).
// `kinds` lists the kind of embed, lm_head, then per layer in, out, gate_up, down.
API void* oracle_model_new(int layers, int every, int hidden, int inter, int vocab, double theta, int kv_f16,
                           const void* const* ptrs, const int* kinds) {
  Model* m = new Model();
  m->layers = layers;
  m->every = every;
  m->hidden = hidden;
  m->inter = inter;
  m->vocab = vocab;
  m->kv_f16 = kv_f16;
  int p = 0, q = 0;
  auto mat = [&](int rows, int k) {
    Mat x{kinds[q++], rows, k, ptrs[p], ptrs[p + 1], ptrs[p + 2]};
    p += 3;
    return x;
  };
  m->embed = mat(vocab, hidden);
  m->lm_head = mat(vocab, hidden);
  m->final_norm = (const float*)ptrs[p++];
  for (int i = 0; i < layers; ++i) {
    Layer l;
    l.attn = (i + 1) % every == 0;
    l.input_norm = (const float*)ptrs[p++];
    l.post_norm = (const float*)ptrs[p++];
    l.in = mat(l.attn ? kAttnProj : kGdnProj, hidden);
    l.out = mat(hidden, kMixerOut);
    l.gate_up = mat(2 * inter, hidden);
    l.down = mat(hidden, inter);
    const float* a = (const float*)ptrs[p++];
    const float* b = (const float*)ptrs[p++];
    l.attn_norms = l.attn ? a : nullptr;
    l.conv_w = l.attn ? nullptr : a;
    l.gdn_params = l.attn ? nullptr : b;
    m->L.push_back(l);
  }
  m->rope.resize((size_t)2 * kMaxCtx * 32);
  oracle_rope_table(theta, m->rope.data());
  m->conv.resize(layers);
  m->rec.resize(layers);
  m->kc.resize(layers);
  m->vc.resize(layers);
  for (int i = 0; i < layers; ++i) {
    if (m->L[i].attn) {
      m->kc[i].assign((size_t)2 * kMaxCtx * 256, 0.f);
      m->vc[i].assign((size_t)2 * kMaxCtx * 256, 0.f);
    } else {
      m->conv[i].assign(6144 * 3, 0.f);
      m->rec[i].assign(16 * 16384, 0.f);
    }
  }
  m->h.resize(hidden);
  m->xn.resize(hidden);
  m->proj.resize(kGdnProj);
  m->mixed.resize(kMixerOut);
  m->act.resize(inter);
  m->logits.resize(vocab);
  return m;
}

API void oracle_model_free(void* h) { delete (Model*)h; }

API void oracle_model_reset(void* hm) {
  Model* m = (Model*)hm;
  for (auto* v : {&m->conv, &m->rec, &m->kc, &m->vc})
    for (auto& x : *v) std::fill(x.begin(), x.end(), 0.f);
}

// One token at `pos`; with logits_out != NULL runs the final norm + LM head too.
API void oracle_model_step(void* hm, uint32_t token, int pos, float* logits_out) {
  Model* m = (Model*)hm;
  const int H = m->hidden;
  for (int c = 0; c < H; ++c) m->h[c] = deq(m->embed, token, c);
  for (int i = 0; i < m->layers; ++i) {
    const Layer& l = m->L[i];
    rmsnorm(m->h.data(), l.input_norm, H, m->xn.data());
    gemv(l.in, m->xn.data(), m->proj.data(), 0);
    if (l.attn) attention(m->proj.data(), m->kc[i].data(), m->vc[i].data(), pos, l.attn_norms, m->rope.data(), m->kv_f16, m->mixed.data());
    else gdn(m->proj.data(), m->conv[i].data(), l.conv_w, m->rec[i].data(), l.gdn_params, m->mixed.data());
    gemv(l.out, m->mixed.data(), m->h.data(), 1);
    rmsnorm(m->h.data(), l.post_norm, H, m->xn.data());
    gemv(l.gate_up, m->xn.data(), m->act.data(), 2);
    gemv(l.down, m->act.data(), m->h.data(), 1);
  }
  if (logits_out) {
    rmsnorm(m->h.data(), m->final_norm, H, m->xn.data());
    gemv(m->lm_head, m->xn.data(), logits_out, 0);
  }
}

// n consecutive tokens from position `start` through the batched CPU path (gemm_tokens,
// gdn_tokens, attention_tokens); with logits_out != NULL the final norm + LM head run on the last
// token. Leaves the state as n oracle_model_step calls would (within the matrix products' f32
// summation order).
API int oracle_model_prefill(void* hm, const uint32_t* ids, int n, int start, float* logits_out) {
  Model* m = (Model*)hm;
  if (n < 1 || start < 0 || start + n > kMaxCtx) return -1;
  const int H = m->hidden, I = m->inter;
  std::vector<float> X((size_t)n * H), XN((size_t)n * H), P((size_t)n * kGdnProj), MIX((size_t)n * kMixerOut),
      A((size_t)n * I);
  parallel_for(n, [&](long t) {
    for (int c = 0; c < H; ++c) X[(size_t)t * H + c] = deq(m->embed, ids[t], c);
  });
  auto norm_rows = [&](const float* g) {
    parallel_for(n, [&](long t) { rmsnorm(X.data() + (size_t)t * H, g, H, XN.data() + (size_t)t * H); });
  };
  for (int i = 0; i < m->layers; ++i) {
    const Layer& l = m->L[i];
    norm_rows(l.input_norm);
    gemm_tokens(l.in, XN.data(), n, P.data(), kGdnProj, 0);
    if (l.attn)
      attention_tokens(P.data(), n, start, m->kc[i].data(), m->vc[i].data(), l.attn_norms, m->rope.data(), m->kv_f16,
                       MIX.data());
    else
      gdn_tokens(P.data(), n, m->conv[i].data(), l.conv_w, m->rec[i].data(), l.gdn_params, MIX.data());
    gemm_tokens(l.out, MIX.data(), n, X.data(), H, 1);
    norm_rows(l.post_norm);
    gemm_tokens(l.gate_up, XN.data(), n, A.data(), I, 2);
    gemm_tokens(l.down, A.data(), n, X.data(), H, 1);
  }
  memcpy(m->h.data(), X.data() + (size_t)(n - 1) * H, (size_t)H * 4);
  if (logits_out) {
    rmsnorm(m->h.data(), m->final_norm, H, m->xn.data());
    gemv(m->lm_head, m->xn.data(), logits_out, 0);
  }
  return 0;
}

// Whole-state copy and restore (Model::snapshot / restore, kernels/src/model.rs:394-414).
API void oracle_model_snapshot(void* hm, void** saved) {
  Model* m = (Model*)hm;
  auto* copy = new std::vector<std::vector<float>>();
  for (auto* v : {&m->conv, &m->rec, &m->kc, &m->vc})
    for (auto& x : *v) copy->push_back(x);
  delete (std::vector<std::vector<float>>*)*saved;
  *saved = copy;
}

API int oracle_model_restore(void* hm, void* saved) {
  Model* m = (Model*)hm;
  auto* copy = (std::vector<std::vector<float>>*)saved;
  if (!copy) return -1;
  size_t j = 0;
  for (auto* v : {&m->conv, &m->rec, &m->kc, &m->vc})
    for (auto& x : *v) x = (*copy)[j++];
  return 0;
}

API void oracle_snapshot_free(void* saved) { delete (std::vector<std::vector<float>>*)saved; }

// Synthetic history for throughput samples: keys/values of positions [0, len) and the GDN states
// and conv windows filled with seeded values (xorshift64, U(-scale, scale)); the cost of a decode
// step depends on the context length only, not on these values.
API void oracle_model_fill_synthetic(void* hm, int len, uint64_t seed) {
  Model* m = (Model*)hm;
  auto fill = [&](float* p, size_t n, float scale, bool f16) {
    uint64_t s = seed * 0x9E3779B97F4A7C15ull + n;
    if (s == 0) s = 1;
    for (size_t i = 0; i < n; ++i) {
      s ^= s << 13;
      s ^= s >> 7;
      s ^= s << 17;
      float v = ((float)((uint32_t)(s >> 32) >> 8) / (float)(1u << 24) * 2.0f - 1.0f) * scale;
      p[i] = f16 ? h2f(f2h(v)) : v;
    }
    ++seed;
  };
  for (int i = 0; i < m->layers; ++i) {
    if (m->L[i].attn) {
      for (int kvh = 0; kvh < 2; ++kvh) {
        fill(m->kc[i].data() + (size_t)kvh * kMaxCtx * 256, (size_t)len * 256, 0.5f, m->kv_f16);
        fill(m->vc[i].data() + (size_t)kvh * kMaxCtx * 256, (size_t)len * 256, 0.5f, m->kv_f16);
      }
    } else {
      fill(m->conv[i].data(), m->conv[i].size(), 0.5f, false);
      fill(m->rec[i].data(), m->rec[i].size(), 0.05f, false);
    }
  }
}

// Test hook for the batched matrix product: Y[n][out] for X[n][k] (epilogues as oracle_gemv).
API void oracle_gemm_tokens(int kind, const void* w, const void* s, const void* z, int rows, int k, const float* x,
                            int n, float* y, int epilogue) {
  gemm_tokens(Mat{kind, rows, k, w, s, z}, x, n, y, epilogue == 2 ? rows / 2 : rows, epilogue);
}

// Copies of the state for inspection: GDN layer i -> conv (6144*3) + rec (16*16384);
// attention layer i -> first `len` positions of K and V per kv head ([2][len][256] each).
API int oracle_model_state(void* hm, int layer, float* a, float* b, int len) {
  Model* m = (Model*)hm;
  if (layer < 0 || layer >= m->layers) return -1;
  if (m->L[layer].attn) {
    for (int kvh = 0; kvh < 2; ++kvh) {
      memcpy(a + (size_t)kvh * len * 256, m->kc[layer].data() + (size_t)kvh * kMaxCtx * 256, (size_t)len * 256 * 4);
      memcpy(b + (size_t)kvh * len * 256, m->vc[layer].data() + (size_t)kvh * kMaxCtx * 256, (size_t)len * 256 * 4);
    }
    return 1;
  }
  memcpy(a, m->conv[layer].data(), 6144 * 3 * 4);
  memcpy(b, m->rec[layer].data(), 16 * 16384 * 4);
  return 0;
}

// The reference's xorshift64 generator (kernels/src/lib.rs:170-182): next_u32 and f32 draws.
API void oracle_rng_u32(uint64_t* state, long n, uint32_t* out) {
  uint64_t s = *state;
  for (long i = 0; i < n; ++i) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    out[i] = (uint32_t)(s >> 32);
  }
  *state = s;
}

API void oracle_rng_f32(uint64_t* state, long n, float* out) {
  uint64_t s = *state;
  for (long i = 0; i < n; ++i) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    out[i] = (float)((uint32_t)(s >> 32) >> 8) / (float)(1u << 24) * 2.0f - 1.0f;
  }
  *state = s;
}
