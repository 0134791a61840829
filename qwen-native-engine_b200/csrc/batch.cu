// Batched decode of independent sequences sharing one weight copy (qne_batch_*).
//
// The reference decodes a single sequence (kernels/src/model.rs:380-449); this runner applies the
// same per-token graph (kernels/src/model.rs:220-269) to `batch` sequences at once, each with its
// own GDN conv windows and recurrent states, its own position, and its own page table into a
// shared pool of 16-token f16 KV pages. Per step and layer:
//   GEMM mixer_in | GDN step + gated norm prep, or paged attention + copy prep | GEMM mixer_out
//   (+= h) | GEMM gate_up (SwiGLU -> hi/lo) | GEMM down (+= h);  before the first layer the
//   embedding prep, after the last the GEMM lm_head and the per-sequence greedy pick.
// The RMSNorms before mixer_in, gate_up and the LM head are folded into the GEMMs on either side
// (GemmArgs::norm_w_out / sumsq_in), so a step is 6 launches per layer plus 3 (int4 weights: one
// more launch per GEMM, which decodes the matrix to f16 for it). All launches of one step are
// captured once into a CUDA graph (programmatic dependent launch between kernels).
#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/qne.h"
#include "batch.cuh"
#include "gdn.cuh"
#include "model.hpp"

namespace qne {

class BatchRunner {
 public:
  BatchRunner(Model* m, int batch, uint32_t pool_pages);
  ~BatchRunner();
  Model* m;
  int B, Bp;
  uint32_t pool_pages;
  SeqState st;
  float *h = nullptr, *proj = nullptr, *raw = nullptr, *logits = nullptr;
  uint16_t *x0h = nullptr, *x0l = nullptr, *x1h = nullptr, *x1l = nullptr;
  uint16_t *xnh = nullptr, *xnl = nullptr;  // planes of h * norm weight (RMSNorm folded into the GEMMs)
  float* sumsq = nullptr;                   // [hidden / 16][kGemmMaxRows] partial sums of h^2
  uint16_t* wdeq = nullptr;  // int4 models: f16 copy of the matrix the next GEMM reads
  int ldx0 = 0;
  uint32_t* picks = nullptr;
  void* argmax_scratch = nullptr;
  void* attn_scratch = nullptr;
  cudaGraphExec_t graph[2] = {nullptr, nullptr};  // 0 greedy, 1 host tokens
  size_t launches_per_step = 0;
  std::vector<uint32_t> host_pos;
  uint32_t* pinned = nullptr;  // staging: ctl entries, picks
  void record(bool greedy, cudaStream_t s);
  void capture();
};

namespace {

void* track(Model* m, SeqState& st, size_t bytes) {
  void* p = m->alloc(bytes);
  st.buffers.push_back({p, bytes});
  return p;
}

struct Guard {
  int prev = -1;
  explicit Guard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cuda_check(cudaSetDevice(dev), "cudaSetDevice");
  }
  ~Guard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

BatchRunner::BatchRunner(Model* model, int batch, uint32_t pool) : m(model), B(batch), pool_pages(pool) {
  const Config& c = m->cfg;
  Bp = (B + 7) / 8 * 8;
  st.batch = B;
  st.pool_pages = pool;
  st.conv.assign(c.layers, nullptr);
  st.rec.assign(c.layers, nullptr);
  st.kv.assign(c.layers, nullptr);
  for (int i = 0; i < c.layers; ++i) {
    if (m->layers[i].attention) {
      st.kv[i] = static_cast<uint16_t*>(track(m, st, (size_t)pool * kPageElems * 2));
    } else {
      st.conv[i] = static_cast<float*>(track(m, st, (size_t)B * kConvSlots * kConvChannels * 4));
      st.rec[i] = static_cast<float*>(track(m, st, (size_t)B * kGdnHeads * kGdnDim * kGdnDim * 4));
    }
  }
  st.ctl = static_cast<SeqCtl*>(track(m, st, (size_t)B * sizeof(SeqCtl)));
  st.page_table = static_cast<uint32_t*>(m->alloc((size_t)B * kPagesPerSeq * 4));
  std::vector<uint32_t> pt((size_t)B * kPagesPerSeq);
  for (size_t i = 0; i < pt.size(); ++i) pt[i] = (uint32_t)i;
  cuda_check(cudaMemcpy(st.page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice), "page table");
  ldx0 = c.hidden > kMixerOut ? c.hidden : kMixerOut;
  h = static_cast<float*>(m->alloc((size_t)B * c.hidden * 4));
  proj = static_cast<float*>(m->alloc((size_t)B * kGdnProj * 4));
  raw = static_cast<float*>(m->alloc((size_t)B * kMixerOut * 4));
  logits = static_cast<float*>(m->alloc((size_t)B * c.vocab * 4));
  x0h = static_cast<uint16_t*>(m->alloc((size_t)Bp * ldx0 * 2));
  x0l = static_cast<uint16_t*>(m->alloc((size_t)Bp * ldx0 * 2));
  x1h = static_cast<uint16_t*>(m->alloc((size_t)Bp * c.inter * 2));
  x1l = static_cast<uint16_t*>(m->alloc((size_t)Bp * c.inter * 2));
  for (auto* p : {x0h, x0l}) cuda_check(cudaMemset(p, 0, (size_t)Bp * ldx0 * 2), "memset");
  for (auto* p : {x1h, x1l}) cuda_check(cudaMemset(p, 0, (size_t)Bp * c.inter * 2), "memset");
  xnh = static_cast<uint16_t*>(m->alloc((size_t)Bp * c.hidden * 2));
  xnl = static_cast<uint16_t*>(m->alloc((size_t)Bp * c.hidden * 2));
  for (auto* p : {xnh, xnl}) cuda_check(cudaMemset(p, 0, (size_t)Bp * c.hidden * 2), "memset");
  sumsq = static_cast<float*>(m->alloc((size_t)(c.hidden / 16) * kGemmMaxRows * 4));
  cuda_check(cudaMemset(sumsq, 0, (size_t)(c.hidden / 16) * kGemmMaxRows * 4), "memset");
  picks = static_cast<uint32_t*>(m->alloc((size_t)B * 4));
  argmax_scratch = m->alloc(argmax_batched_scratch_bytes(B));
  cuda_check(cudaMemset(argmax_scratch, 0, argmax_batched_scratch_bytes(B)), "memset");
  attn_scratch = m->alloc(attention_scratch_bytes(B));
  cuda_check(cudaMemset(attn_scratch, 0, attention_scratch_bytes(B)), "memset");
  host_pos.assign(B, 0);
  cuda_check(cudaMallocHost(&pinned, (size_t)B * 16 + 64), "cudaMallocHost");
  size_t deq_elems = 0;  // the largest int4 matrix a step multiplies, decoded to f16 before its GEMM
  for (const LayerWeights& L : m->layers)
    for (const Mat* w : {&L.in, &L.out, &L.gate_up, &L.down})
      if (w->kind != kF16) deq_elems = std::max(deq_elems, (size_t)w->rows * w->k);
  if (m->lm_head.kind != kF16) deq_elems = std::max(deq_elems, (size_t)m->lm_head.rows * m->lm_head.k);
  if (deq_elems) wdeq = static_cast<uint16_t*>(m->alloc(deq_elems * 2));
}

BatchRunner::~BatchRunner() {
  for (auto& g : graph)
    if (g) cudaGraphExecDestroy(g);
  if (pinned) cudaFreeHost(pinned);
}

void BatchRunner::record(bool greedy, cudaStream_t s) {
  const Model& M = *m;
  const Config& c = M.cfg;
  size_t n = 0;
  auto prep = [&](PrepArgs p) {
    p.xh = x0h;
    p.xl = x0l;
    p.ldx = ldx0;
    cuda_check(launch_prep(p, B, s, true), "prep launch");
    ++n;
  };
  // RMSNorm folded into the GEMMs: the GEMM that updates h writes the planes of h * (next norm
  // weight) and partial sums of h^2; the GEMM that reads those planes applies 1 / rms.
  const int slots = c.hidden / 16;
  auto gemm = [&](const Mat& w, const uint16_t* xh, const uint16_t* xl, int ldx, int epi, float* y, uint16_t* yh,
                  uint16_t* yl, int ldy, const float* norm_out, bool norm_in) {
    GemmArgs g;
    g.w = w.w;
    g.rows = w.rows;
    g.k = w.k;
    g.batch = B;
    g.epi = epi;
    if (w.kind != kF16) {
      // int4: widened to f16 inside the GEMM, or (the many-wave LM head) decoded into the f16
      // scratch first
      g.wkind = w.kind;
      g.ws = w.s;
      g.wz = w.z;
      if (!gemm_int4_direct(g)) {
        if (w.k % 64) throw QneError(kEInval, "batched decode of int4 matrices needs k % 64 == 0");
        cuda_check(launch_dequant_f16(w, wdeq, s, true), "dequant launch");
        ++n;
        g.wkind = kF16;
        g.w = wdeq;
        g.w_after_wait = true;
      }
    }
    g.row_groups = gemm_row_groups(epi == kSwiGlu ? w.rows / 2 : w.rows);
    g.xh = xh;
    g.xl = xl;
    g.ldx = ldx;
    g.y = y;
    g.yh = yh;
    g.yl = yl;
    g.ldy = ldy;
    if (norm_out) {
      g.norm_w_out = norm_out;
      g.out_xh = xnh;
      g.out_xl = xnl;
      g.out_ldx = c.hidden;
      g.sumsq_out = sumsq;
    }
    if (norm_in) {
      g.sumsq_in = sumsq;
      g.sumsq_slots = slots;
      g.norm_k = c.hidden;
    }
    if (const char* why = check_gemm(g)) throw QneError(kEInval, why);
    cuda_check(launch_gemm(g, s, true), "gemm launch");
    ++n;
  };
  {
    PrepArgs p;  // embedding rows -> h, planes of h * input_norm[0], sums of squares
    p.mode = kPrepEmbedNorm;
    p.k = c.hidden;
    p.norm_w = M.layers[0].input_norm;
    p.embed = M.embed;
    p.ctl = st.ctl;
    p.h = h;
    p.ldh = c.hidden;
    p.sumsq_out = sumsq;
    p.sumsq_slots = slots;
    p.xh = xnh;
    p.xl = xnl;
    p.ldx = c.hidden;
    cuda_check(launch_prep(p, B, s, true), "prep launch");
    ++n;
  }
  for (int i = 0; i < c.layers; ++i) {
    const LayerWeights& L = M.layers[i];
    gemm(L.in, xnh, xnl, c.hidden, kStore, proj, nullptr, nullptr, L.in.rows, nullptr, true);
    PrepArgs q;
    q.k = kMixerOut;
    q.src = raw;
    q.lds = kMixerOut;
    if (L.attention) {
      AttnArgs at;
      at.proj = proj;
      at.norms = L.attn_norms;
      at.rope = M.rope;
      at.kv = st.kv[i];
      at.page_table = st.page_table;
      at.pos = &st.ctl->pos;
      at.pos_stride = 4;
      at.flags = &st.ctl->flags;
      at.flags_stride = 4;
      at.out = raw;
      at.out_xh = x0h;  // the out-projection's activation planes, written by the merge itself
      at.out_xl = x0l;
      at.out_ldx = ldx0;
      at.batch = B;
      at.scratch = attn_scratch;
      cuda_check(launch_attention(at, pool_pages, B >= 8 ? 256 : 64, s, true), "attention launch");
      ++n;
    } else {
      cuda_check(launch_gdn_step(proj, st.conv[i], L.conv_w, st.rec[i], L.gdn_params, &st.ctl->count, 4, raw, B, s,
                                 true),
                 "gdn launch");
      ++n;
      q.mode = kPrepGdnGate;
      q.zgate = proj;
      q.norm_w = L.gdn_params + 32;
    }
    if (!L.attention) prep(q);
    gemm(L.out, x0h, x0l, ldx0, kAccumulate, h, nullptr, nullptr, c.hidden, L.post_norm, false);
    gemm(L.gate_up, xnh, xnl, c.hidden, kSwiGlu, nullptr, x1h, x1l, c.inter, nullptr, true);
    const float* next_norm = i + 1 < c.layers ? M.layers[i + 1].input_norm : M.final_norm;
    gemm(L.down, x1h, x1l, c.inter, kAccumulate, h, nullptr, nullptr, c.hidden, next_norm, false);
  }
  gemm(M.lm_head, xnh, xnl, c.hidden, kStore, logits, nullptr, nullptr, c.vocab, nullptr, true);
  cuda_check(launch_argmax_batched(logits, (uint32_t)c.vocab, (size_t)c.vocab, B, st.ctl, picks, argmax_scratch,
                                   greedy ? 1 : 0, s, true),
             "argmax launch");
  ++n;
  launches_per_step = n;
}

void BatchRunner::capture() {
  cudaStream_t cs;
  cuda_check(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "cudaStreamCreate");
  for (int v = 0; v < 2; ++v) {
    cuda_check(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
      record(v == 0, cs);
    } catch (...) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(cs, &g);
      if (g) cudaGraphDestroy(g);
      cudaStreamDestroy(cs);
      throw;
    }
    cudaGraph_t g = nullptr;
    cuda_check(cudaStreamEndCapture(cs, &g), "end capture");
    const cudaError_t e = cudaGraphInstantiate(&graph[v], g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      cudaStreamDestroy(cs);
      cuda_check(e, "graph instantiate");
    }
  }
  cudaStreamDestroy(cs);
}

}  // namespace qne

using namespace qne;

// The C ABI error slot lives in capi.cu; batch entry points report through the same helper.
extern "C" qne_status qne_internal_fail(int code, const char* msg);

namespace {
qne_status bfail(int code, const std::string& msg) { return qne_internal_fail(code, msg.c_str()); }

template <typename F>
qne_status bguard(F&& f) {
  try {
    f();
    qne_internal_fail(0, "");
    return QNE_OK;
  } catch (const QneError& e) {
    return bfail(e.code, e.what());
  } catch (const std::bad_alloc&) {
    return bfail(QNE_ENOMEM, "host allocation failed");
  } catch (const std::exception& e) {
    return bfail(QNE_EINVAL, e.what());
  }
}

struct BatchHandle {
  Model* model;
  BatchRunner* r;
};

void sync_stream(cudaStream_t s, uint32_t timeout_ms) {
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  uint32_t spins = 0;
  for (;;) {
    const cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return;
    if (e != cudaErrorNotReady) cuda_check(e, "stream");
    if (std::chrono::steady_clock::now() > deadline)
      throw QneError(kETimeout, "GPU wait exceeded " + std::to_string(timeout_ms) + " ms");
    if (++spins < 20000) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace

extern "C" {

qne_status qne_batch_create(qne_model* m, uint32_t batch, uint32_t pool_pages, qne_batch** out) {
  if (!out) return bfail(QNE_EINVAL, "null output handle");
  *out = nullptr;
  if (!m) return bfail(QNE_EINVAL, "null model handle");
  return bguard([&] {
    Model* M = reinterpret_cast<Model*>(m);
    if (batch < 1 || batch > 32) throw QneError(kEInval, "batch must be 1..32");
    if (pool_pages < batch * (uint32_t)kPagesPerSeq)
      throw QneError(kEInval, "pool_pages must hold 256 pages per sequence");
    if (pool_pages > (1u << 24)) throw QneError(kEInval, "pool_pages too large");
    Guard g(M->device);
    auto* r = new BatchRunner(M, (int)batch, pool_pages);
    try {
      r->capture();
      for (auto& b : r->st.buffers) cuda_check(cudaMemset(b.first, 0, b.second), "reset");
      cuda_check(cudaDeviceSynchronize(), "batch create");
    } catch (...) {
      delete r;
      throw;
    }
    *out = reinterpret_cast<qne_batch*>(new BatchHandle{M, r});
  });
}

void qne_batch_free(qne_batch* b) {
  if (!b) return;
  auto* h = reinterpret_cast<BatchHandle*>(b);
  delete h->r;
  delete h;
}

#define BATCH(b)                                                    \
  if (!(b)) return bfail(QNE_EINVAL, "null batch handle");         \
  BatchHandle* H = reinterpret_cast<BatchHandle*>(b);               \
  BatchRunner* R = H->r;                                            \
  Model* M = H->model;

qne_status qne_batch_set_page_table(qne_batch* b, const uint32_t* table, size_t n) {
  BATCH(b);
  return bguard([&] {
    if (!table || n != (size_t)R->B * kPagesPerSeq) throw QneError(kEInval, "page table needs batch x 256 entries");
    for (size_t i = 0; i < n; ++i)
      if (table[i] >= R->pool_pages) throw QneError(kEInval, "page id " + std::to_string(table[i]) + " outside the pool");
    Guard g(M->device);
    cuda_check(cudaStreamSynchronize(M->stream()), "page table");
    cuda_check(cudaMemcpy(R->st.page_table, table, n * 4, cudaMemcpyHostToDevice), "page table");
  });
}

qne_status qne_batch_reset(qne_batch* b) {
  BATCH(b);
  return bguard([&] {
    Guard g(M->device);
    for (auto& x : R->st.buffers) cuda_check(cudaMemsetAsync(x.first, 0, x.second, M->stream()), "reset");
    std::fill(R->host_pos.begin(), R->host_pos.end(), 0u);
  });
}

qne_status qne_batch_step(qne_batch* b, const uint32_t* tokens, const uint32_t* pos, float* logits_out,
                          uint32_t* next_out) {
  BATCH(b);
  return bguard([&] {
    if (!tokens || !pos) throw QneError(kEInval, "null tokens or positions");
    for (int i = 0; i < R->B; ++i)
      if (pos[i] >= (uint32_t)kMaxContext)
        throw QneError(kERangeCtx, "context limit of " + std::to_string(kMaxContext) + " tokens reached");
    Guard g(M->device);
    cudaStream_t s = M->stream();
    cuda_check(cudaStreamSynchronize(s), "batch step");
    for (int i = 0; i < R->B; ++i) {
      R->pinned[2 * i] = tokens[i];
      R->pinned[2 * i + 1] = pos[i];
    }
    // (token, pos) of every SeqCtl; count and flags stay on the device
    cuda_check(cudaMemcpy2DAsync(R->st.ctl, sizeof(SeqCtl), R->pinned, 8, 8, R->B, cudaMemcpyHostToDevice, s),
               "batch tokens");
    // The greedy graph: each sequence is left at (its pick, pos + 1), ready for decode_async.
    cuda_check(cudaGraphLaunch(R->graph[0], s), "batch graph");
    for (size_t i = 0; i < R->launches_per_step; ++i) count_launch();
    for (int i = 0; i < R->B; ++i) R->host_pos[i] = pos[i] + 1;
    if (next_out) cuda_check(cudaMemcpyAsync(next_out, R->picks, (size_t)R->B * 4, cudaMemcpyDeviceToHost, s), "picks");
    if (logits_out)
      cuda_check(cudaMemcpyAsync(logits_out, R->logits, (size_t)R->B * M->cfg.vocab * 4, cudaMemcpyDeviceToHost, s),
                 "logits");
    sync_stream(s, 600000);
  });
}

qne_status qne_batch_decode_async(qne_batch* b, uint32_t steps) {
  BATCH(b);
  return bguard([&] {
    for (int i = 0; i < R->B; ++i)
      if ((uint64_t)R->host_pos[i] + steps > (uint64_t)kMaxContext)
        throw QneError(kERangeCtx, "context limit of " + std::to_string(kMaxContext) + " tokens reached (sequence " +
                                       std::to_string(i) + ")");
    Guard g(M->device);
    for (uint32_t k = 0; k < steps; ++k) {
      cuda_check(cudaGraphLaunch(R->graph[0], M->stream()), "batch graph");
      for (size_t i = 0; i < R->launches_per_step; ++i) count_launch();
    }
    for (int i = 0; i < R->B; ++i) R->host_pos[i] += steps;
  });
}

qne_status qne_batch_tokens(qne_batch* b, uint32_t* tokens, uint32_t* pos) {
  BATCH(b);
  return bguard([&] {
    Guard g(M->device);
    std::vector<SeqCtl> ctl(R->B);
    cuda_check(cudaStreamSynchronize(M->stream()), "batch tokens");
    cuda_check(cudaMemcpy(ctl.data(), R->st.ctl, (size_t)R->B * sizeof(SeqCtl), cudaMemcpyDeviceToHost), "ctl");
    for (int i = 0; i < R->B; ++i) {
      if (tokens) tokens[i] = ctl[i].token;
      if (pos) pos[i] = ctl[i].pos;
      R->host_pos[i] = ctl[i].pos;
    }
  });
}

qne_status qne_batch_fill_synthetic(qne_batch* b, uint32_t seq, uint32_t len, uint32_t token, uint64_t seed) {
  BATCH(b);
  return bguard([&] {
    if (seq >= (uint32_t)R->B) throw QneError(kEInval, "sequence index outside the batch");
    if (len >= (uint32_t)kMaxContext) throw QneError(kERangeCtx, "len must be < 4096");
    Guard g(M->device);
    cudaStream_t s = M->stream();
    const uint32_t* table = R->st.page_table + (size_t)seq * kPagesPerSeq;
    for (int i = 0; i < M->cfg.layers; ++i) {
      const uint64_t ls = seed * 1000003ull + (uint64_t)i * 7919ull + seq;
      if (M->layers[i].attention) {
        cuda_check(launch_fill_kv(R->st.kv[i], table, len, ls, R->pool_pages, s), "fill kv");
      } else {
        cuda_check(launch_fill_f32(R->st.rec[i] + (size_t)seq * kGdnHeads * kGdnDim * kGdnDim,
                                   (size_t)kGdnHeads * kGdnDim * kGdnDim, ls, 0.05f, s),
                   "fill state");
        cuda_check(launch_fill_f32(R->st.conv[i] + (size_t)seq * kConvSlots * kConvChannels,
                                   (size_t)kConvSlots * kConvChannels, ls + 1, 0.5f, s),
                   "fill conv");
      }
    }
    SeqCtl c{token, len, len, 0};
    cuda_check(cudaStreamSynchronize(s), "fill");
    cuda_check(cudaMemcpy(R->st.ctl + seq, &c, sizeof(c), cudaMemcpyHostToDevice), "fill ctl");
    R->host_pos[seq] = len;
  });
}

qne_status qne_batch_sync(qne_batch* b, uint32_t timeout_ms) {
  if (!b) return bfail(QNE_EINVAL, "null batch handle");
  Model* M = reinterpret_cast<BatchHandle*>(b)->model;
  return bguard([&] {
    Guard g(M->device);
    sync_stream(M->stream(), timeout_ms);
  });
}

size_t qne_gemm_scratch_bytes(const qne_matrix* m, int batch) {
  (void)m;
  (void)batch;
  return 0;
}

qne_status qne_gemm(const qne_matrix* m, const float* x, int batch, float* y, int epilogue, void* scratch,
                    size_t scratch_bytes, void* stream) {
  (void)scratch;
  (void)scratch_bytes;
  return qne_gemm_ex(m, x, batch, y, epilogue, QNE_GEMM_TENSOR_CORE, stream);
}

qne_status qne_gemm_ex(const qne_matrix* m, const float* x, int batch, float* y, int epilogue, int impl,
                       void* stream) {
  return bguard([&] {
    if (impl != QNE_GEMM_TENSOR_CORE && impl != QNE_GEMM_MMA_SYNC) throw QneError(kEInval, "unknown GEMM kernel");
    if (!m || !x || !y) throw QneError(kEInval, "null argument");
    if (m->kind != QNE_KIND_F16 && impl != QNE_GEMM_TENSOR_CORE)
      throw QneError(kEInval, "int4 weights need the tensor-core GEMM");
    if (epilogue < 0 || epilogue > 2) throw QneError(kEInval, "unknown epilogue");
    if (batch < 1 || batch > (impl == QNE_GEMM_MMA_SYNC ? 32 : kGemmMaxRows))
      throw QneError(kEInval, impl == QNE_GEMM_MMA_SYNC ? "batch must be 1..32" : "batch must be 1..64");
    if (m->k % 32 || m->k <= 0 || m->rows <= 0) throw QneError(kEInval, "batched GEMM needs k % 32 == 0");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Stage x as hi/lo planes (8-row padded) in a per-device workspace that lives until exit.
    const int Bp = (batch + 7) / 8 * 8;
    const size_t plane = (size_t)Bp * m->k * 2;
    static thread_local std::vector<std::pair<void*, size_t>> ws(64, {nullptr, 0});
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    auto& slot = ws.at(dev);
    const int out_rows = epilogue == QNE_EPI_SWIGLU ? m->rows / 2 : m->rows;
    const size_t need = 2 * plane + (epilogue == QNE_EPI_SWIGLU ? 2 * (size_t)Bp * out_rows * 2 : 0);
    if (slot.second < need) {
      if (slot.first) {
        cuda_check(cudaStreamSynchronize(s), "gemm workspace");
        cudaFree(slot.first);
      }
      slot.first = nullptr;
      cuda_check(cudaMalloc(&slot.first, need), "gemm workspace");
      cuda_check(cudaMemset(slot.first, 0, need), "gemm workspace");
      slot.second = need;
    }
    uint16_t* xh = static_cast<uint16_t*>(slot.first);
    uint16_t* xl = xh + plane / 2;
    PrepArgs p;
    p.mode = kPrepCopy;
    p.k = m->k;
    p.src = x;
    p.lds = m->k;
    p.xh = xh;
    p.xl = xl;
    p.ldx = m->k;
    cuda_check(launch_prep(p, batch, s, false), "gemm prep");
    GemmArgs g;
    g.w = m->w;
    if (m->kind != QNE_KIND_F16) {  // QNE_KIND_* are the engine's weight kinds
      g.wkind = m->kind;
      g.ws = m->s;
      g.wz = m->z;
    }
    g.rows = m->rows;
    g.k = m->k;
    g.batch = batch;
    g.epi = epilogue;
    g.row_groups = gemm_row_groups(out_rows);
    g.xh = xh;
    g.xl = xl;
    g.ldx = m->k;
    g.ldy = out_rows;
    g.impl = impl == QNE_GEMM_MMA_SYNC ? kGemmMmaSync : kGemmTensorCore;
    uint16_t* yh = xl + plane / 2;
    uint16_t* yl = yh + (size_t)Bp * out_rows;
    if (epilogue == QNE_EPI_SWIGLU) {
      g.yh = yh;
      g.yl = yl;
    } else {
      g.y = y;
    }
    if (const char* why = check_gemm(g)) throw QneError(kEInval, why);
    cuda_check(launch_gemm(g, s, false), "gemm");
    if (epilogue == QNE_EPI_SWIGLU) {
      // the operator returns f32: hi + lo
      cuda_check(launch_hilo_to_f32(yh, yl, y, (size_t)batch * out_rows, s), "gemm swiglu output");
    }
  });
}

}  // extern "C"
