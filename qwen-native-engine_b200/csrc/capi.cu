// extern "C" entry points declared in include/qne.h. Every call converts C++ exceptions into
// a status code plus a thread-local message; nothing escapes across the ABI.
#include <cstring>
#include <string>

#include "../../include/qne.h"
#include "gdn.cuh"
#include "json.hpp"
#include "model.hpp"

using namespace qne;

namespace {

thread_local std::string g_error;

int fail(int code, const std::string& msg) {
  g_error = msg;
  return code;
}

template <typename F>
qne_status guarded(F&& f) {
  try {
    f();
    g_error.clear();
    return QNE_OK;
  } catch (const QneError& e) {
    return fail(e.code, e.what());
  } catch (const std::bad_alloc&) {
    return fail(QNE_ENOMEM, "host allocation failed");
  } catch (const std::exception& e) {
    return fail(QNE_EINVAL, e.what());
  }
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

Mat to_mat(const qne_matrix* m) {
  if (!m) throw QneError(kEInval, "null matrix");
  Mat r;
  r.kind = m->kind;
  r.rows = m->rows;
  r.k = m->k;
  r.w = m->w;
  r.s = m->s;
  r.z = m->z;
  return r;
}

void check_launch(cudaError_t e, const char* what) { cuda_check(e, what); }

}  // namespace

extern "C" {

// Error slot shared with the batch entry points (not exported).
qne_status qne_internal_fail(int code, const char* msg) {
  g_error = msg ? msg : "";
  return code;
}

const char* qne_last_error(void) { return g_error.c_str(); }
const char* qne_version(void) { return "qne-b200 0.1 (sm_100a)"; }
uint64_t qne_kernel_launches(void) { return launches_issued(); }

qne_status qne_model_load(const char* index_json, size_t index_len, const void* weights,
                          size_t weights_len, int device, qne_model** out) {
  return qne_model_load_ex(index_json, index_len, weights, weights_len, device, 0, out);
}

qne_status qne_model_load_ex(const char* index_json, size_t index_len, const void* weights, size_t weights_len,
                             int device, uint32_t flags, qne_model** out) {
  if (!out) return fail(QNE_EINVAL, "null output handle");
  *out = nullptr;
  if (flags & ~(uint32_t)QNE_LOAD_ANY_SHAPE) return fail(QNE_EINVAL, "unknown load flags");
  return guarded([&] {
    *out = reinterpret_cast<qne_model*>(
        Model::load(index_json, index_len, weights, weights_len, device, (flags & QNE_LOAD_ANY_SHAPE) != 0));
  });
}

void qne_model_free(qne_model* m) { delete reinterpret_cast<Model*>(m); }

#define MODEL(m)                                                     \
  if (!(m)) return fail(QNE_EINVAL, "null model handle");           \
  Model* M = reinterpret_cast<Model*>(m);

qne_status qne_model_info_get(const qne_model* m, qne_model_info* out) {
  if (!m || !out) return fail(QNE_EINVAL, "null argument");
  const Model* M = reinterpret_cast<const Model*>(m);
  out->layers = M->cfg.layers;
  out->hidden = M->cfg.hidden;
  out->intermediate = M->cfg.inter;
  out->vocab = M->cfg.vocab;
  out->weight_kind = M->weight_kind;
  out->embed_kind = M->embed_kind;
  out->tied_lm_head = M->tied ? 1 : 0;
  out->device = M->device;
  out->weight_bytes = M->weight_bytes;
  out->device_bytes = M->device_bytes;
  return QNE_OK;
}

qne_status qne_model_set_stream(qne_model* m, void* cuda_stream) {
  MODEL(m);
  M->set_stream(as_stream(cuda_stream));
  return QNE_OK;
}

qne_status qne_model_set_fused(qne_model* m, int enable) {
  MODEL(m);
  return guarded([&] {
    if (!M->set_fused(enable != 0))
      throw QneError(kEInval, "the fused layer kernels need one sequence, f16 weights with k % 256 == 0 and a "
                              "device that co-schedules the grid");
  });
}

qne_status qne_model_set_path(qne_model* m, int path) {
  MODEL(m);
  return guarded([&] {
    if (path < QNE_PATH_OPERATIONS || path > QNE_PATH_TOKEN) throw QneError(kEInval, "unknown launch path");
    if (!M->set_path(path))
      throw QneError(kEInval, path == QNE_PATH_TOKEN
                                  ? "the token kernel needs one sequence, f16 matrices with k % 256 == 0 and "
                                    "k <= 6144, and a CTA per SM co-resident"
                                  : "the fused layer kernels need one sequence, f16 weights with k % 256 == 0 and a "
                                    "device that co-schedules the grid");
  });
}

int qne_model_path(const qne_model* m) { return m ? reinterpret_cast<const Model*>(m)->path() : -1; }

qne_status qne_model_set_phase_trace(qne_model* m, int enable) {
  MODEL(m);
  return guarded([&] { M->set_phase_trace(enable != 0); });
}

qne_status qne_model_phase_trace(qne_model* m, uint64_t* out, size_t cap, size_t* n_out, size_t* ctas) {
  MODEL(m);
  return guarded([&] {
    const size_t n = M->read_phase_trace(out, cap, ctas);
    if (n_out) *n_out = n;
  });
}

qne_status qne_profile_token(qne_model* m, qne_profile_entry* out, size_t cap, size_t* n_out) {
  MODEL(m);
  return guarded([&] {
    const auto prof = M->profile_token();
    if (n_out) *n_out = prof.size();
    for (size_t i = 0; i < prof.size() && i < cap && out; ++i) {
      std::memset(&out[i], 0, sizeof(out[i]));
      std::strncpy(out[i].label, prof[i].first.c_str(), sizeof(out[i].label) - 1);
      out[i].ms = prof[i].second.first;
      out[i].dispatches = prof[i].second.second;
    }
  });
}

qne_status qne_model_test_barrier_timeout(qne_model* m, uint32_t limit_us) {
  MODEL(m);
  return guarded([&] {
    if (limit_us > 2000000u) throw QneError(kEInval, "limit_us must be at most 2000000");
    M->set_wait_test((uint64_t)limit_us * 1000ull);
  });
}

int qne_model_fused(const qne_model* m) {
  return m ? (reinterpret_cast<const Model*>(m)->fused() ? 1 : 0) : 0;
}

const char* qne_adapter(const qne_model* m) {
  return m ? reinterpret_cast<const Model*>(m)->adapter.c_str() : "";
}

size_t qne_dispatches_per_token(const qne_model* m) {
  return m ? reinterpret_cast<const Model*>(m)->dispatches_per_token() : 0;
}

qne_status qne_validate_tiles(const char* tiles_json, size_t len) {
  // ModelTiles::validate, kernels/src/model.rs:101-109.
  return guarded([&] {
    if (!tiles_json) throw QneError(kEInval, "null tile profile");
    Json j;
    try {
      j = Json::parse(tiles_json, len);
    } catch (const JsonError& e) {
      throw QneError(kEFormat, e.what());
    }
    for (const char* name : {"gdn_in", "attn_in", "out", "gate_up", "down", "lm_head"}) {
      const Json* t = j.get(name);
      if (!t || t->type != Json::Object) throw QneError(kEFormat, std::string("invalid kernel tile profile: missing ") + name);
      auto field = [&](const char* f) -> double {
        const Json* v = t->get(f);
        if (!v || !v->is_number()) throw QneError(kEFormat, std::string("invalid kernel tile profile: ") + name);
        return v->num;
      };
      const Json* f16 = t->get("f16");
      if (!f16 || f16->type != Json::Bool) throw QneError(kEFormat, std::string("invalid kernel tile profile: ") + name);
      const double tpr = field("tpr"), rpw = field("rpw"), rpt = field("rpt"), splits = field("splits");
      auto in = [](double v, std::initializer_list<int> set) {
        for (int s : set)
          if (v == s) return true;
        return false;
      };
      const bool ok = in(tpr, {1, 2, 4, 8, 16, 32, 64}) && in(rpw, {2, 4, 8, 16, 32}) && in(rpt, {1, 2, 4, 8}) &&
                      in(splits, {1, 2, 4, 8}) && tpr * rpw <= 256 && (f16->b || (rpt == 1 && splits == 1));
      if (!ok) throw QneError(kEFormat, std::string("invalid kernel tile profile: ") + name);
    }
  });
}

qne_status qne_reset(qne_model* m) {
  MODEL(m);
  return guarded([&] { M->reset(); });
}

qne_status qne_prefill(qne_model* m, const uint32_t* ids, uint32_t n) {
  MODEL(m);
  return guarded([&] {
    // Model::prefill, kernels/src/model.rs:324-335: prompt length 1..4095 from position 0.
    if (n == 0 || n >= (uint32_t)kMaxContext)
      throw QneError(kERangeCtx, "prompt length must be 1.." + std::to_string(kMaxContext));
    M->prefill_chunk(ids, n, 0, true, false);
  });
}

qne_status qne_prefill_chunk(qne_model* m, const uint32_t* ids, uint32_t n, uint32_t start,
                             int finish_logits) {
  MODEL(m);
  return guarded([&] { M->prefill_chunk(ids, n, start, finish_logits != 0); });
}

int qne_prefill_chunk_batched(const qne_model* m) {
  if (!m) return 0;
  return reinterpret_cast<const Model*>(m)->prefill_batched_supported() ? 1 : 0;
}

qne_status qne_logits(qne_model* m, float* out, size_t out_len) {
  MODEL(m);
  return guarded([&] { M->logits(out, out_len); });
}

qne_status qne_step(qne_model* m, uint32_t token, uint32_t pos, float* logits_out, size_t out_len) {
  MODEL(m);
  return guarded([&] { M->step(token, pos, logits_out, out_len); });
}

qne_status qne_snapshot(qne_model* m) {
  MODEL(m);
  return guarded([&] { M->snapshot(); });
}

qne_status qne_restore(qne_model* m) {
  MODEL(m);
  return guarded([&] { M->restore(); });
}

qne_status qne_last_token(qne_model* m, uint32_t* token, uint32_t* pos) {
  MODEL(m);
  return guarded([&] { M->last_token(token, pos); });
}

qne_status qne_decode(qne_model* m, uint32_t n, uint32_t window, const uint32_t* stop, uint32_t nstop,
                      uint32_t* ids_out, uint32_t* n_out) {
  MODEL(m);
  if (nstop && !stop) return fail(QNE_EINVAL, "null stop list");
  return guarded([&] { M->decode(n, window, stop, nstop, ids_out, n_out); });
}

qne_status qne_decode_async(qne_model* m, uint32_t steps) {
  MODEL(m);
  return guarded([&] { M->decode_async(steps); });
}

qne_status qne_step_async(qne_model* m, uint32_t token, uint32_t pos) {
  MODEL(m);
  return guarded([&] { M->step_async(token, pos); });
}

qne_status qne_sync(qne_model* m, uint32_t timeout_ms) {
  MODEL(m);
  return guarded([&] { M->sync(timeout_ms); });
}

const float* qne_logits_device(const qne_model* m) {
  return m ? reinterpret_cast<const Model*>(m)->logits_device() : nullptr;
}

qne_status qne_model_matrix(const qne_model* m, const char* name, qne_matrix* out) {
  if (!m || !name || !out) return fail(QNE_EINVAL, "null argument");
  const Model* M = reinterpret_cast<const Model*>(m);
  return guarded([&] {
    const std::string n(name);
    const Mat* x = nullptr;
    if (n == "embed") x = &M->embed;
    else if (n == "lm_head") x = &M->lm_head;
    else if (n.rfind("layer", 0) == 0) {
      const size_t dot = n.find('.');
      if (dot == std::string::npos) throw QneError(kEInval, "unknown matrix " + n);
      const int i = std::stoi(n.substr(5, dot - 5));
      if (i < 0 || i >= M->cfg.layers) throw QneError(kEInval, "unknown matrix " + n);
      const std::string part = n.substr(dot + 1);
      const LayerWeights& L = M->layers[i];
      if (part == "mixer_in") x = &L.in;
      else if (part == "mixer_out") x = &L.out;
      else if (part == "gate_up") x = &L.gate_up;
      else if (part == "down") x = &L.down;
    }
    if (!x) throw QneError(kEInval, "unknown matrix " + n);
    out->kind = x->kind;
    out->rows = x->rows;
    out->k = x->k;
    out->pad = 0;
    out->w = x->w;
    out->s = x->s;
    out->z = x->z;
  });
}

qne_status qne_model_tensor(const qne_model* m, const char* name, const void** out) {
  if (!m || !name || !out) return fail(QNE_EINVAL, "null argument");
  const Model* M = reinterpret_cast<const Model*>(m);
  return guarded([&] {
    const std::string n(name);
    const void* p = nullptr;
    if (n == "final_norm") p = M->final_norm;
    else if (n.rfind("layer", 0) == 0) {
      const size_t dot = n.find('.');
      if (dot == std::string::npos) throw QneError(kEInval, "unknown tensor " + n);
      const int i = std::stoi(n.substr(5, dot - 5));
      if (i < 0 || i >= M->cfg.layers) throw QneError(kEInval, "unknown tensor " + n);
      const std::string part = n.substr(dot + 1);
      const LayerWeights& L = M->layers[i];
      if (part == "input_norm") p = L.input_norm;
      else if (part == "post_norm") p = L.post_norm;
      else if (part == "attn_norms") p = L.attn_norms;
      else if (part == "conv_w") p = L.conv_w;
      else if (part == "gdn_params") p = L.gdn_params;
    }
    if (!p) throw QneError(kEInval, "unknown tensor " + n);
    *out = p;
  });
}

// ---- batched decode: see batch.cu ----

// ---- operators ----

qne_status qne_gemv(const qne_matrix* m, const float* x, float* y, int epilogue, void* stream) {
  return guarded([&] {
    GemvArgs a;
    a.m = to_mat(m);
    a.pro = kProCopy;
    a.x = x;
    a.y = y;
    if (epilogue < 0 || epilogue > 2) throw QneError(kEInval, "unknown epilogue");
    a.epi = epilogue;
    if (const char* why = check_gemv(a)) throw QneError(kEInval, why);
    check_launch(launch_gemv(a, as_stream(stream), false), "gemv");
  });
}

qne_status qne_gemv_ex(const qne_matrix* m, const float* x, float* y, int epilogue, int variant, int ctas_per_sm,
                       void* stream) {
  return guarded([&] {
    GemvArgs a;
    a.m = to_mat(m);
    a.pro = kProCopy;
    a.x = x;
    a.y = y;
    if (epilogue < 0 || epilogue > 2) throw QneError(kEInval, "unknown epilogue");
    if (ctas_per_sm != 1 && ctas_per_sm != 2) throw QneError(kEInval, "ctas_per_sm must be 1 or 2");
    a.epi = epilogue;
    a.variant = variant;
    a.ctas_per_sm = ctas_per_sm;
    if (const char* why = check_gemv(a)) throw QneError(kEInval, why);
    check_launch(launch_gemv(a, as_stream(stream), false), "gemv");
  });
}

qne_status qne_rmsnorm_gemv(const qne_matrix* m, const float* h, const float* norm_w, float eps,
                            float* y, int epilogue, void* stream) {
  return guarded([&] {
    GemvArgs a;
    a.m = to_mat(m);
    a.pro = kProRmsNorm;
    a.x = h;
    a.norm_w = norm_w;
    a.eps = eps;
    a.y = y;
    if (epilogue < 0 || epilogue > 2) throw QneError(kEInval, "unknown epilogue");
    a.epi = epilogue;
    if (const char* why = check_gemv(a)) throw QneError(kEInval, why);
    check_launch(launch_gemv(a, as_stream(stream), false), "rmsnorm_gemv");
  });
}

qne_status qne_dequant_rows(const qne_matrix* m, int row0, int nrows, float* out, void* stream) {
  return guarded([&] {
    const Mat mm = to_mat(m);
    if (!out || row0 < 0 || nrows < 0 || row0 + (long)nrows > mm.rows || mm.k <= 0)
      throw QneError(kEInval, "row range outside the matrix");
    if (mm.kind != kF16 && mm.kind != kQ4 && mm.kind != kQ4G64) throw QneError(kEInval, "unknown weight kind");
    if (mm.kind == kQ4 && mm.k % 256) throw QneError(kEInval, "block-32 int4 needs k % 256 == 0");
    if (mm.kind == kQ4G64 && mm.k % 64) throw QneError(kEInval, "group-64 int4 needs k % 64 == 0");
    if (nrows == 0) return;
    check_launch(launch_dequant_rows(mm, row0, nrows, out, as_stream(stream)), "dequant_rows");
  });
}

qne_status qne_embed(const qne_matrix* e, const uint32_t* tok, float* h, void* stream) {
  return guarded([&] {
    const Mat mm = to_mat(e);
    if (!tok || !h) throw QneError(kEInval, "null argument");
    // The embedding is a dequantized row: reuse dequant_rows on the row named by tok[0].
    uint32_t row = 0;
    cuda_check(cudaMemcpyAsync(&row, tok, 4, cudaMemcpyDeviceToHost, as_stream(stream)), "embed token");
    cuda_check(cudaStreamSynchronize(as_stream(stream)), "embed token");
    if (row >= (uint32_t)mm.rows) throw QneError(kEInval, "token id outside the embedding");
    check_launch(launch_dequant_rows(mm, (int)row, 1, h, as_stream(stream)), "embed");
  });
}

size_t qne_argmax_scratch_bytes(uint32_t n) {
  (void)n;
  return argmax_scratch_bytes();
}

qne_status qne_argmax(const float* logits, uint32_t n, uint32_t* tok, void* scratch, size_t scratch_bytes,
                      void* stream) {
  return guarded([&] {
    if (!logits || !tok || !scratch || n == 0) throw QneError(kEInval, "null argument or empty logits");
    if (scratch_bytes < argmax_scratch_bytes()) throw QneError(kEInval, "argmax scratch too small");
    // tok is [token, pos, ...]: the same first two words as SeqCtl.
    check_launch(launch_argmax(logits, n, reinterpret_cast<SeqCtl*>(tok), scratch, as_stream(stream), false),
                 "argmax");
  });
}

qne_status qne_gdn_step(const float* proj, float* conv, const float* conv_w, float* state, const float* params,
                        const uint32_t* counter, float* out, int batch, void* stream) {
  return guarded([&] {
    if (!proj || !conv || !conv_w || !state || !params || !counter || !out || batch < 1)
      throw QneError(kEInval, "null argument or batch < 1");
    // Raw output goes to `out`, then the gated norm rewrites it in place per head.
    check_launch(launch_gdn_step(proj, conv, conv_w, state, params, counter, 1, out, batch, as_stream(stream), false),
                 "gdn_step");
    check_launch(launch_gdn_gate(out, proj, params + 32, out, batch, as_stream(stream), false), "gdn_gate");
  });
}

size_t qne_attention_scratch_bytes(int batch) { return batch > 0 ? attention_scratch_bytes(batch) : 0; }

qne_status qne_attention_step(const float* proj, const float* norms, double rope_theta, void* kv,
                              uint32_t pool_pages, const uint32_t* page_table, const uint32_t* pos, float* out,
                              int batch, void* scratch, size_t scratch_bytes, void* stream) {
  return qne_attention_step_ex(proj, norms, rope_theta, kv, pool_pages, page_table, pos, out, batch, scratch,
                               scratch_bytes, QNE_ATTN_TENSOR_CORE, stream);
}

qne_status qne_attention_step_ex(const float* proj, const float* norms, double rope_theta, void* kv,
                                 uint32_t pool_pages, const uint32_t* page_table, const uint32_t* pos, float* out,
                                 int batch, void* scratch, size_t scratch_bytes, int impl, void* stream) {
  return guarded([&] {
    if (impl != QNE_ATTN_TENSOR_CORE && impl != QNE_ATTN_CUDA_CORE) throw QneError(kEInval, "unknown attention kernel");
    if (!proj || !norms || !kv || !page_table || !pos || !out || !scratch || batch < 1 || pool_pages == 0)
      throw QneError(kEInval, "null argument, batch < 1 or empty page pool");
    if (!(rope_theta > 0)) throw QneError(kEInval, "rope_theta must be positive");
    if (scratch_bytes < attention_scratch_bytes(batch)) throw QneError(kEInval, "attention scratch too small");
    AttnArgs a;
    a.proj = proj;
    a.norms = norms;
    a.rope = rope_table_device(rope_theta);
    a.kv = static_cast<uint16_t*>(kv);
    a.page_table = page_table;
    a.pos = pos;
    a.out = out;
    a.batch = batch;
    a.scratch = scratch;
    a.impl = impl == QNE_ATTN_CUDA_CORE ? 1 : 0;
    check_launch(launch_attention(a, pool_pages, batch >= 8 ? 256 : 64, as_stream(stream), false), "attention");
  });
}

qne_status qne_kv_gather(const void* kv, const uint32_t* page_table, uint32_t len, void* out_k, void* out_v,
                         void* stream) {
  return guarded([&] {
    if (!kv || !page_table || !out_k || !out_v) throw QneError(kEInval, "null argument");
    if (len > (uint32_t)kMaxContext) throw QneError(kEInval, "len above 4096");
    check_launch(launch_kv_gather(static_cast<const uint16_t*>(kv), page_table, len, static_cast<uint16_t*>(out_k),
                                  static_cast<uint16_t*>(out_v), as_stream(stream)),
                 "kv_gather");
  });
}

qne_status qne_dispatch_cost(uint32_t n, int mode, float* y, void* stream, double* us_per_dispatch) {
  return guarded([&] {
    if (!y || !us_per_dispatch || n == 0 || n > 100000 || mode < 0 || mode > 3)
      throw QneError(kEInval, "dispatch cost needs y, an output, 1..100000 launches and mode 0..3");
    *us_per_dispatch = dispatch_cost(n, mode, y, as_stream(stream));
  });
}

qne_status qne_bandwidth_probe(const void* data, size_t bytes, uint32_t* sink, void* stream) {
  return guarded([&] {
    if (!data || !sink || bytes == 0 || bytes % 16) throw QneError(kEInval, "bandwidth probe needs a non-empty multiple of 16 bytes");
    check_launch(launch_bandwidth_probe(data, bytes, sink, as_stream(stream)), "bandwidth_probe");
  });
}

}  // extern "C"
