// Decoder runtime: index.json validation (Index::validate, kernels/src/model.rs:51-86), weight
// upload with (offset, bytes) de-duplication (kernels/src/model.rs:184-194), device state, the
// per-token launch graph (kernels/src/model.rs:220-269) captured once as CUDA graphs whose
// kernels are chained by programmatic dependent launch, and the Model API
// (kernels/src/model.rs:305-449).
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <map>
#include <thread>

#include "gdn.cuh"
#include "json.hpp"
#include "model.hpp"
#include "prefill.hpp"
#include "persist.cuh"

namespace qne {

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw QneError(e == cudaErrorMemoryAllocation ? kENoMem : kECuda,
                   std::string(what) + ": " + cudaGetErrorString(e));
  }
}

namespace {


struct TensorEntry {
  uint64_t offset = 0, bytes = 0;
};

int kind_of(const std::string& k) {
  if (k == "f16") return kF16;
  if (k == "q4") return kQ4;
  if (k == "q4g64") return kQ4G64;
  throw QneError(kEFormat, "unsupported matrix kind: " + k);
}

double num(const Json& j, const char* key, bool required = true, double dflt = 0) {
  const Json* v = j.get(key);
  if (!v) {
    if (required) throw QneError(kEFormat, std::string("index.json: missing config.") + key);
    return dflt;
  }
  if (!v->is_number()) throw QneError(kEFormat, std::string("index.json: config.") + key + " is not a number");
  return v->num;
}

int as_int(double v, const char* what) {
  if (v != (double)(int64_t)v || v < 0 || v > 1e9)
    throw QneError(kEFormat, std::string("index.json: ") + what + " is not a valid integer");
  return (int)v;
}

}  // namespace

void* Model::alloc(size_t bytes, bool track) {
  void* p = nullptr;
  cuda_check(cudaMalloc(&p, bytes < 256 ? 256 : bytes), "cudaMalloc");
  allocations_.push_back(p);
  device_bytes += bytes;
  (void)track;
  return p;
}

void Model::free_all() {
  prefill_.reset();
  single_.reset();
  for (void* p : allocations_) cudaFree(p);
  allocations_.clear();
  if (host_ctl_) cudaFreeHost(host_ctl_);
  host_ctl_ = nullptr;
  if (own_stream_) cudaStreamDestroy(own_stream_);
  own_stream_ = nullptr;
}

Model::~Model() {
  // Never throws: a model that failed half-way through load() is destroyed here too.
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) {
    cudaGetLastError();
    prev = -1;
  }
  if (!allocations_.empty() || own_stream_ || host_ctl_) {
    if (prev != device) cudaSetDevice(device);
    free_all();
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
  }
  cudaGetLastError();
}

Model* Model::load(const char* json, size_t json_len, const void* weights, size_t weights_len,
                   int device, bool any_shape) {
  if (!json || !weights) throw QneError(kEInval, "null index or weights");
  if (device < 0) throw QneError(kEInval, "negative device index");

  Json index;
  try {
    index = Json::parse(json, json_len);
  } catch (const JsonError& e) {
    throw QneError(kEFormat, e.what());
  }
  const Json* cj = index.get("config");
  const Json* mj = index.get("matrices");
  const Json* tj = index.get("tensors");
  if (!cj || cj->type != Json::Object || !mj || mj->type != Json::Object || !tj || tj->type != Json::Object)
    throw QneError(kEFormat, "index.json: needs config, matrices and tensors objects");

  std::unique_ptr<Model> m(new Model());
  m->device = device;
  Config& c = m->cfg;
  c.layers = as_int(num(*cj, "layers"), "config.layers");
  c.every = as_int(num(*cj, "full_attention_every"), "config.full_attention_every");
  c.hidden = as_int(num(*cj, "hidden"), "config.hidden");
  c.inter = as_int(num(*cj, "intermediate", false, 0), "config.intermediate");
  if (c.inter == 0) c.inter = c.hidden == 1024 ? 3584 : 6144;  // kernels/src/model.rs:47-50
  c.vocab = as_int(num(*cj, "vocab"), "config.vocab");
  c.theta = num(*cj, "rope_theta");
  c.rope_dim = as_int(num(*cj, "rope_dim"), "config.rope_dim");
  // kernels/src/model.rs:51-55: the reference accepts the two Qwen3.5 sizes only (24 layers,
  // attention every 4th, (hidden, intermediate) (1024, 3584) or (2048, 6144), vocab 248320, rotary
  // width 64, theta 1e7), with this message.
  const bool reference_arch = c.layers == 24 && c.every == 4 &&
                              ((c.hidden == 1024 && c.inter == 3584) || (c.hidden == 2048 && c.inter == 6144)) &&
                              c.vocab == kVocab && c.rope_dim == 64 && c.theta == 10000000.0;
  if (!any_shape && !reference_arch)
    throw QneError(kEFormat, "unsupported model architecture: these kernels require Qwen3.5-0.8B or Qwen3.5-2B");
  // With QNE_LOAD_ANY_SHAPE the kernels still need: rotary width 64, hidden and intermediate
  // multiples of 256 (16-byte chunks per lane of a warp, int4 blocks of 32), fixed head geometry
  // (implied by the matrix shapes).
  if (c.layers < 1 || c.layers > 256 || c.every < 1 || c.hidden < 256 || c.hidden > 8192 ||
      c.hidden % 256 || c.inter < 256 || c.inter > 16384 || c.inter % 256 || c.vocab < 1 ||
      c.rope_dim != 64 || !(c.theta > 0))
    throw QneError(kEFormat, "unsupported model architecture: these kernels need a Qwen3.5-shaped "
                             "hybrid decoder (rope_dim 64, hidden and intermediate multiples of 256)");

  std::map<std::string, TensorEntry> tensors;
  for (const auto& kv : tj->obj) {
    const Json& t = kv.second;
    const Json* off = t.get("offset");
    const Json* by = t.get("bytes");
    if (!off || !by || !off->is_number() || !by->is_number())
      throw QneError(kEFormat, "invalid tensor range: " + kv.first);
    TensorEntry e;
    if (off->num < 0 || by->num < 0 || off->num != (double)(uint64_t)off->num || by->num != (double)(uint64_t)by->num)
      throw QneError(kEFormat, "invalid tensor range: " + kv.first);
    e.offset = (uint64_t)off->num;
    e.bytes = (uint64_t)by->num;
    // kernels/src/model.rs:56-60: in range, 4-byte aligned, non-empty, whole words.
    if (e.offset + e.bytes < e.offset || e.offset + e.bytes > weights_len || e.offset % 4 ||
        e.bytes == 0 || e.bytes % 4)
      throw QneError(kEFormat, "invalid tensor range: " + kv.first);
    tensors[kv.first] = e;
  }
  auto tensor = [&](const std::string& name, uint64_t expected) -> const TensorEntry& {
    auto it = tensors.find(name);
    if (it == tensors.end() || it->second.bytes != expected)
      throw QneError(kEFormat, "invalid tensor size: " + name);
    return it->second;
  };
  struct MatSpec {
    std::string name;
    int kind, rows, k;
  };
  std::vector<MatSpec> specs;
  auto matrix = [&](const std::string& name, int rows, int k) {
    const Json* s = mj->get(name);
    if (!s || !s->get("rows") || !s->get("k") || !s->get("rows")->is_number() || !s->get("k")->is_number() ||
        s->get("rows")->num != rows || s->get("k")->num != k)
      throw QneError(kEFormat, "invalid matrix shape: " + name);
    const Json* kj = s->get("kind");
    const int kind = kind_of(kj && kj->type == Json::String ? kj->str : std::string("q4"));
    const uint64_t el = (uint64_t)rows * (uint64_t)k;
    if (kind == kF16) {
      tensor(name + ".w", el * 2);
    } else if (kind == kQ4) {
      tensor(name + ".w", el / 2);
      tensor(name + ".s", el / 16);
      tensor(name + ".z", el / 64);
    } else {
      if (k % 64) throw QneError(kEFormat, "invalid matrix shape: " + name);
      tensor(name + ".w", el / 2);
      tensor(name + ".s", el / 32);
      tensor(name + ".z", el / 32);
    }
    specs.push_back({name, kind, rows, k});
  };
  matrix("embed", c.vocab, c.hidden);
  matrix("lm_head", c.vocab, c.hidden);
  tensor("final_norm", (uint64_t)c.hidden * 4);
  for (int i = 0; i < c.layers; ++i) {
    const bool attn = (i + 1) % c.every == 0;
    const std::string p = "layer" + std::to_string(i);
    tensor(p + ".input_norm", (uint64_t)c.hidden * 4);
    tensor(p + ".post_norm", (uint64_t)c.hidden * 4);
    matrix(p + ".mixer_in", attn ? kAttnProj : kGdnProj, c.hidden);
    matrix(p + ".mixer_out", c.hidden, kMixerOut);
    matrix(p + ".gate_up", c.inter * 2, c.hidden);
    matrix(p + ".down", c.hidden, c.inter);
    if (attn) {
      tensor(p + ".attn_norms", 2048);
    } else {
      tensor(p + ".conv_w", 98304);
      tensor(p + ".gdn_params", 640);
    }
  }

  // Validation is done; from here on the device is needed.
  int ndev = 0;
  cuda_check(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
  if (device >= ndev) throw QneError(kEInval, "no CUDA device " + std::to_string(device));
  DeviceGuard guard(device);
  cudaDeviceProp prop;
  cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major < 10)
    throw QneError(kECuda, std::string("device ") + prop.name + " is not sm_100 (this library is built for sm_100a)");
  m->adapter = std::string(prop.name) + " (sm_" + std::to_string(prop.major) + std::to_string(prop.minor) +
               "a, " + std::to_string(prop.multiProcessorCount) + " SMs, CUDA device " +
               std::to_string(device) + ")";

  // Upload every distinct (offset, bytes) range once into one arena, 256-byte aligned.
  std::map<std::pair<uint64_t, uint64_t>, uint64_t> placed;
  uint64_t arena_bytes = 0;
  for (const auto& kv : tensors) {
    const auto key = std::make_pair(kv.second.offset, kv.second.bytes);
    if (placed.count(key)) continue;
    placed[key] = arena_bytes;
    arena_bytes += (kv.second.bytes + 255) & ~uint64_t(255);
  }
  uint8_t* arena = static_cast<uint8_t*>(m->alloc(arena_bytes));
  m->arena_ = arena;
  for (const auto& kv : placed)
    cuda_check(cudaMemcpy(arena + kv.second, static_cast<const uint8_t*>(weights) + kv.first.first,
                          kv.first.second, cudaMemcpyHostToDevice),
               "upload weights");
  auto dptr = [&](const std::string& name) -> const void* {
    const TensorEntry& e = tensors.at(name);
    return arena + placed.at(std::make_pair(e.offset, e.bytes));
  };
  auto mat = [&](const MatSpec& s) {
    Mat r;
    r.kind = s.kind;
    r.rows = s.rows;
    r.k = s.k;
    r.w = dptr(s.name + ".w");
    if (s.kind != kF16) {
      r.s = dptr(s.name + ".s");
      r.z = dptr(s.name + ".z");
    }
    return r;
  };
  auto mat_bytes = [](const Mat& x) -> uint64_t {
    const uint64_t el = (uint64_t)x.rows * x.k;
    if (x.kind == kF16) return el * 2;
    if (x.kind == kQ4) return el / 2 + el / 16 + el / 64;
    return el / 2 + el / 16;
  };
  size_t si = 0;
  m->embed = mat(specs[si++]);
  m->lm_head = mat(specs[si++]);
  m->tied = m->embed.w == m->lm_head.w;
  m->final_norm = static_cast<const float*>(dptr("final_norm"));
  m->embed_kind = m->embed.kind;
  m->weight_bytes = mat_bytes(m->lm_head) + (uint64_t)c.hidden * 4;
  for (int i = 0; i < c.layers; ++i) {
    LayerWeights L;
    const std::string p = "layer" + std::to_string(i);
    L.attention = (i + 1) % c.every == 0;
    L.in = mat(specs[si++]);
    L.out = mat(specs[si++]);
    L.gate_up = mat(specs[si++]);
    L.down = mat(specs[si++]);
    L.input_norm = static_cast<const float*>(dptr(p + ".input_norm"));
    L.post_norm = static_cast<const float*>(dptr(p + ".post_norm"));
    if (L.attention) L.attn_norms = static_cast<const float*>(dptr(p + ".attn_norms"));
    else {
      L.conv_w = static_cast<const float*>(dptr(p + ".conv_w"));
      L.gdn_params = static_cast<const float*>(dptr(p + ".gdn_params"));
    }
    m->weight_bytes += mat_bytes(L.in) + mat_bytes(L.out) + mat_bytes(L.gate_up) + mat_bytes(L.down);
    m->layers.push_back(L);
  }
  m->weight_kind = m->layers[0].in.kind;

  std::vector<float> rope((size_t)2 * kMaxContext * kRopeHalf);
  rope_table_host(rope.data(), c.theta);
  m->rope = static_cast<float*>(m->alloc(rope.size() * 4));
  cuda_check(cudaMemcpy(m->rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice), "upload rope");

  cuda_check(cudaStreamCreateWithFlags(&m->own_stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  cuda_check(cudaMallocHost(&m->host_ctl_, (size_t)kMaxContext * 2 * sizeof(uint32_t) + 64), "cudaMallocHost");
  m->single_.reset(new Runner(m.get(), 1, kPagesPerSeq));
  m->single_->capture_graphs();
  m->single_->reset(m->stream());
  cuda_check(cudaStreamSynchronize(m->stream()), "load");
  return m.release();
}

// ------------------------------------------------------------------------------------------
// Runner
// ------------------------------------------------------------------------------------------
Runner::Runner(Model* model, int batch, uint32_t pool_pages) : m(model) {
  const Config& c = m->cfg;
  st.batch = batch;
  st.pool_pages = pool_pages;
  auto track = [&](size_t bytes) {
    void* p = m->alloc(bytes);
    st.buffers.push_back({p, bytes});
    return p;
  };
  st.conv.assign(c.layers, nullptr);
  st.rec.assign(c.layers, nullptr);
  st.kv.assign(c.layers, nullptr);
  for (int i = 0; i < c.layers; ++i) {
    if (m->layers[i].attention) {
      st.kv[i] = static_cast<uint16_t*>(track((size_t)pool_pages * kPageElems * 2));
    } else {
      st.conv[i] = static_cast<float*>(track((size_t)batch * kConvSlots * kConvChannels * 4));
      st.rec[i] = static_cast<float*>(track((size_t)batch * kGdnHeads * kGdnDim * kGdnDim * 4));
    }
  }
  st.ctl = static_cast<SeqCtl*>(track((size_t)batch * sizeof(SeqCtl)));
  barrier = static_cast<uint32_t*>(track(64));
  st.page_table = static_cast<uint32_t*>(m->alloc((size_t)batch * kPagesPerSeq * 4));
  std::vector<uint32_t> pt((size_t)batch * kPagesPerSeq);
  for (size_t i = 0; i < pt.size(); ++i) pt[i] = (uint32_t)i;
  cuda_check(cudaMemcpy(st.page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice), "page table");

  h = static_cast<float*>(m->alloc((size_t)batch * c.hidden * 4));
  proj = static_cast<float*>(m->alloc((size_t)batch * kGdnProj * 4));
  raw = static_cast<float*>(m->alloc((size_t)batch * kMixerOut * 4));
  act = static_cast<float*>(m->alloc((size_t)batch * c.inter * 4));
  logits = static_cast<float*>(m->alloc((size_t)batch * c.vocab * 4));
  argmax_scratch = m->alloc(argmax_scratch_bytes() * batch);
  cuda_check(cudaMemset(argmax_scratch, 0, argmax_scratch_bytes() * batch), "memset");
  attn_scratch = m->alloc(attention_scratch_bytes(batch));
  cuda_check(cudaMemset(attn_scratch, 0, attention_scratch_bytes(batch)), "memset");
}

Runner::~Runner() {
  for (auto& g : graph)
    if (g) cudaGraphExecDestroy(g);
  for (auto& g : fgraph)
    if (g) cudaGraphExecDestroy(g);
  for (auto& g : tgraph)
    if (g) cudaGraphExecDestroy(g);
}

Runner::LayerArgs Runner::layer_args(int i) const {
  const Model& M = *m;
  const LayerWeights& L = M.layers[i];
  LayerArgs r;
  r.attention = L.attention;
  GemvArgs& in = r.in;
  in.m = L.in;
  in.epi = kStore;
  in.y = proj;
  in.norm_w = L.input_norm;
  if (i == 0) {
    in.pro = kProEmbedNorm;
    in.embed = M.embed;
    in.ctl = st.ctl;
    in.h_out = h;
  } else {
    in.pro = kProRmsNorm;
    in.x = h;
  }
  GemvArgs& out = r.out;
  out.m = L.out;
  out.epi = kAccumulate;
  out.y = h;
  out.x = raw;
  if (L.attention) {
    AttnArgs& at = r.at;
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
    at.batch = 1;
    at.scratch = attn_scratch;
    out.pro = kProCopy;
  } else {
    r.gdn = dev::GdnArgs{proj, st.conv[i], L.conv_w, st.rec[i], L.gdn_params, &st.ctl->count, 4, raw};
    out.pro = kProGdnGate;
    out.zgate = proj + 6144;
    out.norm_w = L.gdn_params + 32;
  }
  GemvArgs& gu = r.gate_up;
  gu.m = L.gate_up;
  gu.pro = kProRmsNorm;
  gu.x = h;
  gu.norm_w = L.post_norm;
  gu.epi = kSwiGlu;
  gu.y = act;
  GemvArgs& dn = r.down;
  dn.m = L.down;
  dn.pro = kProCopy;
  dn.x = act;
  dn.epi = kAccumulate;
  dn.y = h;
  for (GemvArgs* g : {&r.in, &r.out, &r.gate_up, &r.down}) g->err = &st.ctl->flags;
  return r;
}

GemvArgs Runner::head_args(Variant v) const {
  const Model& M = *m;
  GemvArgs hd;
  hd.m = M.lm_head;
  hd.pro = kProRmsNorm;
  hd.x = h;
  hd.norm_w = M.final_norm;
  hd.epi = kArgmax;
  hd.y = logits;
  argmax_scratch_carve(argmax_scratch, &hd.part_val, &hd.part_idx, &hd.ticket);
  hd.ctl = st.ctl;
  hd.update_token = (v == kGreedy) ? 1 : 0;
  hd.err = &st.ctl->flags;
  return hd;
}

// Dispatch label in the reference's form (kernels/src/lib.rs:337: gemv_<rows>x<k>_<epilogue>).
static std::string gemv_label(const GemvArgs& a) {
  static const char* epi[] = {"Store", "Accumulate", "SwiGlu", "Argmax"};
  return "gemv_" + std::to_string(a.m.rows) + "x" + std::to_string(a.m.k) + "_" + epi[a.epi & 3];
}

void Runner::record(Variant v, cudaStream_t s, const std::function<void(const std::string&)>* after) {
  const Model& M = *m;
  const bool pdl = after == nullptr;
  size_t n = 0;
  auto gemv = [&](const GemvArgs& a) {
    if (const char* why = check_gemv(a)) throw QneError(kEInval, why);
    cuda_check(launch_gemv(a, s, pdl), "gemv launch");
    ++n;
    if (after) (*after)(gemv_label(a));
  };
  for (int i = 0; i < M.cfg.layers; ++i) {
    const LayerArgs r = layer_args(i);
    gemv(r.in);
    if (r.attention) {
      cuda_check(launch_attention(r.at, st.pool_pages, 64, s, pdl), "attention launch");
    } else {
      const dev::GdnArgs& g = r.gdn;
      cuda_check(launch_gdn_step(g.proj, g.conv, g.conv_w, g.state, g.params, g.counter, g.counter_stride, g.out,
                                 1, s, pdl),
                 "gdn launch");
    }
    ++n;
    if (after) (*after)(r.attention ? "attention" : "gdn");
    gemv(r.out);
    gemv(r.gate_up);
    gemv(r.down);
  }
  if (v != kLayers) gemv(head_args(v));
  if (v == kGreedy && !after) launches_per_token = n;
}

// Whether the fused layer kernels can run this model: one sequence, f16 GEMV weights with
// k % 256 == 0 (the register-streaming pipeline's segments), and a co-resident grid large
// enough for one CTA per mixer work item.
bool Runner::fused_supported() {
  const Model& M = *m;
  if (st.batch != 1 || M.cfg.layers < 1) return false;
  auto ok = [](const Mat& x) { return x.kind == kF16 && x.k % 256 == 0 && x.k <= 16384; };
  int max_k = M.lm_head.k;
  if (!ok(M.lm_head) || M.embed.k != M.layers[0].in.k) return false;
  for (const LayerWeights& L : M.layers) {
    for (const Mat* x : {&L.in, &L.out, &L.gate_up, &L.down}) {
      if (!ok(*x)) return false;
      max_k = std::max(max_k, x->k);
    }
  }
  fused_max_k = max_k;
  fused_ctas = persist_ctas(max_k);
  return fused_ctas > 0;
}

void Runner::record_fused(Variant v, cudaStream_t s) {
  const Model& M = *m;
  std::vector<LayerLaunch> launches(M.cfg.layers);
  for (int i = 0; i < M.cfg.layers; ++i) {
    const LayerArgs r = layer_args(i);
    LayerLaunch& la = launches[i];
    la.g[kPhIn] = r.in;
    la.g[kPhOut] = r.out;
    la.g[kPhGateUp] = r.gate_up;
    la.g[kPhDown] = r.down;
    const bool head = (i + 1 == M.cfg.layers) && v != kLayers;
    if (head) la.g[kPhHead] = head_args(v);
    for (int ph : {(int)kPhIn, (int)kPhOut, (int)kPhGateUp, (int)kPhDown})
      if (const char* why = check_gemv(la.g[ph])) throw QneError(kEInval, why);
    if (head)
      if (const char* why = check_gemv(la.g[kPhHead])) throw QneError(kEInval, why);
    la.attn.a = r.at;
    la.attn.split = dev::kSub;
    la.attn.max_splits = dev::kMaxSplits;
    la.attn.pool_pages = st.pool_pages;
    la.gdn = r.gdn;
    la.barrier = reinterpret_cast<unsigned long long*>(barrier);
    la.err = &st.ctl->flags;
    la.trace = trace_on ? trace + (size_t)i * fused_ctas * 32 : nullptr;
    la.xs_bytes = (uint32_t)persist_xs_bytes(fused_max_k);
    la.wait_limit_ns = wait_test_ns ? wait_test_ns : kBarrierLimitNs;
    la.wait_extra = wait_test_ns ? 1u : 0u;
  }
  for (int i = 0; i < M.cfg.layers; ++i) {
    const bool head = (i + 1 == M.cfg.layers) && v != kLayers;
    cuda_check(launch_layer(launches[i], M.layers[i].attention, head, fused_ctas, fused_max_k, s, true),
               "fused layer launch");
  }
  if (v == kGreedy) fused_launches_per_token = (size_t)M.cfg.layers;
}

void Runner::capture_set(cudaGraphExec_t* out, bool fused) {
  cudaStream_t cs;
  cuda_check(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "cudaStreamCreate");
  for (int v = 0; v < kVariants; ++v) {
    cuda_check(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
      if (fused) record_fused((Variant)v, cs);
      else record((Variant)v, cs);
    } catch (...) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(cs, &g);
      if (g) cudaGraphDestroy(g);
      cudaStreamDestroy(cs);
      throw;
    }
    cudaGraph_t g = nullptr;
    cuda_check(cudaStreamEndCapture(cs, &g), "end capture");
    cudaError_t e = cudaGraphInstantiate(&out[v], g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      cudaStreamDestroy(cs);
      cuda_check(e, "graph instantiate");
    }
  }
  cudaStreamDestroy(cs);
}

// Whether the token kernel can run this model: one sequence, f16 matrices whose shapes the ring
// slots take (k a multiple of 256 up to 6144), the GDN gated norm on 2048-wide outputs, and a
// device with a co-resident CTA per SM.
bool Runner::token_supported() {
  const Model& M = *m;
  if (st.batch != 1 || M.cfg.layers < 1) return false;
  if (M.lm_head.kind != kF16 || !token_gemv_ok(M.lm_head.rows, M.lm_head.k, kArgmax)) return false;
  if (M.embed.k != M.layers[0].in.k) return false;
  for (const LayerWeights& L : M.layers) {
    if (L.in.kind != kF16 || L.out.kind != kF16 || L.gate_up.kind != kF16 || L.down.kind != kF16) return false;
    if (!token_gemv_ok(L.in.rows, L.in.k, kStore) || !token_gemv_ok(L.out.rows, L.out.k, kAccumulate) ||
        !token_gemv_ok(L.gate_up.rows, L.gate_up.k, kSwiGlu) || !token_gemv_ok(L.down.rows, L.down.k, kAccumulate))
      return false;
    if (L.out.k != kMixerOut) return false;
  }
  token_ctas = qne::token_ctas();
  return token_ctas > 0;
}

// The token's phases in launch order (kernels/src/model.rs:220-269), with the same buffers and
// prologues / epilogues as the per-operation graph, cut into launches at the attention mixers.
std::vector<TkPhase> Runner::token_phase_list(Variant v, std::vector<TokenSeg>& segs) const {
  std::vector<TkPhase> ph;
  segs.clear();
  segs.push_back(TokenSeg{});
  auto gemv = [&](const GemvArgs& a) {
    TkPhase p;
    p.kind = kTkGemv;
    p.pro = a.pro;
    p.epi = a.epi;
    p.rows = a.m.rows;
    p.k = a.m.k;
    p.w = static_cast<const uint16_t*>(a.m.w);
    p.x = a.x;
    p.y = a.y;
    p.norm_w = a.norm_w;
    p.zgate = a.zgate;
    ph.push_back(p);
  };
  for (int i = 0; i < m->cfg.layers; ++i) {
    const LayerArgs r = layer_args(i);
    gemv(r.in);
    if (r.attention) {
      segs.back().count = (int)ph.size() - segs.back().first;
      segs.back().attn_layer = i;
      TokenSeg next;
      next.first = (int)ph.size();
      segs.push_back(next);
    } else {
      TkPhase mix;
      mix.kind = kTkGdn;
      mix.gdn = r.gdn;
      ph.push_back(mix);
    }
    gemv(r.out);
    gemv(r.gate_up);
    gemv(r.down);
  }
  if (v != kLayers) gemv(head_args(v));
  segs.back().count = (int)ph.size() - segs.back().first;
  return ph;
}

TkArgs Runner::token_args(Variant v, const TokenSeg& seg) const {
  TkArgs a;
  a.phases = token_phases[v] + seg.first;
  a.nphases = seg.count;
  a.ctl = st.ctl;
  a.embed = m->embed;
  a.h_out = h;
  argmax_scratch_carve(argmax_scratch, &a.part_val, &a.part_idx, &a.ticket);
  a.update_token = v == kGreedy ? 1 : 0;
  a.barrier = reinterpret_cast<unsigned long long*>(barrier);
  a.err = &st.ctl->flags;
  a.wait_limit_ns = wait_test_ns ? wait_test_ns : kBarrierLimitNs;
  a.wait_extra = wait_test_ns ? 1u : 0u;
  return a;
}

// Uploads the phase lists once and captures one graph per variant: the token-kernel launches and,
// between them, the attention kernels, chained by programmatic dependent launch.
void Runner::capture_token() {
  for (int v = 0; v < kVariants; ++v) {
    const std::vector<TkPhase> list = token_phase_list((Variant)v, token_segs[v]);
    if (!token_phases[v]) token_phases[v] = static_cast<TkPhase*>(m->alloc(list.size() * sizeof(TkPhase)));
    cuda_check(cudaMemcpy(token_phases[v], list.data(), list.size() * sizeof(TkPhase), cudaMemcpyHostToDevice),
               "token phases");
  }
  cudaStream_t cs;
  cuda_check(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "cudaStreamCreate");
  for (int v = 0; v < kVariants; ++v) {
    if (tgraph[v]) {
      cudaGraphExecDestroy(tgraph[v]);
      tgraph[v] = nullptr;
    }
    cuda_check(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "begin capture");
    cudaError_t le = cudaSuccess;
    size_t launches = 0;
    for (const TokenSeg& seg : token_segs[v]) {
      if (le == cudaSuccess && seg.count > 0) {
        le = launch_token(token_args((Variant)v, seg), token_ctas, cs, true);
        ++launches;
      }
      if (le == cudaSuccess && seg.attn_layer >= 0) {
        le = launch_attention(layer_args(seg.attn_layer).at, st.pool_pages, 64, cs, true);
        ++launches;
      }
    }
    token_launches[v] = launches;
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(cs, &g);
    cudaError_t ie = cudaSuccess;
    if (le == cudaSuccess && ce == cudaSuccess) ie = cudaGraphInstantiate(&tgraph[v], g, 0);
    if (g) cudaGraphDestroy(g);
    if (le != cudaSuccess || ce != cudaSuccess || ie != cudaSuccess) {
      cudaStreamDestroy(cs);
      cuda_check(le != cudaSuccess ? le : ce != cudaSuccess ? ce : ie, "token graph");
    }
  }
  cudaStreamDestroy(cs);
}

// The launch paths are captured once; the per-operation graphs are the default until
// set_path chooses another.
void Runner::capture_graphs() {
  capture_set(graph, false);
  use_fused = false;
  path = kPathOps;
  if (token_supported()) {
    try {
      capture_token();
    } catch (const QneError&) {
      for (auto& g : tgraph)
        if (g) {
          cudaGraphExecDestroy(g);
          g = nullptr;
        }
      token_ctas = 0;
    }
  }
  if (fused_supported()) {
    try {
      capture_set(fgraph, true);
    } catch (const QneError&) {
      // A device that cannot co-schedule the grid lands here; the per-operation graphs remain.
      for (auto& g : fgraph)
        if (g) {
          cudaGraphExecDestroy(g);
          g = nullptr;
        }
      fused_ctas = 0;
    }
  }
}

bool Runner::set_fused(bool on) { return set_path(on ? kPathLayers : kPathOps); }

bool Runner::set_path(int p) {
  if (p == kPathLayers && !fgraph[0]) return false;
  if (p == kPathToken && !tgraph[0]) return false;
  if (p < kPathOps || p > kPathToken) return false;
  path = p;
  use_fused = p == kPathLayers;
  return true;
}

bool Runner::set_trace(bool on) {
  if (!fgraph[0]) return false;
  if (on == trace_on) return true;
  if (on && !trace) trace = static_cast<unsigned long long*>(m->alloc((size_t)m->cfg.layers * fused_ctas * 32 * 8));
  if (on) cuda_check(cudaMemset(trace, 0, (size_t)m->cfg.layers * fused_ctas * 32 * 8), "trace");
  trace_on = on;
  for (auto& g : fgraph)
    if (g) {
      cudaGraphExecDestroy(g);
      g = nullptr;
    }
  capture_set(fgraph, true);
  return true;
}

bool Runner::set_wait_test(uint64_t limit_ns) {
  if (!fgraph[0] && !tgraph[0]) return false;
  if (limit_ns == wait_test_ns) return true;
  wait_test_ns = limit_ns;
  if (fgraph[0]) {
    for (auto& g : fgraph)
      if (g) {
        cudaGraphExecDestroy(g);
        g = nullptr;
      }
    capture_set(fgraph, true);
  }
  if (tgraph[0]) capture_token();
  return true;
}

size_t Runner::per_token() const {
  return path == kPathToken ? token_launches[kGreedy] : use_fused ? fused_launches_per_token : launches_per_token;
}

void Runner::launch(Variant v, cudaStream_t s) {
  cuda_check(cudaGraphLaunch(path == kPathToken ? tgraph[v] : use_fused ? fgraph[v] : graph[v], s), "graph launch");
  const size_t n = path == kPathToken ? token_launches[v]
                   : use_fused        ? fused_launches_per_token
                                      : (v == kLayers ? launches_per_token - 1 : launches_per_token);
  for (size_t i = 0; i < n; ++i) count_launch();
}

void Runner::reset(cudaStream_t s) {
  for (auto& b : st.buffers) cuda_check(cudaMemsetAsync(b.first, 0, b.second, s), "reset");
}

void Runner::snapshot(cudaStream_t s) {
  if (saved.empty())
    for (auto& b : st.buffers) saved.push_back({m->alloc(b.second), b.second});
  for (size_t i = 0; i < st.buffers.size(); ++i)
    cuda_check(cudaMemcpyAsync(saved[i].first, st.buffers[i].first, st.buffers[i].second,
                               cudaMemcpyDeviceToDevice, s),
               "snapshot");
  has_snapshot = true;
}

void Runner::restore(cudaStream_t s) {
  if (!has_snapshot) throw QneError(kENoSnap, "no snapshot taken");
  for (size_t i = 0; i < st.buffers.size(); ++i)
    cuda_check(cudaMemcpyAsync(st.buffers[i].first, saved[i].first, st.buffers[i].second,
                               cudaMemcpyDeviceToDevice, s),
               "restore");
}

// ------------------------------------------------------------------------------------------
// Model API
// ------------------------------------------------------------------------------------------
void Model::set_stream(cudaStream_t s) { ext_stream_ = s; }

bool Model::set_fused(bool on) {
  DeviceGuard g(device);
  cuda_check(cudaStreamSynchronize(stream()), "set_fused");
  return single_->set_fused(on);
}

bool Model::fused() const { return single_->use_fused; }

bool Model::set_path(int p) {
  DeviceGuard g(device);
  cuda_check(cudaStreamSynchronize(stream()), "set_path");
  return single_->set_path(p);
}

int Model::path() const { return single_->path; }

void Model::set_phase_trace(bool on) {
  DeviceGuard g(device);
  cuda_check(cudaStreamSynchronize(stream()), "set_phase_trace");
  if (!single_->set_trace(on)) throw QneError(kEInval, "the phase trace needs the fused layer kernels");
}

// Model::profile_token (kernels/src/model.rs:305-307; Gpu::profile, kernels/src/lib.rs:366-396):
// consumes one greedy token. Its kernels are launched one by one on the model's stream, without
// programmatic dependent launch (so no kernel overlaps its neighbours), with a CUDA event behind
// each; the time between consecutive events is summed per dispatch label. Diagnostic only: the
// graphs that decode() replays overlap consecutive kernels and take less time in total.
std::vector<std::pair<std::string, std::pair<double, uint32_t>>> Model::profile_token() {
  DeviceGuard g(device);
  cudaStream_t s = stream();
  if (host_pos_ >= (uint32_t)kMaxContext)
    throw QneError(kERangeCtx, "context limit of " + std::to_string(kMaxContext) + " tokens reached");
  cuda_check(cudaStreamSynchronize(s), "profile_token");
  std::vector<cudaEvent_t> ev;
  std::vector<std::string> labels;
  auto event = [&]() {
    cudaEvent_t e = nullptr;
    cuda_check(cudaEventCreate(&e), "cudaEventCreate");
    ev.push_back(e);
    cuda_check(cudaEventRecord(e, s), "cudaEventRecord");
  };
  std::vector<std::pair<std::string, std::pair<double, uint32_t>>> out;
  try {
    event();
    std::function<void(const std::string&)> after = [&](const std::string& label) {
      event();
      labels.push_back(label);
    };
    single_->record(Runner::kGreedy, s, &after);
    sync(600000);
    std::map<std::string, std::pair<double, uint32_t>> acc;
    for (size_t i = 0; i < labels.size(); ++i) {
      float ms = 0.f;
      cuda_check(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]), "cudaEventElapsedTime");
      auto& slot = acc[labels[i]];
      slot.first += ms;
      slot.second += 1;
    }
    out.assign(acc.begin(), acc.end());
  } catch (...) {
    for (cudaEvent_t e : ev) cudaEventDestroy(e);
    throw;
  }
  for (cudaEvent_t e : ev) cudaEventDestroy(e);
  ++host_pos_;
  uint32_t tok = 0, pos = 0;
  last_token(&tok, &pos);  // reports a timed-out wait like decode() does
  return out;
}

void Model::set_wait_test(uint64_t limit_ns) {
  DeviceGuard g(device);
  cuda_check(cudaStreamSynchronize(stream()), "set_wait_test");
  if (!single_->set_wait_test(limit_ns)) throw QneError(kEInval, "the barrier test needs the fused layer kernels");
}

size_t Model::read_phase_trace(uint64_t* out, size_t cap, size_t* ctas) {
  DeviceGuard g(device);
  if (!single_->trace_on) throw QneError(kEInval, "the phase trace is off");
  const size_t n = std::min(cap, (size_t)cfg.layers * single_->fused_ctas * 32);
  if (ctas) *ctas = (size_t)single_->fused_ctas;
  cuda_check(cudaStreamSynchronize(stream()), "read_phase_trace");
  if (out && n) cuda_check(cudaMemcpy(out, single_->trace, n * 8, cudaMemcpyDeviceToHost), "read_phase_trace");
  return n;
}

// A bounded device wait that gave up leaves kFlagTimeout in the control words; the barrier
// words may then be out of step, so they are cleared with the flag before the error surfaces.
void Model::check_flags(uint32_t flags) {
  if (!(flags & kFlagTimeout)) return;
  cuda_check(cudaMemsetAsync(single_->barrier, 0, 64, stream()), "clear barrier");
  cuda_check(cudaMemsetAsync(single_->attn_scratch, 0, attention_scratch_bytes(1), stream()), "clear attention tickets");
  cuda_check(cudaMemsetAsync(&single_->st.ctl->flags, 0, 4, stream()), "clear flags");
  cuda_check(cudaStreamSynchronize(stream()), "clear flags");
  throw QneError(kETimeout, "a device-side wait timed out; the token's results are invalid");
}

size_t Model::dispatches_per_token() const { return single_->per_token(); }
const float* Model::logits_device() const { return single_->logits; }

void Model::reset() {
  DeviceGuard g(device);
  single_->reset(stream());
  host_pos_ = 0;
}

bool Model::prefill_batched_supported() const { return PrefillRunner::supported(*this); }

void Model::prefill_chunk(const uint32_t* ids, uint32_t n, uint32_t start, bool finish, bool batched) {
  DeviceGuard g(device);
  if (!ids && n) throw QneError(kEInval, "null ids");
  if (n == 0 || (uint64_t)start + n >= (uint64_t)kMaxContext)
    throw QneError(kERangeCtx, "context limit: " + std::to_string(start) + " + " + std::to_string(n) +
                                   " tokens does not fit in " + std::to_string(kMaxContext));
  cuda_check(cudaStreamSynchronize(stream()), "prefill");  // host staging may still feed a copy
  if (batched && prefill_batched_supported()) {
    if (!prefill_) prefill_.reset(new PrefillRunner(this, single_.get()));
    prefill_->run(ids, n, start, finish, stream());
    host_pos_ = finish ? start + n : start + n - 1;
    sync(600000);
    return;
  }
  for (uint32_t i = 0; i < n; ++i) {
    host_ctl_[2 * i] = ids[i];
    host_ctl_[2 * i + 1] = start + i;
  }
  for (uint32_t i = 0; i < n; ++i) {
    cuda_check(cudaMemcpyAsync(single_->st.ctl, host_ctl_ + 2 * i, 8, cudaMemcpyHostToDevice, stream()),
               "prefill token");
    single_->launch((i + 1 == n && finish) ? Runner::kGreedy : Runner::kLayers, stream());
  }
  host_pos_ = finish ? start + n : start + n - 1;
  sync(600000);
}

void Model::logits(float* out, size_t n) {
  DeviceGuard g(device);
  if (!out || n < (size_t)cfg.vocab) throw QneError(kEInval, "logits buffer shorter than the vocabulary");
  cuda_check(cudaMemcpyAsync(out, single_->logits, (size_t)cfg.vocab * 4, cudaMemcpyDeviceToHost, stream()),
             "logits");
  sync(600000);
}

void Model::step_async(uint32_t token, uint32_t pos) {
  if (pos >= (uint32_t)kMaxContext)
    throw QneError(kERangeCtx, "context limit of " + std::to_string(kMaxContext) + " tokens reached");
  cuda_check(cudaStreamSynchronize(stream()), "step");
  host_ctl_[0] = token;
  host_ctl_[1] = pos;
  cuda_check(cudaMemcpyAsync(single_->st.ctl, host_ctl_, 8, cudaMemcpyHostToDevice, stream()), "step token");
  single_->launch(Runner::kStep, stream());
  host_pos_ = pos;
}

void Model::step(uint32_t token, uint32_t pos, float* out, size_t n) {
  DeviceGuard g(device);
  if (!out || n < (size_t)cfg.vocab) throw QneError(kEInval, "logits buffer shorter than the vocabulary");
  step_async(token, pos);
  cuda_check(cudaMemcpyAsync(out, single_->logits, (size_t)cfg.vocab * 4, cudaMemcpyDeviceToHost, stream()),
             "step logits");
  sync(600000);
}

void Model::snapshot() {
  DeviceGuard g(device);
  single_->snapshot(stream());
  saved_pos_ = host_pos_;
}

void Model::restore() {
  DeviceGuard g(device);
  single_->restore(stream());
  host_pos_ = saved_pos_;
}

void Model::last_token(uint32_t* token, uint32_t* pos) {
  DeviceGuard g(device);
  cuda_check(cudaStreamSynchronize(stream()), "last_token");
  cuda_check(cudaMemcpyAsync(host_ctl_ + 2 * kMaxContext, single_->st.ctl, 16, cudaMemcpyDeviceToHost, stream()),
             "last_token");
  sync(600000);
  check_flags(host_ctl_[2 * kMaxContext + 3]);
  if (token) *token = host_ctl_[2 * kMaxContext];
  if (pos) *pos = host_ctl_[2 * kMaxContext + 1];
  host_pos_ = host_ctl_[2 * kMaxContext + 1];
}

void Model::decode(uint32_t n, uint32_t window, const uint32_t* stop, uint32_t nstop, uint32_t* ids,
                   uint32_t* n_out) {
  DeviceGuard g(device);
  if (!ids || n == 0) throw QneError(kEInval, "decode needs an output buffer of n >= 1 ids");
  if (window == 0) throw QneError(kEInval, "window must be >= 1");
  uint32_t first = 0, next_pos = 0;
  last_token(&first, &next_pos);
  uint32_t count = 0;
  ids[count++] = first;
  auto stopped = [&](uint32_t t) {
    for (uint32_t i = 0; i < nstop; ++i)
      if (stop[i] == t) return true;
    return false;
  };
  while (count < n && !stopped(ids[count - 1])) {
    const uint32_t steps = std::min(window, n - count);
    if ((uint64_t)next_pos + steps > (uint64_t)kMaxContext) {
      if (n_out) *n_out = count;
      throw QneError(kERangeCtx, "context limit of " + std::to_string(kMaxContext) + " tokens reached after " +
                                     std::to_string(count) + " generated tokens");
    }
    next_pos += steps;
    for (uint32_t s = 0; s < steps; ++s) single_->launch(Runner::kGreedy, stream());
    cuda_check(cudaMemcpyAsync(host_ctl_ + 2 * kMaxContext, single_->st.ctl, 16, cudaMemcpyDeviceToHost, stream()),
               "decode readback");
    sync(600000);
    check_flags(host_ctl_[2 * kMaxContext + 3]);
    if (steps == 1) ids[count++] = host_ctl_[2 * kMaxContext];
    else
      for (uint32_t s = 0; s < steps; ++s) ids[count++] = 0xFFFFFFFFu;
  }
  host_pos_ = next_pos;
  if (n_out) *n_out = count;
}

void Model::decode_async(uint32_t steps) {
  DeviceGuard g(device);
  if ((uint64_t)host_pos_ + steps > (uint64_t)kMaxContext)
    throw QneError(kERangeCtx, "context limit of " + std::to_string(kMaxContext) + " tokens reached");
  for (uint32_t s = 0; s < steps; ++s) single_->launch(Runner::kGreedy, stream());
  host_pos_ += steps;
}

void Model::sync(uint32_t timeout_ms) {
  DeviceGuard g(device);
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  uint32_t spins = 0;
  for (;;) {
    const cudaError_t e = cudaStreamQuery(stream());
    if (e == cudaSuccess) return;
    if (e != cudaErrorNotReady) cuda_check(e, "stream");
    const auto now = std::chrono::steady_clock::now();
    if (now > deadline) throw QneError(kETimeout, "GPU wait exceeded " + std::to_string(timeout_ms) + " ms");
    if (++spins < 20000) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace qne
