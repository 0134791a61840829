// The decoder runtime behind the C ABI: weight loading and validation, device state, the
// per-token launch graph, and the Model API of kernels/src/model.rs.
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <stdexcept>
#include <functional>
#include <string>
#include <vector>

#include "common.cuh"
#include "gdn.cuh"
#include "gdn_dev.cuh"
#include "gemv.cuh"
#include "persist.cuh"
#include "token.cuh"

namespace qne {

struct QneError : std::runtime_error {
  int code;
  QneError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// Error codes (mirrors qne.h).
constexpr int kEInval = -1, kERangeCtx = -2, kEFormat = -3, kECuda = -4, kETimeout = -5,
              kENoSnap = -6, kENoMem = -7;

void cuda_check(cudaError_t e, const char* what);

// Makes `dev` current for the guard's lifetime (the previous device is restored).
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cuda_check(cudaSetDevice(dev), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

struct LayerWeights {
  bool attention = false;
  Mat in, out, gate_up, down;
  const float* input_norm = nullptr;
  const float* post_norm = nullptr;
  const float* attn_norms = nullptr;  // attention layers: q_norm[256], k_norm[256]
  const float* conv_w = nullptr;      // GDN layers: [6144][4]
  const float* gdn_params = nullptr;  // GDN layers: dt_bias[16], A_neg_exp[16], norm_w[128]
};

struct Config {
  int layers = 0, every = 4, hidden = 0, inter = 0, vocab = 0, rope_dim = 64;
  double theta = 1e7;
};

// Device state of `batch` sequences: GDN conv rings and recurrent states, KV page pools.
struct SeqState {
  int batch = 0;
  uint32_t pool_pages = 0;
  std::vector<float*> conv;      // per layer (GDN): [batch][4][6144]
  std::vector<float*> rec;       // per layer (GDN): [batch][16][128][128]
  std::vector<uint16_t*> kv;     // per layer (attention): [pool_pages][16384] halves
  SeqCtl* ctl = nullptr;         // [batch]
  uint32_t* page_table = nullptr;  // [batch][256]
  std::vector<std::pair<void*, size_t>> buffers;  // everything cleared by reset
};

class Model;

// Activations and launch graphs of one sequence set.
class Runner;
// Chunked prompt processing on the B = 1 sequence (prefill.cu).
class PrefillRunner;

class Model {
 public:
  // any_shape = false (the default of qne_model_load) accepts exactly the architectures the
  // reference's Index::validate accepts (kernels/src/model.rs:51-55); true also accepts other
  // layer counts, vocabularies and widths the kernels can run (qne_model_load_ex's
  // QNE_LOAD_ANY_SHAPE, used by small test models).
  static Model* load(const char* json, size_t json_len, const void* weights, size_t weights_len,
                     int device, bool any_shape = false);
  ~Model();

  Config cfg;
  int device = 0;
  int weight_kind = kF16, embed_kind = kF16;
  bool tied = false;
  uint64_t weight_bytes = 0;  // bytes one decode token reads from the weights
  uint64_t device_bytes = 0;
  std::string adapter;
  std::vector<LayerWeights> layers;
  Mat embed, lm_head;
  const float* final_norm = nullptr;
  float* rope = nullptr;  // [2][4096][32]

  // B = 1 API (kernels/src/model.rs)
  void reset();
  // batched: 32-token chunks through tensor-core GEMMs when the weights allow it (f16
  // matrices), else one token per step like `prefill` (kernels/src/model.rs:324-335).
  void prefill_chunk(const uint32_t* ids, uint32_t n, uint32_t start, bool finish_logits, bool batched = true);
  bool prefill_batched_supported() const;
  void logits(float* out, size_t n);
  void step(uint32_t token, uint32_t pos, float* out, size_t n);
  void step_async(uint32_t token, uint32_t pos);
  void snapshot();
  void restore();
  void last_token(uint32_t* token, uint32_t* pos);
  void decode(uint32_t n, uint32_t window, const uint32_t* stop, uint32_t nstop, uint32_t* ids,
              uint32_t* n_out);
  void decode_async(uint32_t steps);
  void sync(uint32_t timeout_ms);
  void set_stream(cudaStream_t s);
  bool set_fused(bool on);
  bool fused() const;
  bool set_path(int p);  // false if that path cannot run this model
  int path() const;
  void set_phase_trace(bool on);
  void set_wait_test(uint64_t limit_ns);
  // Model::profile_token: one greedy token, kernel by kernel, milliseconds per dispatch label.
  std::vector<std::pair<std::string, std::pair<double, uint32_t>>> profile_token();
  size_t read_phase_trace(uint64_t* out, size_t cap, size_t* ctas);
  size_t dispatches_per_token() const;
  const float* logits_device() const;

  cudaStream_t stream() const { return ext_stream_ ? ext_stream_ : own_stream_; }
  void* alloc(size_t bytes, bool track = true);  // device allocation owned by the model

  Runner* single() { return single_.get(); }

 private:
  Model() = default;
  void free_all();
  std::vector<void*> allocations_;
  void* arena_ = nullptr;
  cudaStream_t own_stream_ = nullptr;
  cudaStream_t ext_stream_ = nullptr;
  std::unique_ptr<Runner> single_;
  std::unique_ptr<PrefillRunner> prefill_;  // created by the first batched prefill
  uint32_t* host_ctl_ = nullptr;  // pinned staging: (token, pos) pairs
  uint32_t host_pos_ = 0;         // host mirror of the next position
  uint32_t saved_pos_ = 0;
  void check_flags(uint32_t flags);  // throws (and clears the barrier) after a device timeout
  friend class Runner;
};

// One set of sequences with its state, activations and captured graphs.
class Runner {
 public:
  Runner(Model* m, int batch, uint32_t pool_pages);
  ~Runner();
  Model* m;
  SeqState st;
  // activations
  float* h = nullptr;
  float* proj = nullptr;
  float* raw = nullptr;
  float* act = nullptr;
  float* logits = nullptr;
  void* argmax_scratch = nullptr;
  void* attn_scratch = nullptr;
  // snapshot copies (allocated on the first snapshot)
  std::vector<std::pair<void*, size_t>> saved;
  bool has_snapshot = false;

  uint32_t* barrier = nullptr;  // grid barrier words of the fused layer kernels
  bool trace_on = false;
  unsigned long long* trace = nullptr;  // fused path phase timestamps [layers][ctas][32]

  // Token graphs: kGreedy = layers + LM head + pick (the pick becomes the next token),
  // kStep = the same without advancing, kLayers = layers only (prefill).
  enum Variant { kGreedy = 0, kStep = 1, kLayers = 2, kVariants = 3 };
  cudaGraphExec_t graph[kVariants] = {nullptr, nullptr, nullptr};   // one kernel per op
  cudaGraphExec_t fgraph[kVariants] = {nullptr, nullptr, nullptr};  // one fused launch per layer
  cudaGraphExec_t tgraph[kVariants] = {nullptr, nullptr, nullptr};  // one token-kernel launch
  size_t launches_per_token = 0;
  size_t fused_launches_per_token = 0;
  // Launch path of a token: kPathOps (one kernel per operation), kPathLayers (one fused launch
  // per layer), kPathToken (one launch per token).
  enum Path { kPathOps = 0, kPathLayers = 1, kPathToken = 2 };
  int path = kPathOps;
  bool use_fused = false;  // path == kPathLayers
  int fused_ctas = 0, fused_max_k = 0;
  int token_ctas = 0;                            // 0: the token kernel cannot run this model
  TkPhase* token_phases[kVariants] = {nullptr, nullptr, nullptr};  // device phase lists
  size_t token_launches[kVariants] = {0, 0, 0};  // launches of one token, per variant
  // One token-kernel launch: phases [first, first + count) of the variant's list, followed by the
  // attention mixer of layer attn_layer (-1: none, the last launch of a token).
  struct TokenSeg {
    int first = 0, count = 0, attn_layer = -1;
  };
  std::vector<TokenSeg> token_segs[kVariants];
  bool token_supported();
  std::vector<TkPhase> token_phase_list(Variant v, std::vector<TokenSeg>& segs) const;
  TkArgs token_args(Variant v, const TokenSeg& seg) const;
  void capture_token();
  bool set_path(int p);

  struct LayerArgs {
    bool attention = false;
    GemvArgs in, out, gate_up, down;
    AttnArgs at;
    dev::GdnArgs gdn{};
  };
  LayerArgs layer_args(int i) const;
  GemvArgs head_args(Variant v) const;
  // Enqueues one token's kernels on s. With `after` set (profiling), the launches are plain
  // (no programmatic dependent launch) and after(label) runs behind each one.
  void record(Variant v, cudaStream_t s, const std::function<void(const std::string&)>* after = nullptr);
  void record_fused(Variant v, cudaStream_t s);  // the same as one fused launch per layer
  bool set_trace(bool on);
  // Test hook of the bounded grid-barrier waits: nonzero = every barrier of the fused kernels also
  // waits for one arrival that never comes, with this limit (ns), so every wait runs out.
  uint64_t wait_test_ns = 0;
  bool set_wait_test(uint64_t limit_ns);
  bool fused_supported();
  void capture_set(cudaGraphExec_t* out, bool fused);
  void capture_graphs();
  bool set_fused(bool on);  // false if the fused kernels are not available
  size_t per_token() const;
  void launch(Variant v, cudaStream_t s);
  void reset(cudaStream_t s);
  void snapshot(cudaStream_t s);
  void restore(cudaStream_t s);
};

}  // namespace qne
