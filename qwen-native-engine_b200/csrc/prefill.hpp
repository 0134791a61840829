// Batched prompt processing for the B = 1 sequence: chunks of up to 64 consecutive tokens per
// pass through tensor-core GEMMs (Model::prefill_chunk, kernels/src/model.rs:349-372).
#pragma once

#include <cuda_runtime.h>

#include <map>

#include "model.hpp"

namespace qne {

class PrefillRunner {
 public:
  static constexpr int kRows = 64;  // tokens per chunk (the tensor-core GEMM's batch limit)

  // Whether `m` can run chunks: decoder matrices f16 (the batched GEMM's operand) or int4 (block
  // 32 or group 64, decoded to f16 per matrix before its GEMM), k a multiple of 64.
  static bool supported(const Model& m);

  PrefillRunner(Model* m, Runner* single);
  ~PrefillRunner();

  // Enqueues ids[0..n) at positions start.. on stream s, `kRows` tokens per chunk, on the state
  // of `single`. Afterwards the control words hold (ids[n-1], start + n - 1) and the token
  // counter has advanced by n; with `finish` the LM head then runs on the last token, leaving
  // its logits and (greedy pick, start + n) as the per-token path does. The caller synchronizes
  // before reusing `ids`' staging (one pinned row array per runner).
  void run(const uint32_t* ids, uint32_t n, uint32_t start, bool finish, cudaStream_t s);

  size_t launches_per_chunk(int n) const;

 private:
  void record(int n, cudaStream_t s);
  cudaGraphExec_t graph_for(int n);

  Model* m;
  Runner* r;
  int ldx0 = 0;
  float* h = nullptr;     // [kRows][hidden] residual stream of the chunk
  float* proj = nullptr;  // [kRows][8224] mixer_in output
  float* raw = nullptr;   // [kRows][2048] mixer output before mixer_out
  uint16_t *x0h = nullptr, *x0l = nullptr, *x1h = nullptr, *x1l = nullptr;  // GEMM operand planes
  uint16_t *xnh = nullptr, *xnl = nullptr;  // planes of h * norm weight (RMSNorm folded into the GEMMs)
  float* sumsq = nullptr;                   // [hidden / 16][kGemmMaxRows] partial sums of h^2
  SeqCtl* rows = nullptr;    // [kRows] device: (token, position) of each chunk row
  SeqCtl* pinned = nullptr;  // [kMaxContext] host staging of the rows of one call
  void* attn_scratch = nullptr;
  float* conv_tail = nullptr;  // [3][6144] last conv inputs of a chunk, from the GDN scan to the prep
  uint16_t* wdeq = nullptr;    // int4 models: f16 copy of the decoder matrix the next GEMM reads
  std::map<int, cudaGraphExec_t> graphs;
  std::map<int, size_t> launches;
};

}  // namespace qne
