// Host-side interface of the GEMV / GEMM launchers shared by the runtime and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace qne {

struct Mat {
  int kind = kF16;
  int rows = 0;  // physical rows
  int k = 0;
  const void* w = nullptr;
  const void* s = nullptr;
  const void* z = nullptr;
};

// Everything one B=1 GEMV launch may use; unused fields stay null.
struct GemvArgs {
  Mat m;
  int pro = kProCopy;
  int epi = kStore;
  const float* x = nullptr;      // input vector (copy / rmsnorm / gdn-gate prologues)
  float* y = nullptr;            // output (logits for kArgmax)
  const float* norm_w = nullptr; // rmsnorm weight (kProRmsNorm, kProEmbedNorm) or GDN norm weight
  float eps = 1e-6f;
  const float* zgate = nullptr;  // kProGdnGate: z vector [2048]
  Mat embed;                     // kProEmbedNorm: embedding matrix
  SeqCtl* ctl = nullptr;         // kProEmbedNorm (token, count) / kArgmax (token, pos)
  float* h_out = nullptr;        // kProEmbedNorm: receives the embedding row
  float* part_val = nullptr;     // kArgmax scratch: per-CTA best value
  uint32_t* part_idx = nullptr;  // kArgmax scratch: per-CTA best index
  uint32_t* ticket = nullptr;    // kArgmax scratch: CTA completion counter (starts at 0)
  int update_token = 0;          // kArgmax: write the pick to ctl->token and advance ctl->pos
  uint32_t* err = nullptr;       // optional: receives kFlagTimeout if a bounded wait gives up
  int variant = 0;               // 0 auto, 1 register-streamed loads, 2 bulk-copy (TMA) ring
  int ctas_per_sm = 2;           // register-streamed kernel: CTAs per SM in the grid (1 or 2)
  int row_groups = 1;            // set by the launcher (tensor-core int4 kernel)
};

// Bytes of scratch the kArgmax epilogue needs.
size_t argmax_scratch_bytes();
void argmax_scratch_carve(void* scratch, float** part_val, uint32_t** part_idx, uint32_t** ticket);

// Validates shapes (k multiple of 256 for f16, of 1024 for int4 is not required: int4 needs
// k % 64 == 0 and the block-32 layout k % 256 == 0) and launches. pdl = launch with
// programmatic stream serialization (the kernel waits on its predecessor in-kernel).
cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl);
const char* check_gemv(const GemvArgs& a);  // nullptr if valid, else a message

cudaError_t launch_dequant_rows(const Mat& m, int row0, int nrows, float* out, cudaStream_t stream);
cudaError_t launch_argmax(const float* logits, uint32_t n, SeqCtl* ctl, void* scratch,
                          cudaStream_t stream, bool pdl);
uint64_t launches_issued();
void count_launch();

}  // namespace qne
