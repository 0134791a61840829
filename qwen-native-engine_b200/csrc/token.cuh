// Host interface of the token kernel: one launch runs a stretch of a B = 1 decode token (the
// GEMVs and GDN mixers of the layers between two attention mixers, and the LM head) on one CTA
// per SM, with a bulk-copy producer warp per CTA streaming the stretch's weights through a
// shared-memory ring.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "attn_dev.cuh"
#include "common.cuh"
#include "gdn_dev.cuh"
#include "gemv.cuh"

namespace qne {

// Phase kinds, in launch order per layer: GEMV (in-projection), GDN (attention layers end a
// launch after their in-projection), GEMV (out-projection), GEMV (gate_up), GEMV (down); then the
// LM head GEMV with the greedy pick.
enum TkKind : int { kTkGemv = 0, kTkGdn = 1 };

struct TkPhase {
  int kind = kTkGemv;
  // GEMV: f16 matrix w [rows][k] (SwiGLU: gate rows, then up rows), prologue, epilogue.
  int pro = kProCopy, epi = kStore, rows = 0, k = 0;
  const uint16_t* w = nullptr;
  const float* x = nullptr;       // input vector (copy / RMSNorm / gated-norm prologues)
  float* y = nullptr;             // output (logits for kArgmax)
  const float* norm_w = nullptr;  // RMSNorm weight, or the GDN output norm weight
  const float* zgate = nullptr;   // kProGdnGate: z vector [2048]
  // GDN mixer.
  dev::GdnArgs gdn{};
};

struct TkArgs {
  const TkPhase* phases = nullptr;  // device array
  int nphases = 0;
  SeqCtl* ctl = nullptr;
  Mat embed;                        // layer-0 prologue: embedding row of ctl->token
  float* h_out = nullptr;           // receives the embedding row (the residual stream)
  float* part_val = nullptr;        // greedy pick: per-CTA best value / index, ticket
  uint32_t* part_idx = nullptr;
  uint32_t* ticket = nullptr;
  int update_token = 0;             // write the pick to ctl->token and advance ctl->pos
  unsigned long long* barrier = nullptr;  // [2] grid barrier arrivals / exits (zero between launches)
  uint32_t* err = nullptr;          // receives kFlagTimeout if a bounded wait gives up
  uint64_t wait_limit_ns = 0;       // one grid-barrier wait
  uint32_t wait_extra = 0;          // arrivals a barrier waits for beyond the grid (timeout test)
};

// CTAs of the token kernel on this device (one per SM), or 0 if it cannot run here.
int token_ctas();
// Whether a GEMV of this shape can run in the token kernel (f16, 16-byte rows, k <= 6144).
bool token_gemv_ok(int rows, int k, int epi);
cudaError_t launch_token(const TkArgs& args, int ctas, cudaStream_t stream, bool pdl);

}  // namespace qne
