// Host interface of the fused (one launch per decoder layer) decode kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "attn_dev.cuh"
#include "common.cuh"
#include "gdn_dev.cuh"
#include "gemv.cuh"

namespace qne {

// Phases of a fused layer launch, in order.
enum LayerPhase : int { kPhIn = 0, kPhMixer = 1, kPhOut = 2, kPhGateUp = 3, kPhDown = 4, kPhHead = 5, kPhases = 6 };

// Arguments of one fused layer launch, prepared on the host exactly as the per-kernel path
// passes them to its launches, and passed by value as a grid constant so that the kernel reads
// them through the constant cache (about 1.3 KB of the 32 KB parameter space).
struct LayerLaunch {
  GemvArgs g[kPhases];    // GEMV of each phase (kPhMixer unused; kPhHead: final norm + LM head +
                          // greedy pick, last layer of a token only)
  dev::KernelArgs attn;   // attention layers (one split of kSub tokens per work item)
  dev::GdnArgs gdn;       // GDN layers
  unsigned long long* barrier;  // [2] grid barrier arrivals and exits (zero between launches)
  uint32_t* err;          // receives kFlagTimeout if a barrier wait gives up
  unsigned long long* trace;  // optional phase timestamps ([ctas][32]); null when off
  uint32_t xs_bytes;          // dynamic shared memory before the ring / mixer region
  uint64_t wait_limit_ns;     // time limit of one grid-barrier wait (kBarrierLimitNs normally)
  uint32_t wait_extra;        // arrivals each barrier waits for beyond the grid: 0, or 1 in the
                              // timeout test, where no barrier can complete and every wait runs out
};

constexpr uint64_t kBarrierLimitNs = 2000000000ull;  // 2 s; a healthy barrier takes about a microsecond

// CTAs of a co-resident grid for the largest GEMV k of the model (0 if the kernels cannot run:
// the grid must hold at least one CTA per mixer work item).
int persist_ctas(int max_k);
size_t persist_xs_bytes(int max_k);
cudaError_t launch_layer(const LayerLaunch& args, bool attention, bool head, int ctas, int max_k,
                         cudaStream_t stream, bool pdl);

}  // namespace qne
