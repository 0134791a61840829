// Gated DeltaNet decode step (gdn, kernels/src/shaders.rs:445-520; CPU form
// kernels/src/lib.rs:578-628), for any number of independent sequences.
//
// Per head h: causal conv (kernel 4) + SiLU on the q, k, v channels; L2-normalized q (times
// 1/sqrt(128)) and k; decay g = exp(A * ln(1 + exp(a + dt_bias))), write strength
// beta = sigmoid(b); with the 128x128 f32 state S[key j][value t]:
//   sk[t] = sum_j S[j][t] k[j],  sq[t] = sum_j S[j][t] q[j],  dv[t] = beta (v[t] - g sk[t])
//   S[j][t] <- g S[j][t] + dv[t] k[j],  out[t] = g sq[t] + dv[t] (k . q).
//
// B200 layout: one CTA per (16-column slice, head, sequence), so one decode step spreads over
// 128 CTAs per sequence instead of 16. Each CTA recomputes q and k for its head (256 channels,
// L2-resident) and streams only its 8 KB slice of S. The convolution windows are a ring of the
// last four inputs per channel, indexed by the per-sequence token counter: this step's input
// goes to slot (count - 1) % 4, which no CTA of this step reads, so CTAs of one head never race
// on the window the way an in-place shift would.
//
// The gated RMSNorm of the output (kernels/src/shaders.rs:514-516) is applied by the consumer:
// the mixer_out GEMV prologue on the model path, or gdn_gate_kernel below.
#include <math.h>

#include "gdn.cuh"
#include "gdn_dev.cuh"
#include "gemv.cuh"

namespace qne {
namespace {

using namespace dev;

// kPre: the constant operands, the state slice and the conv window are loaded before the
// dependency wait (one sequence: 128 CTAs, one wave, latency-bound); with many sequences the kernel
// keeps the smaller register footprint (32 registers, so at least seven CTAs fit per SM), so more
// state slices are in flight per SM.
template <bool kPre>
__global__ void __launch_bounds__(256, kPre ? 1 : 7) gdn_step_kernel(const GdnArgs a) {
  __shared__ GdnShared sh;
  const int item = (blockIdx.z * kGdnHeads + blockIdx.y) * kSlices + blockIdx.x;
  GdnItem it;
  pdl_launch();
  // One sequence: the constants, the state slice and the conv window go to registers before the
  // wait (preload); with many sequences (register budget) the state slice is only warmed in L2
  // and read after the wait.
  if (kPre) it.preload(a, item);
  else it.warm_l2(a, item);
  pdl_wait();
  it.prefetch(a, item);
  it.run(a, sh);
}

// out = raw * rsqrt(mean_head(raw^2) + 1e-6) * silu(z) * norm_w, per 128-wide head.
__global__ void __launch_bounds__(128) gdn_gate_kernel(const float* raw, const float* proj,
                                                       const float* norm_w, float* out) {
  const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
  __shared__ float red[4];
  pdl_launch();
  pdl_wait();
  const float v = raw[(size_t)b * kMixerOut + h * kGdnDim + t];
  const float tot = block_sum<128>(v * v, red);
  const float inv = rsqrtf(tot / (float)kGdnDim + 1e-6f);
  const float z = proj[(size_t)b * kGdnProj + 6144 + h * kGdnDim + t];
  out[(size_t)b * kMixerOut + h * kGdnDim + t] = v * inv * silu(z) * norm_w[t];
}

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, cudaStream_t stream, bool pdl,
                            cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

}  // namespace

cudaError_t launch_gdn_step(const float* proj, float* conv, const float* conv_w, float* state,
                            const float* params, const uint32_t* counter, int counter_stride,
                            float* out_raw, int batch, cudaStream_t stream, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(dev::kSlices, kGdnHeads, batch), dim3(256), stream, pdl, attr);
  count_launch();
  const GdnArgs a{proj, conv, conv_w, state, params, counter, counter_stride, out_raw};
  return batch == 1 ? cudaLaunchKernelEx(&cfg, gdn_step_kernel<true>, a) : cudaLaunchKernelEx(&cfg, gdn_step_kernel<false>, a);
}

cudaError_t launch_gdn_gate(const float* raw, const float* proj, const float* norm_w, float* out,
                            int batch, cudaStream_t stream, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(kGdnHeads, batch), dim3(128), stream, pdl, attr);
  count_launch();
  return cudaLaunchKernelEx(&cfg, gdn_gate_kernel, raw, proj, norm_w, out);
}

}  // namespace qne
