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
#include "gemv.cuh"

namespace qne {
namespace {

constexpr int kSlice = 16;            // value columns per CTA

__device__ __forceinline__ float sel4(const float* r, int i) {
  return i == 0 ? r[0] : i == 1 ? r[1] : i == 2 ? r[2] : r[3];
}
constexpr int kSlices = kGdnDim / kSlice;  // 8

__global__ void __launch_bounds__(256) gdn_step_kernel(const float* __restrict__ proj, float* conv,
                                                       const float* __restrict__ conv_w,
                                                       float* state, const float* __restrict__ params,
                                                       const uint32_t* counter, int counter_stride,
                                                       float* out) {
  __shared__ float qs[kGdnDim];
  __shared__ float ks[kGdnDim];
  __shared__ float vs[kSlice];
  __shared__ float red[8];
  __shared__ float psk[16][kSlice];
  __shared__ float psq[16][kSlice];
  __shared__ float sk_s[kSlice], sq_s[kSlice];
  __shared__ float kq_s;

  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = s * kSlice;
  const int jg = tid >> 4, tl = tid & 15;  // state slice: column t0 + tl, rows jg*8 .. jg*8+7
  float* S = state + ((size_t)b * kGdnHeads + h) * kGdnDim * kGdnDim + t0 + tl;
  pdl_launch();
  // The state slice is not produced by the previous kernel: warm L2 with it while waiting
  // (a prefetch only moves lines closer; correctness never depends on it).
  if (tid < kGdnDim) asm volatile("prefetch.global.L2 [%0];" ::"l"(S - tl + (size_t)tid * kGdnDim));
  pdl_wait();

  // Issue every independent load at once: state slice, counter, proj, all four ring slots (the
  // slot this step overwrites is read too and discarded, which saves waiting for the counter).
  float sv[8];
#pragma unroll
  for (int jj = 0; jj < 8; ++jj) sv[jj] = S[(size_t)(jg * 8 + jj) * kGdnDim];
  const uint32_t cnt = counter[(size_t)b * counter_stride];
  const float* pr = proj + (size_t)b * kGdnProj;
  float* ring = conv + (size_t)b * kConvSlots * kConvChannels;
  const int i = tid & (kGdnDim - 1);
  const int ch = (tid < kGdnDim ? 0 : 2048) + h * kGdnDim + i;
  const float x = pr[ch];
  const float4 w = *reinterpret_cast<const float4*>(conv_w + (size_t)ch * 4);
  float rv[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) rv[r] = ring[r * kConvChannels + ch];
  float vx = 0.f, vrv[4] = {0.f, 0.f, 0.f, 0.f};
  float4 vw = make_float4(0.f, 0.f, 0.f, 0.f);
  const int cv = 4096 + h * kGdnDim + t0 + (tid & (kSlice - 1));
  if (tid < kSlice) {
    vx = pr[cv];
    vw = *reinterpret_cast<const float4*>(conv_w + (size_t)cv * 4);
#pragma unroll
    for (int r = 0; r < 4; ++r) vrv[r] = ring[r * kConvChannels + cv];
  }
  const int slot_new = (int)((cnt - 1u) & 3u);
  const int s2 = (int)((cnt - 2u) & 3u);  // previous input
  const int s1 = (int)((cnt - 3u) & 3u);
  const int s0 = (int)((cnt - 4u) & 3u);  // oldest input of the window

  // q (threads 0..127) and k (threads 128..255) channels of head h.
  float val;
  {
    const float y = sel4(rv, s0) * w.x + sel4(rv, s1) * w.y + sel4(rv, s2) * w.z + x * w.w;
    val = silu(y);
    if (i >= t0 && i < t0 + kSlice) ring[slot_new * kConvChannels + ch] = x;
  }
  if (tid < kSlice) {
    const float y = sel4(vrv, s0) * vw.x + sel4(vrv, s1) * vw.y + sel4(vrv, s2) * vw.z + vx * vw.w;
    vs[tid] = silu(y);
    ring[slot_new * kConvChannels + cv] = vx;
  }
  // L2 norms: warps 0-3 hold q, warps 4-7 hold k.
  const float ss = warp_sum(val * val);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  const float nq = rsqrtf(red[0] + red[1] + red[2] + red[3] + 1e-6f);
  const float nk = rsqrtf(red[4] + red[5] + red[6] + red[7] + 1e-6f);
  if (tid < kGdnDim) qs[i] = val * nq * 0.08838834764f;
  else ks[i] = val * nk;
  __syncthreads();
  if (warp < 4) {
    const float p = warp_sum(ks[tid] * qs[tid]);
    if (lane == 0) red[warp] = p;  // red[0..3] no longer needed for nq
  }
  // Decay and write strength.
  const float g = expf(params[16 + h] * logf(1.0f + expf(pr[8192 + h] + params[h])));
  const float beta = 1.0f / (1.0f + expf(-pr[8208 + h]));

  float sk = 0.f, sq = 0.f;
#pragma unroll
  for (int jj = 0; jj < 8; ++jj) {
    sk = fmaf(sv[jj], ks[jg * 8 + jj], sk);
    sq = fmaf(sv[jj], qs[jg * 8 + jj], sq);
  }
  psk[jg][tl] = sk;
  psq[jg][tl] = sq;
  __syncthreads();
  if (tid < kSlice) {
    float a = 0.f, c = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      a += psk[r][tid];
      c += psq[r][tid];
    }
    sk_s[tid] = a;
    sq_s[tid] = c;
  }
  if (tid == 0) kq_s = red[0] + red[1] + red[2] + red[3];
  __syncthreads();
  const float dv = beta * (vs[tl] - g * sk_s[tl]);
#pragma unroll
  for (int jj = 0; jj < 8; ++jj) S[(size_t)(jg * 8 + jj) * kGdnDim] = g * sv[jj] + dv * ks[jg * 8 + jj];
  if (jg == 0) out[(size_t)b * kMixerOut + h * kGdnDim + t0 + tl] = g * sq_s[tl] + dv * kq_s;
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
  cudaLaunchConfig_t cfg = make_cfg(dim3(kSlices, kGdnHeads, batch), dim3(256), stream, pdl, attr);
  count_launch();
  return cudaLaunchKernelEx(&cfg, gdn_step_kernel, proj, conv, conv_w, state, params, counter,
                            counter_stride, out_raw);
}

cudaError_t launch_gdn_gate(const float* raw, const float* proj, const float* norm_w, float* out,
                            int batch, cudaStream_t stream, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(kGdnHeads, batch), dim3(128), stream, pdl, attr);
  count_launch();
  return cudaLaunchKernelEx(&cfg, gdn_gate_kernel, raw, proj, norm_w, out);
}

}  // namespace qne
