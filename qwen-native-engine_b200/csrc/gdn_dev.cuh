// Gated DeltaNet decode step, one work item = (16-column slice, head, sequence); shared by the
// per-kernel path (gdn.cu) and the persistent decode kernel. prefetch() reads only the
// recurrent state of this item (last written by the previous token), so callers issue it before
// waiting on the in-projection that produces proj.
#pragma once

#include "common.cuh"

namespace qne {
namespace dev {

constexpr int kSlice = 16;                 // value columns per item
constexpr int kSlices = kGdnDim / kSlice;  // 8
constexpr int kGdnItemsPerSeq = kSlices * kGdnHeads;  // 128

__device__ __forceinline__ float sel4(const float* r, int i) {
  return i == 0 ? r[0] : i == 1 ? r[1] : i == 2 ? r[2] : r[3];
}

struct GdnArgs {
  const float* proj;       // [batch][8224]
  float* conv;             // [batch][4][6144] ring
  const float* conv_w;     // [6144][4]
  float* state;            // [batch][16][128][128]
  const float* params;     // [160]
  const uint32_t* counter; // counter[b * counter_stride]: tokens processed including this one
  int counter_stride;
  float* out;              // [batch][2048] raw (before the gated norm)
};

struct GdnShared {
  float qs[kGdnDim];
  float ks[kGdnDim];
  float vs[kSlice];
  float red[8];
  float psk[16][kSlice];
  float psq[16][kSlice];
  float sk_s[kSlice], sq_s[kSlice];
  float kq_s;
};

struct GdnItem {
  int s, h, b, t0, jg, tl;
  float* S;
  float sv[8];
  // Operands that depend on nothing (conv weights of this thread's channels, the head's decay
  // parameters), loaded by preload() before the dependency wait; run_with loads them itself when
  // preload() was not called.
  bool pre = false;
  float4 cw, cvw;
  float pA, pDt;
  float rv[4], vrv[4];  // the conv window slots of this thread's channels (preload only)

  // L2 warm-up of the item's state rows: a hint only, safe before any dependency wait.
  __device__ __forceinline__ void warm_l2(const GdnArgs& a, int item) const {
    const int ss = item % kSlices, hh = (item / kSlices) % kGdnHeads, bb = item / kGdnItemsPerSeq;
    const float* base = a.state + ((size_t)bb * kGdnHeads + hh) * kGdnDim * kGdnDim + ss * kSlice;
    if (threadIdx.x < kGdnDim) asm volatile("prefetch.global.L2 [%0];" ::"l"(base + (size_t)threadIdx.x * kGdnDim));
  }

  // Constant operands, the item's state slice and its conv window slots into registers. The
  // state and the window were last written by this layer's step of an earlier token (an earlier
  // graph or stream launch; the slot this step overwrites is read too and discarded), so this is
  // safe before the dependency wait of a decode step. Not for prompt chunks.
  __device__ __forceinline__ void preload(const GdnArgs& a, int item) {
    geometry(a, item);
    const int tid = threadIdx.x;
    const int ch = (tid < kGdnDim ? 0 : 2048) + h * kGdnDim + (tid & (kGdnDim - 1));
    const int cv = 4096 + h * kGdnDim + s * kSlice + (tid & (kSlice - 1));
    cw = __ldg(reinterpret_cast<const float4*>(a.conv_w + (size_t)ch * 4));
    cvw = tid < kSlice ? __ldg(reinterpret_cast<const float4*>(a.conv_w + (size_t)cv * 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
    pA = __ldg(a.params + 16 + h);
    pDt = __ldg(a.params + h);
    const float* ring = a.conv + (size_t)b * kConvSlots * kConvChannels;
#pragma unroll
    for (int r = 0; r < kConvSlots; ++r) {
      rv[r] = ring[r * kConvChannels + ch];
      vrv[r] = tid < kSlice ? ring[r * kConvChannels + cv] : 0.f;
    }
    load_state();
    pre = true;
  }

  // Loads the item's state slice (after geometry) unless preload() did.
  __device__ __forceinline__ void prefetch(const GdnArgs& a, int item) {
    if (pre) return;
    geometry(a, item);
    load_state();
  }

  __device__ __forceinline__ void load_state() {
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) sv[jj] = S[(size_t)(jg * 8 + jj) * kGdnDim];
  }

  __device__ __forceinline__ void geometry(const GdnArgs& a, int item) {
    s = item % kSlices;
    h = (item / kSlices) % kGdnHeads;
    b = item / kGdnItemsPerSeq;
    const int tid = threadIdx.x;
    t0 = s * kSlice;
    jg = tid >> 4;
    tl = tid & 15;  // state slice: column t0 + tl, rows jg*8 .. jg*8+7
    S = a.state + ((size_t)b * kGdnHeads + h) * kGdnDim * kGdnDim + t0 + tl;
  }

  __device__ __forceinline__ void run(const GdnArgs& a, GdnShared& sh) { run_with(a, sh, BlockSync()); }

  // The item's 256 threads are threads 0..255 of the CTA; `sync` is a barrier over exactly those
  // (the whole CTA, or a named barrier when other warps of the CTA do other work).
  struct BlockSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
  };
  template <class Sync>
  __device__ __forceinline__ void run_with(const GdnArgs& a, GdnShared& sh, Sync sync) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // Issue every independent load at once: counter, proj, all four ring slots (the slot this
    // step overwrites is read too and discarded, which saves waiting for the counter).
    const uint32_t cnt = a.counter[(size_t)b * a.counter_stride];
    const float* pr = a.proj + (size_t)b * kGdnProj;
    float* ring = a.conv + (size_t)b * kConvSlots * kConvChannels;
    const int i = tid & (kGdnDim - 1);
    const int ch = (tid < kGdnDim ? 0 : 2048) + h * kGdnDim + i;
    const float x = pr[ch];
    // the decay and write-strength inputs of the head, with the other step inputs (one round trip)
    const float ga = pr[8192 + h], gb = pr[8208 + h];
    const float4 w = pre ? cw : *reinterpret_cast<const float4*>(a.conv_w + (size_t)ch * 4);
    if (!pre) {
#pragma unroll
      for (int r = 0; r < 4; ++r) rv[r] = ring[r * kConvChannels + ch];
    }
    float vx = 0.f;
    float4 vw = make_float4(0.f, 0.f, 0.f, 0.f);
    const int cv = 4096 + h * kGdnDim + t0 + (tid & (kSlice - 1));
    if (!pre) {
#pragma unroll
      for (int r = 0; r < 4; ++r) vrv[r] = 0.f;
    }
    if (tid < kSlice) {
      vx = pr[cv];
      vw = pre ? cvw : *reinterpret_cast<const float4*>(a.conv_w + (size_t)cv * 4);
      if (!pre) {
#pragma unroll
        for (int r = 0; r < 4; ++r) vrv[r] = ring[r * kConvChannels + cv];
      }
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
      sh.vs[tid] = silu(y);
      ring[slot_new * kConvChannels + cv] = vx;
    }
    // Decay and write strength (their transcendental latency overlaps the barriers below).
    const float pa = pre ? pA : a.params[16 + h], pd = pre ? pDt : a.params[h];
    const float g = expf(pa * logf(1.0f + expf(ga + pd)));
    const float beta = 1.0f / (1.0f + expf(-gb));
    // L2 norms: warps 0-3 hold q, warps 4-7 hold k.
    const float ss = warp_sum(val * val);
    if (lane == 0) sh.red[warp] = ss;
    sync();
    const float nq = rsqrtf(sh.red[0] + sh.red[1] + sh.red[2] + sh.red[3] + 1e-6f);
    const float nk = rsqrtf(sh.red[4] + sh.red[5] + sh.red[6] + sh.red[7] + 1e-6f);
    if (tid < kGdnDim) sh.qs[i] = val * nq * 0.08838834764f;
    else sh.ks[i] = val * nk;
    sync();
    if (warp < 4) {
      const float p = warp_sum(sh.ks[tid] * sh.qs[tid]);
      if (lane == 0) sh.red[warp] = p;  // red[0..3] no longer needed for nq
    }
    float sk = 0.f, sq = 0.f;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      sk = fmaf(sv[jj], sh.ks[jg * 8 + jj], sk);
      sq = fmaf(sv[jj], sh.qs[jg * 8 + jj], sq);
    }
    sh.psk[jg][tl] = sk;
    sh.psq[jg][tl] = sq;
    sync();
    if (tid < kSlice) {
      float a0 = 0.f, c0 = 0.f;
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        a0 += sh.psk[r][tid];
        c0 += sh.psq[r][tid];
      }
      sh.sk_s[tid] = a0;
      sh.sq_s[tid] = c0;
    }
    if (tid == 0) sh.kq_s = sh.red[0] + sh.red[1] + sh.red[2] + sh.red[3];
    sync();
    const float dv = beta * (sh.vs[tl] - g * sh.sk_s[tl]);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) S[(size_t)(jg * 8 + jj) * kGdnDim] = g * sv[jj] + dv * sh.ks[jg * 8 + jj];
    if (jg == 0) a.out[(size_t)b * kMixerOut + h * kGdnDim + t0 + tl] = g * sh.sq_s[tl] + dv * sh.kq_s;
    sync();  // shared memory is reused by the next item
  }
};

}  // namespace dev
}  // namespace qne
