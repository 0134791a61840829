// Gated full-attention decode step over a paged f16 KV cache (attention,
// kernels/src/shaders.rs:531-633; CPU form kernels/src/lib.rs:630-677).
//
// What it computes, per query head h (8 heads of 256 sharing 2 KV heads, 4:1):
//   q = RMSNorm_256(q_h) * q_norm, k = RMSNorm_256(k_kvh) * k_norm (eps 1e-6),
//   rotate-half RoPE on dims 0..63 (pairs (i, i + 32)) at angle pos * theta^(-2i/64),
//   the current K/V are appended to the cache, then softmax(q K^T / 16) V over positions
//   0..pos, times sigmoid(gate_h).
//
// B200 design: the cache is paged (16-token f16 pages, per-sequence page tables); one CTA per
// (context split, KV head, sequence) serves the 4 query heads of the KV head, streams its
// split's K and V rows with 16-byte loads (K and V of eight tokens in flight per lane), keeps
// an online softmax per head, and writes a partial (max, sum, 4 x 256 accumulator). The last
// CTA of each (sequence, KV head) to finish merges the partials and applies the output gate.
// The CTA whose split holds `pos` normalizes, rotates and appends the current K/V (rounded to
// f16) and uses the rounded values for that position; no other CTA reads that slot.
// RoPE angles come from a host-built table (double precision), identical for every consumer.
#include <math.h>

#include <cmath>

#include "gdn.cuh"
#include "gemv.cuh"

namespace qne {
namespace {

constexpr int kSub = 64;           // tokens per sub-block (8 per warp)
constexpr int kMaxSplits = kMaxContext / kSub;  // 64
constexpr int kQPerKv = kAttnHeads / kKvHeads;  // 4

struct Scratch {
  float* acc;        // [batch][2][kMaxSplits][4][256]
  float* ml;         // [batch][2][kMaxSplits][4][2]
  uint32_t* ticket;  // [batch][2]
};

__host__ __device__ inline size_t scratch_acc_bytes(int batch) {
  return (size_t)batch * kKvHeads * kMaxSplits * kQPerKv * kHeadDim * 4;
}
__host__ __device__ inline size_t scratch_ml_bytes(int batch) {
  return (size_t)batch * kKvHeads * kMaxSplits * kQPerKv * 2 * 4;
}
__host__ __device__ inline Scratch carve(void* p, int batch) {
  Scratch s;
  uint8_t* b = static_cast<uint8_t*>(p);
  s.acc = reinterpret_cast<float*>(b);
  s.ml = reinterpret_cast<float*>(b + scratch_acc_bytes(batch));
  s.ticket = reinterpret_cast<uint32_t*>(b + scratch_acc_bytes(batch) + scratch_ml_bytes(batch));
  return s;
}

__device__ __forceinline__ const uint16_t* kv_row(const uint16_t* kv, uint32_t page, int kind,
                                                  int kvh, int slot) {
  return kv + (size_t)page * kPageElems + ((size_t)(kind * kKvHeads + kvh) * kPageTokens + slot) * kHeadDim;
}

__device__ __forceinline__ void unpack8(const uint4& w, float* f) {
  float2 a = h2f2(w.x), b = h2f2(w.y), c = h2f2(w.z), d = h2f2(w.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

struct KernelArgs {
  AttnArgs a;
  int split;        // tokens per CTA (multiple of kSub)
  uint32_t pool_pages;
};

__global__ void __launch_bounds__(256) attention_kernel(const KernelArgs ka) {
  const AttnArgs& a = ka.a;
  __shared__ __align__(16) float q_s[kQPerKv][kHeadDim];
  __shared__ __align__(16) float kc_s[kHeadDim];
  __shared__ __align__(16) float vc_s[kHeadDim];
  __shared__ float sc[kQPerKv][kSub];
  __shared__ float red[8][kQPerKv];
  __shared__ float blk_scale[kQPerKv];
  __shared__ float run_m[kQPerKv], run_l[kQPerKv];
  __shared__ __align__(16) float accw[8][kQPerKv][kHeadDim];  // 32 KB, per-warp partials
  __shared__ uint32_t is_last;

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  pdl_launch();
  pdl_wait();

  uint32_t pos = a.pos[(size_t)b * a.pos_stride];
  if (pos >= (uint32_t)kMaxContext) {
    if (a.flags && t == 0 && split == 0 && kvh == 0) atomicOr(a.flags + (size_t)b * a.flags_stride, kFlagPosClamped);
    pos = kMaxContext - 1;
  }
  const int len = (int)pos + 1;
  const int nsplit = (len + ka.split - 1) / ka.split;
  if (split >= nsplit) return;
  const int l0 = split * ka.split;
  const int l1 = min(l0 + ka.split, len);
  const bool owner = (int)pos >= l0 && (int)pos < l1;
  const float* pr = a.proj + (size_t)b * kAttnProj;
  const uint32_t* pt = a.page_table + (size_t)b * kPagesPerSeq;
  const float* rc = a.rope + (size_t)pos * kRopeHalf;                      // cos
  const float* rs = a.rope + (size_t)kMaxContext * kRopeHalf + (size_t)pos * kRopeHalf;  // sin

  // ---- q of the 4 heads (and the current k) : RMSNorm, RoPE ----
  float xq[kQPerKv];
  float ssq[kQPerKv];
#pragma unroll
  for (int hh = 0; hh < kQPerKv; ++hh) {
    xq[hh] = pr[(kvh * kQPerKv + hh) * kHeadDim + t];
    ssq[hh] = warp_sum(xq[hh] * xq[hh]);
  }
  const float xk = owner ? pr[4096 + kvh * kHeadDim + t] : 0.f;
  const float ssk = warp_sum(xk * xk);
  if (lane == 0) {
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) red[warp][hh] = ssq[hh];
  }
  __shared__ float redk[8];
  if (lane == 0) redk[warp] = ssk;
  __syncthreads();
#pragma unroll
  for (int hh = 0; hh < kQPerKv; ++hh) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w][hh];
    q_s[hh][t] = xq[hh] * rsqrtf(s / (float)kHeadDim + 1e-6f) * a.norms[t];
  }
  if (owner) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += redk[w];
    kc_s[t] = xk * rsqrtf(s / (float)kHeadDim + 1e-6f) * a.norms[kHeadDim + t];
  }
  __syncthreads();
  float qr[kQPerKv];
  float kr = 0.f;
#pragma unroll
  for (int hh = 0; hh < kQPerKv; ++hh) qr[hh] = q_s[hh][t];
  if (owner) kr = kc_s[t];
  if (t < 2 * kRopeHalf) {
    const int i = t & (kRopeHalf - 1);
    const float c = rc[i], s = rs[i];
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh)
      qr[hh] = (t < kRopeHalf) ? q_s[hh][t] * c - q_s[hh][t + kRopeHalf] * s
                               : q_s[hh][t] * c + q_s[hh][t - kRopeHalf] * s;
    if (owner)
      kr = (t < kRopeHalf) ? kc_s[t] * c - kc_s[t + kRopeHalf] * s : kc_s[t] * c + kc_s[t - kRopeHalf] * s;
  }
  __syncthreads();
#pragma unroll
  for (int hh = 0; hh < kQPerKv; ++hh) q_s[hh][t] = qr[hh] * 0.0625f;  // 1/sqrt(256), exact
  if (owner) {
    // Append the current key and value, rounded to f16, and use the rounded values below.
    const uint32_t page = pt[pos / kPageTokens];
    if (page < ka.pool_pages) {
      const __half kh = __float2half_rn(kr);
      const __half vh = __float2half_rn(pr[4608 + kvh * kHeadDim + t]);
      uint16_t* kdst = const_cast<uint16_t*>(kv_row(a.kv, page, 0, kvh, pos % kPageTokens));
      uint16_t* vdst = const_cast<uint16_t*>(kv_row(a.kv, page, 1, kvh, pos % kPageTokens));
      kdst[t] = __half_as_ushort(kh);
      vdst[t] = __half_as_ushort(vh);
      kc_s[t] = __half2float(kh);
      vc_s[t] = __half2float(vh);
    } else {
      kc_s[t] = 0.f;
      vc_s[t] = 0.f;
    }
  }
  if (t < kQPerKv) {
    run_m[t] = -INFINITY;
    run_l[t] = 0.f;
  }
  __syncthreads();

  // q slice of this lane (dims lane*8 .. lane*8+7) for the 4 heads.
  float qv[kQPerKv][8];
#pragma unroll
  for (int hh = 0; hh < kQPerKv; ++hh) {
    *reinterpret_cast<float4*>(&qv[hh][0]) = *reinterpret_cast<const float4*>(&q_s[hh][lane * 8]);
    *reinterpret_cast<float4*>(&qv[hh][4]) = *reinterpret_cast<const float4*>(&q_s[hh][lane * 8 + 4]);
  }
  float acc[kQPerKv][8];
#pragma unroll
  for (int hh = 0; hh < kQPerKv; ++hh)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[hh][e] = 0.f;

  for (int sb = l0; sb < l1; sb += kSub) {
    // Issue the K and V loads of this warp's 8 tokens.
    uint4 kw[8], vw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int l = sb + warp + 8 * i;
      kw[i] = make_uint4(0, 0, 0, 0);
      vw[i] = make_uint4(0, 0, 0, 0);
      if (l < l1 && l != (int)pos) {
        const uint32_t page = pt[l / kPageTokens];
        if (page < ka.pool_pages) {
          kw[i] = ld_stream(kv_row(a.kv, page, 0, kvh, l % kPageTokens) + lane * 8);
          vw[i] = ld_stream(kv_row(a.kv, page, 1, kvh, l % kPageTokens) + lane * 8);
        }
      }
    }
    // Scores.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int l = sb + warp + 8 * i;
      float kf[8];
      if (l == (int)pos) {
        *reinterpret_cast<float4*>(kf) = *reinterpret_cast<const float4*>(&kc_s[lane * 8]);
        *reinterpret_cast<float4*>(kf + 4) = *reinterpret_cast<const float4*>(&kc_s[lane * 8 + 4]);
      } else {
        unpack8(kw[i], kf);
      }
      float d[kQPerKv];
#pragma unroll
      for (int hh = 0; hh < kQPerKv; ++hh) {
        float p0 = qv[hh][0] * kf[0], p1 = qv[hh][4] * kf[4];
#pragma unroll
        for (int e = 1; e < 4; ++e) {
          p0 = fmaf(qv[hh][e], kf[e], p0);
          p1 = fmaf(qv[hh][4 + e], kf[4 + e], p1);
        }
        d[hh] = warp_sum(p0 + p1);
      }
      if (lane == 0) {
#pragma unroll
        for (int hh = 0; hh < kQPerKv; ++hh) sc[hh][warp + 8 * i] = (l < l1) ? d[hh] : -INFINITY;
      }
    }
    __syncthreads();
    // Block max per head: thread (hh = t / 64, j = t % 64).
    {
      const int hh = t >> 6, j = t & 63;
      const float s = sc[hh][j];
      float m = warp_max(s);
      if (lane == 0) red[warp][0] = m;
      __syncthreads();
      if (j == 0) {
        const float mb = fmaxf(red[2 * hh][0], red[2 * hh + 1][0]);
        const float mnew = fmaxf(run_m[hh], mb);
        blk_scale[hh] = (run_m[hh] == -INFINITY) ? 0.f : expf(run_m[hh] - mnew);
        run_m[hh] = mnew;
      }
      __syncthreads();
      const float p = (s == -INFINITY) ? 0.f : expf(s - run_m[hh]);
      sc[hh][j] = p;
      const float ps = warp_sum(p);
      if (lane == 0) red[warp][1] = ps;
      __syncthreads();
      if (j == 0) run_l[hh] = run_l[hh] * blk_scale[hh] + red[2 * hh][1] + red[2 * hh + 1][1];
    }
    // Rescale this warp's accumulators, then add p * V for its tokens.
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) {
      const float f = blk_scale[hh];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[hh][e] *= f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int l = sb + warp + 8 * i;
      if (l < l1) {
        float vf[8];
        if (l == (int)pos) {
          *reinterpret_cast<float4*>(vf) = *reinterpret_cast<const float4*>(&vc_s[lane * 8]);
          *reinterpret_cast<float4*>(vf + 4) = *reinterpret_cast<const float4*>(&vc_s[lane * 8 + 4]);
        } else {
          unpack8(vw[i], vf);
        }
#pragma unroll
        for (int hh = 0; hh < kQPerKv; ++hh) {
          const float p = sc[hh][warp + 8 * i];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[hh][e] = fmaf(p, vf[e], acc[hh][e]);
        }
      }
    }
    __syncthreads();  // sc is rewritten by the next sub-block
  }

  // Merge the 8 warps' accumulators and write this split's partial.
#pragma unroll
  for (int hh = 0; hh < kQPerKv; ++hh) {
    *reinterpret_cast<float4*>(&accw[warp][hh][lane * 8]) = *reinterpret_cast<float4*>(&acc[hh][0]);
    *reinterpret_cast<float4*>(&accw[warp][hh][lane * 8 + 4]) = *reinterpret_cast<float4*>(&acc[hh][4]);
  }
  __syncthreads();
  Scratch S = carve(a.scratch, a.batch);
  const size_t part = ((size_t)b * kKvHeads + kvh) * kMaxSplits + split;
#pragma unroll
  for (int hh = 0; hh < kQPerKv; ++hh) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += accw[w][hh][t];
    S.acc[(part * kQPerKv + hh) * kHeadDim + t] = s;
  }
  if (t < kQPerKv) {
    S.ml[(part * kQPerKv + t) * 2 + 0] = run_m[t];
    S.ml[(part * kQPerKv + t) * 2 + 1] = run_l[t];
  }
  __threadfence();
  __syncthreads();
  if (t == 0) {
    const uint32_t done = atomicAdd(S.ticket + (size_t)b * kKvHeads + kvh, 1u);
    is_last = (done == (uint32_t)nsplit - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();

  // ---- merge: thread (hh = t / 64, dims (t % 64) * 4 .. +4) ----
  {
    const int hh = t >> 6, d0 = (t & 63) * 4;
    const size_t base = ((size_t)b * kKvHeads + kvh) * kMaxSplits;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(S.ml + ((base + s) * kQPerKv + hh) * 2));
    float L = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    int s = 0;
    for (; s + 8 <= nsplit; s += 8) {
      float4 av[8];
      float wv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        av[u] = __ldcg(reinterpret_cast<const float4*>(S.acc + ((base + s + u) * kQPerKv + hh) * kHeadDim + d0));
        const float m = __ldcg(S.ml + ((base + s + u) * kQPerKv + hh) * 2);
        const float l = __ldcg(S.ml + ((base + s + u) * kQPerKv + hh) * 2 + 1);
        wv[u] = (m == -INFINITY) ? 0.f : expf(m - M);
        L = fmaf(wv[u], l, L);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        o.x = fmaf(wv[u], av[u].x, o.x);
        o.y = fmaf(wv[u], av[u].y, o.y);
        o.z = fmaf(wv[u], av[u].z, o.z);
        o.w = fmaf(wv[u], av[u].w, o.w);
      }
    }
    for (; s < nsplit; ++s) {
      const float4 av = __ldcg(reinterpret_cast<const float4*>(S.acc + ((base + s) * kQPerKv + hh) * kHeadDim + d0));
      const float m = __ldcg(S.ml + ((base + s) * kQPerKv + hh) * 2);
      const float l = __ldcg(S.ml + ((base + s) * kQPerKv + hh) * 2 + 1);
      const float w = (m == -INFINITY) ? 0.f : expf(m - M);
      L = fmaf(w, l, L);
      o.x = fmaf(w, av.x, o.x);
      o.y = fmaf(w, av.y, o.y);
      o.z = fmaf(w, av.z, o.z);
      o.w = fmaf(w, av.w, o.w);
    }
    const int h = kvh * kQPerKv + hh;
    const float4 gate = *reinterpret_cast<const float4*>(pr + 2048 + h * kHeadDim + d0);
    float4 r;
    r.x = o.x / L / (1.0f + expf(-gate.x));
    r.y = o.y / L / (1.0f + expf(-gate.y));
    r.z = o.z / L / (1.0f + expf(-gate.z));
    r.w = o.w / L / (1.0f + expf(-gate.w));
    *reinterpret_cast<float4*>(a.out + (size_t)b * kMixerOut + h * kHeadDim + d0) = r;
  }
  if (t == 0) S.ticket[(size_t)b * kKvHeads + kvh] = 0u;
}

__global__ void kv_gather_kernel(const uint16_t* kv, const uint32_t* pt, uint32_t len,
                                 uint16_t* out_k, uint16_t* out_v) {
  // one CTA per (position, kv head), 256 threads = dims
  const uint32_t l = blockIdx.x;
  const int kvh = blockIdx.y, d = threadIdx.x;
  if (l >= len) return;
  const uint32_t page = pt[l / kPageTokens];
  out_k[((size_t)kvh * len + l) * kHeadDim + d] = kv_row(kv, page, 0, kvh, l % kPageTokens)[d];
  out_v[((size_t)kvh * len + l) * kHeadDim + d] = kv_row(kv, page, 1, kvh, l % kPageTokens)[d];
}

}  // namespace

size_t attention_scratch_bytes(int batch) {
  return scratch_acc_bytes(batch) + scratch_ml_bytes(batch) + (size_t)batch * kKvHeads * 4 + 256;
}

cudaError_t launch_attention(const AttnArgs& a, uint32_t pool_pages, int split_tokens,
                             cudaStream_t stream, bool pdl) {
  KernelArgs ka;
  ka.a = a;
  ka.split = split_tokens;
  ka.pool_pages = pool_pages;
  const int max_splits = (kMaxContext + split_tokens - 1) / split_tokens;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(max_splits, kKvHeads, a.batch);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  return cudaLaunchKernelEx(&cfg, attention_kernel, ka);
}

cudaError_t launch_kv_gather(const uint16_t* kv, const uint32_t* page_table, uint32_t len,
                             uint16_t* out_k, uint16_t* out_v, cudaStream_t stream) {
  if (len == 0) return cudaSuccess;
  count_launch();
  kv_gather_kernel<<<dim3(len, kKvHeads), kHeadDim, 0, stream>>>(kv, page_table, len, out_k, out_v);
  return cudaGetLastError();
}

void rope_table_host(float* table, double theta) {
  for (int p = 0; p < kMaxContext; ++p)
    for (int i = 0; i < kRopeHalf; ++i) {
      const double inv_freq = std::pow(theta, -(2.0 * i) / 64.0);
      const double ang = (double)p * inv_freq;
      table[p * kRopeHalf + i] = (float)std::cos(ang);
      table[kMaxContext * kRopeHalf + p * kRopeHalf + i] = (float)std::sin(ang);
    }
}

}  // namespace qne
