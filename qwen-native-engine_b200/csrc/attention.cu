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
constexpr int kGroup = 8;          // splits merged per first-level merge
constexpr int kMaxGroups = kMaxSplits / kGroup;
constexpr int kQPerKv = kAttnHeads / kKvHeads;  // 4
constexpr int kPart = kQPerKv * kHeadDim;       // floats of one partial accumulator

// Scratch (per sequence and KV head): split partials, group partials, completion tickets.
struct Scratch {
  float* acc;         // [batch][2][kMaxSplits][4][256]
  float* ml;          // [batch][2][kMaxSplits][4][2]  (running max, sum)
  float* gacc;        // [batch][2][kMaxGroups][4][256]
  float* gml;         // [batch][2][kMaxGroups][4][2]
  uint32_t* gticket;  // [batch][2][kMaxGroups]
  uint32_t* ticket;   // [batch][2]
};

__host__ __device__ inline size_t sz_acc(int batch) { return (size_t)batch * kKvHeads * kMaxSplits * kPart * 4; }
__host__ __device__ inline size_t sz_ml(int batch) { return (size_t)batch * kKvHeads * kMaxSplits * kQPerKv * 2 * 4; }
__host__ __device__ inline size_t sz_gacc(int batch) { return (size_t)batch * kKvHeads * kMaxGroups * kPart * 4; }
__host__ __device__ inline size_t sz_gml(int batch) { return (size_t)batch * kKvHeads * kMaxGroups * kQPerKv * 2 * 4; }
__host__ __device__ inline size_t sz_gt(int batch) { return (size_t)batch * kKvHeads * kMaxGroups * 4; }
__host__ __device__ inline size_t sz_t(int batch) { return (size_t)batch * kKvHeads * 4; }
__host__ __device__ inline Scratch carve(void* p, int batch) {
  Scratch s;
  uint8_t* b = static_cast<uint8_t*>(p);
  s.acc = reinterpret_cast<float*>(b);
  b += sz_acc(batch);
  s.ml = reinterpret_cast<float*>(b);
  b += sz_ml(batch);
  s.gacc = reinterpret_cast<float*>(b);
  b += sz_gacc(batch);
  s.gml = reinterpret_cast<float*>(b);
  b += sz_gml(batch);
  s.gticket = reinterpret_cast<uint32_t*>(b);
  b += sz_gt(batch);
  s.ticket = reinterpret_cast<uint32_t*>(b);
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

// Merges n partials (each: 4 heads x 256 unnormalized sums, plus (max, sum) per head) for the
// calling thread's head hh and dims d0..d0+3. Returns the merged (max, sum) and sums.
__device__ __forceinline__ void merge_parts(const float* acc, const float* ml, int n, int hh, int d0, float& M,
                                            float& L, float4& o) {
  float m[kGroup], l[kGroup];
  float4 av[kGroup];
#pragma unroll
  for (int u = 0; u < kGroup; ++u) {
    if (u < n) {
      m[u] = __ldcg(ml + ((size_t)u * kQPerKv + hh) * 2);
      l[u] = __ldcg(ml + ((size_t)u * kQPerKv + hh) * 2 + 1);
      av[u] = __ldcg(reinterpret_cast<const float4*>(acc + (size_t)u * kPart + hh * kHeadDim + d0));
    }
  }
  M = -INFINITY;
#pragma unroll
  for (int u = 0; u < kGroup; ++u)
    if (u < n) M = fmaxf(M, m[u]);
  L = 0.f;
  o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int u = 0; u < kGroup; ++u) {
    if (u < n) {
      const float w = (m[u] == -INFINITY) ? 0.f : expf(m[u] - M);
      L = fmaf(w, l[u], L);
      o.x = fmaf(w, av[u].x, o.x);
      o.y = fmaf(w, av[u].y, o.y);
      o.z = fmaf(w, av[u].z, o.z);
      o.w = fmaf(w, av[u].w, o.w);
    }
  }
}

__global__ void __launch_bounds__(256, 2) attention_kernel(const KernelArgs ka) {
  const AttnArgs& a = ka.a;
  __shared__ __align__(16) float q_s[kQPerKv][kHeadDim];
  __shared__ __align__(16) float kc_s[kHeadDim];
  __shared__ __align__(16) float vc_s[kHeadDim];
  __shared__ float sc[kQPerKv][kSub];
  __shared__ float red[8][kQPerKv];
  __shared__ float redk[8];
  __shared__ float blk_scale[kQPerKv];
  __shared__ float run_m[kQPerKv], run_l[kQPerKv];
  __shared__ __align__(16) float accw[8][kPart];  // 32 KB, per-warp partials
  __shared__ uint32_t flag;

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

  // K of this warp's 8 tokens of the first sub-block is issued before the q/k work below; V of
  // every sub-block is issued once its scores are computed, ahead of the softmax.
  uint4 kw[8], vw[8];
  auto issue = [&](uint4* dst, int kind, int sb) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int l = sb + warp + 8 * i;
      dst[i] = make_uint4(0, 0, 0, 0);
      if (l < l1 && l != (int)pos) {
        const uint32_t page = pt[l / kPageTokens];
        if (page < ka.pool_pages) dst[i] = ld_stream(kv_row(a.kv, page, kind, kvh, l % kPageTokens) + lane * 8);
      }
    }
  };
  issue(kw, 0, l0);

  // ---- q of the 4 heads (and the current k): RMSNorm, RoPE ----
  const float* rc = a.rope + (size_t)pos * kRopeHalf;                                  // cos
  const float* rs = a.rope + (size_t)kMaxContext * kRopeHalf + (size_t)pos * kRopeHalf;  // sin
  {
    float xq[kQPerKv];
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) {
      xq[hh] = pr[(kvh * kQPerKv + hh) * kHeadDim + t];
      const float ss = warp_sum(xq[hh] * xq[hh]);
      if (lane == 0) red[warp][hh] = ss;
    }
    const float xk = owner ? pr[4096 + kvh * kHeadDim + t] : 0.f;
    const float ssk = warp_sum(xk * xk);
    if (lane == 0) redk[warp] = ssk;
    __syncthreads();
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sum += red[w][hh];
      q_s[hh][t] = xq[hh] * rsqrtf(sum / (float)kHeadDim + 1e-6f) * a.norms[t];
    }
    if (owner) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sum += redk[w];
      kc_s[t] = xk * rsqrtf(sum / (float)kHeadDim + 1e-6f) * a.norms[kHeadDim + t];
    }
  }
  __syncthreads();
  {
    float qr[kQPerKv];
    float kr = 0.f;
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) qr[hh] = q_s[hh][t];
    if (owner) kr = kc_s[t];
    if (t < 2 * kRopeHalf) {
      const int i = t & (kRopeHalf - 1);
      const float c = rc[i], sn = rs[i];
#pragma unroll
      for (int hh = 0; hh < kQPerKv; ++hh)
        qr[hh] = (t < kRopeHalf) ? q_s[hh][t] * c - q_s[hh][t + kRopeHalf] * sn
                                 : q_s[hh][t] * c + q_s[hh][t - kRopeHalf] * sn;
      if (owner)
        kr = (t < kRopeHalf) ? kc_s[t] * c - kc_s[t + kRopeHalf] * sn : kc_s[t] * c + kc_s[t - kRopeHalf] * sn;
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
  }
  __syncthreads();

  float acc[kQPerKv][8];
#pragma unroll
  for (int hh = 0; hh < kQPerKv; ++hh)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[hh][e] = 0.f;

  for (int sb = l0; sb < l1; sb += kSub) {
    if (sb != l0) issue(kw, 0, sb);
    // Scores (q read from shared memory: keeps registers for the loads in flight).
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
        const float4 qa = *reinterpret_cast<const float4*>(&q_s[hh][lane * 8]);
        const float4 qb = *reinterpret_cast<const float4*>(&q_s[hh][lane * 8 + 4]);
        float p0 = qa.x * kf[0], p1 = qb.x * kf[4];
        p0 = fmaf(qa.y, kf[1], p0);
        p1 = fmaf(qb.y, kf[5], p1);
        p0 = fmaf(qa.z, kf[2], p0);
        p1 = fmaf(qb.z, kf[6], p1);
        p0 = fmaf(qa.w, kf[3], p0);
        p1 = fmaf(qb.w, kf[7], p1);
        d[hh] = warp_sum(p0 + p1);
      }
      if (lane == 0) {
#pragma unroll
        for (int hh = 0; hh < kQPerKv; ++hh) sc[hh][warp + 8 * i] = (l < l1) ? d[hh] : -INFINITY;
      }
    }
    issue(vw, 1, sb);  // V latency overlaps the softmax below
    __syncthreads();
    // Block max per head: thread (hh = t / 64, j = t % 64).
    {
      const int hh = t >> 6, j = t & 63;
      const float sval = sc[hh][j];
      const float m = warp_max(sval);
      if (lane == 0) red[warp][0] = m;
      __syncthreads();
      if (j == 0) {
        const float mb = fmaxf(red[2 * hh][0], red[2 * hh + 1][0]);
        const float mnew = fmaxf(run_m[hh], mb);
        blk_scale[hh] = (run_m[hh] == -INFINITY) ? 0.f : expf(run_m[hh] - mnew);
        run_m[hh] = mnew;
      }
      __syncthreads();
      const float p = (sval == -INFINITY) ? 0.f : expf(sval - run_m[hh]);
      sc[hh][j] = p;
      const float ps = warp_sum(p);
      if (lane == 0) red[warp][1] = ps;
      __syncthreads();
      if (j == 0) run_l[hh] = run_l[hh] * blk_scale[hh] + red[2 * hh][1] + red[2 * hh + 1][1];
    }
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
    *reinterpret_cast<float4*>(&accw[warp][hh * kHeadDim + lane * 8]) = *reinterpret_cast<float4*>(&acc[hh][0]);
    *reinterpret_cast<float4*>(&accw[warp][hh * kHeadDim + lane * 8 + 4]) = *reinterpret_cast<float4*>(&acc[hh][4]);
  }
  __syncthreads();
  Scratch S = carve(a.scratch, a.batch);
  const size_t sk = (size_t)b * kKvHeads + kvh;  // (sequence, KV head)
  const int hh = t >> 6, d0 = (t & 63) * 4;       // merge mapping
  const int group = split / kGroup, ngroups = (nsplit + kGroup - 1) / kGroup;
  const int gsize = min(kGroup, nsplit - group * kGroup);
  float* gacc = S.gacc + (sk * kMaxGroups) * kPart;
  float* gml = S.gml + (sk * kMaxGroups) * kQPerKv * 2;

  if (nsplit == 1) {
    // A single split needs no merge: normalize and gate directly.
    float4 o;
    o.x = o.y = o.z = o.w = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float4 v = *reinterpret_cast<const float4*>(&accw[w][hh * kHeadDim + d0]);
      o.x += v.x;
      o.y += v.y;
      o.z += v.z;
      o.w += v.w;
    }
    const float L = run_l[hh];
    const int h = kvh * kQPerKv + hh;
    const float4 gate = *reinterpret_cast<const float4*>(pr + 2048 + h * kHeadDim + d0);
    float4 r;
    r.x = o.x / L / (1.0f + expf(-gate.x));
    r.y = o.y / L / (1.0f + expf(-gate.y));
    r.z = o.z / L / (1.0f + expf(-gate.z));
    r.w = o.w / L / (1.0f + expf(-gate.w));
    *reinterpret_cast<float4*>(a.out + (size_t)b * kMixerOut + h * kHeadDim + d0) = r;
    return;
  }

  {
    float* pacc = S.acc + (sk * kMaxSplits + split) * kPart;
    float* pml = S.ml + (sk * kMaxSplits + split) * kQPerKv * 2;
    float4 o;
    o.x = o.y = o.z = o.w = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float4 v = *reinterpret_cast<const float4*>(&accw[w][hh * kHeadDim + d0]);
      o.x += v.x;
      o.y += v.y;
      o.z += v.z;
      o.w += v.w;
    }
    *reinterpret_cast<float4*>(pacc + hh * kHeadDim + d0) = o;
    if (t < kQPerKv) {
      pml[t * 2 + 0] = run_m[t];
      pml[t * 2 + 1] = run_l[t];
    }
  }
  // First level: the last split of each group of 8 merges the group.
  __threadfence();
  __syncthreads();
  if (t == 0) flag = (atomicAdd(S.gticket + sk * kMaxGroups + group, 1u) == (uint32_t)gsize - 1) ? 1u : 0u;
  __syncthreads();
  if (!flag) return;
  __threadfence();
  float M, L;
  float4 o;
  merge_parts(S.acc + (sk * kMaxSplits + group * kGroup) * kPart,
              S.ml + (sk * kMaxSplits + group * kGroup) * kQPerKv * 2, gsize, hh, d0, M, L, o);
  if (t == 0) S.gticket[sk * kMaxGroups + group] = 0u;
  if (ngroups > 1) {
    *reinterpret_cast<float4*>(gacc + (size_t)group * kPart + hh * kHeadDim + d0) = o;
    if ((t & 63) == 0) {
      gml[((size_t)group * kQPerKv + hh) * 2 + 0] = M;
      gml[((size_t)group * kQPerKv + hh) * 2 + 1] = L;
    }
    // Second level: the last group to finish merges the groups.
    __threadfence();
    __syncthreads();
    if (t == 0) flag = (atomicAdd(S.ticket + sk, 1u) == (uint32_t)ngroups - 1) ? 1u : 0u;
    __syncthreads();
    if (!flag) return;
    __threadfence();
    merge_parts(gacc, gml, ngroups, hh, d0, M, L, o);
    if (t == 0) S.ticket[sk] = 0u;
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
  return sz_acc(batch) + sz_ml(batch) + sz_gacc(batch) + sz_gml(batch) + sz_gt(batch) + sz_t(batch) + 256;
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
