// Paged-KV attention decode step, one work item = (context split, KV head, sequence); shared by
// the per-kernel path (attention.cu) and the persistent decode kernel. prefetch() reads the
// position, the page table and the first 64 keys of the split (rows of earlier tokens), so the
// persistent kernel issues it before the barrier that publishes proj.
#pragma once

#include "common.cuh"
#include "gdn.cuh"

namespace qne {
namespace dev {

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
  uint8_t* q = static_cast<uint8_t*>(p);
  s.acc = reinterpret_cast<float*>(q);
  q += sz_acc(batch);
  s.ml = reinterpret_cast<float*>(q);
  q += sz_ml(batch);
  s.gacc = reinterpret_cast<float*>(q);
  q += sz_gacc(batch);
  s.gml = reinterpret_cast<float*>(q);
  q += sz_gml(batch);
  s.gticket = reinterpret_cast<uint32_t*>(q);
  q += sz_gt(batch);
  s.ticket = reinterpret_cast<uint32_t*>(q);
  return s;
}

__device__ __forceinline__ const uint16_t* kv_row(const uint16_t* kv, uint32_t page, int kind, int kvh, int slot) {
  return kv + (size_t)page * kPageElems + ((size_t)(kind * kKvHeads + kvh) * kPageTokens + slot) * kHeadDim;
}

__device__ __forceinline__ void unpack8(const uint4& w, float* f) {
  float2 a = h2f2(w.x), b = h2f2(w.y), c = h2f2(w.z), d = h2f2(w.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

struct KernelArgs {
  AttnArgs a;
  int split;        // tokens per item (multiple of kSub)
  int max_splits;   // items per (sequence, KV head) = ceil(4096 / split)
  uint32_t pool_pages;
  int spread = 0;   // 1: spread merge (every CTA of the launch is resident at once; host-checked)
};

// Shared memory of one attention work item (about 71 KB, so it is dynamic shared memory).
struct AttnShared {
  // K and V rows of the current 64-token sub-block, [token][dim] f16. Lane l of warp w stages
  // (and later reads) bytes 16l..16l+15 of the rows of tokens 8w..8w+7, so the staging needs no
  // synchronization beyond the lane's own cp.async group. After the last sub-block the K area
  // holds the per-warp partial accumulators (accw).
  __align__(16) uint16_t kst[kSub][kHeadDim];
  __align__(16) uint16_t vst[kSub][kHeadDim];
  __align__(16) float q_s[kQPerKv][kHeadDim];
  __align__(16) float kc_s[kHeadDim];  // the current token's key and value (f16-rounded)
  __align__(16) float vc_s[kHeadDim];
  float sc[kQPerKv][kSub];
  float red[8][kQPerKv];
  float redk[8];
  float blk_scale[kQPerKv];
  float run_m[kQPerKv], run_l[kQPerKv];
  uint32_t flag;
  __device__ __forceinline__ float* accw(int w) { return reinterpret_cast<float*>(&kst[0][0]) + w * kPart; }
};
static_assert(sizeof(AttnShared::kst) >= 8 * kPart * sizeof(float), "accw aliases the K staging area");

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

// Writes the 4 merged outputs r at (row b, column col) also as f16 hi / lo planes when the
// caller asked for them: the form the tensor-core GEMMs read their activations in, so the
// out-projection needs no separate conversion launch.
__device__ __forceinline__ void attn_store_planes(const AttnArgs& a, int b, int col, float4 r) {
  if (!a.out_xh) return;
  const float v[4] = {r.x, r.y, r.z, r.w};
  uint16_t hi[4], lo[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __half h = __float2half_rn(v[e]);
    hi[e] = __half_as_ushort(h);
    lo[e] = __half_as_ushort(__float2half_rn(v[e] - __half2float(h)));
  }
  const size_t o = (size_t)b * a.out_ldx + col;
  *reinterpret_cast<uint2*>(a.out_xh + o) = make_uint2(hi[0] | ((uint32_t)hi[1] << 16), hi[2] | ((uint32_t)hi[3] << 16));
  *reinterpret_cast<uint2*>(a.out_xl + o) = make_uint2(lo[0] | ((uint32_t)lo[1] << 16), lo[2] | ((uint32_t)lo[3] << 16));
}

constexpr int kSpread = 8;                        // mergers of a spread merge
constexpr uint64_t kMergeWaitNs = 1000000000ull;  // bound of a spread merger's wait (1 s)

__device__ __forceinline__ uint64_t attn_global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t attn_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Spread merge of the partials of (sequence b, KV head kvh), entered by every split after its
// partial is stored; used when all CTAs of the launch are resident at once (the host checks the
// grid against the occupancy), since mergers wait for the other splits. Every split arrives on a
// counter with a release reduction (no round trip); the last nm = min(nsplit, 8) splits are the
// mergers: merger j waits (bounded by kMergeWaitNs; on timeout kFlagTimeout goes to the flags
// word) until every split has arrived, then merges output slices j, j + nm, ... (slice s: head
// s / 2, dims 128 (s % 2) .. +127) over all splits in split order -- thread (g, f) combines splits
// g, g + 8, ... of float4 f, and the 8 groups are combined through shared memory (the V staging
// area, free after the last sub-block) -- applies the output gate and stores. The last merger to
// count itself out clears the counters for the next launch. Ends with __syncthreads.
template <class SH>
__device__ __forceinline__ void attn_spread_merge(const AttnArgs& a, SH& sh, int b, int kvh, int split, int nsplit,
                                                  const Scratch& S, size_t sk) {
  const int t = threadIdx.x;
  uint32_t* arrive = S.ticket + sk;
  uint32_t* leave = S.gticket + sk * kMaxGroups;  // group tickets are unused by this merge
  const int nm = min(nsplit, kSpread);
  const int j = split - (nsplit - nm);  // merger index; negative: not a merger
  __syncthreads();  // the CTA's partial stores precede thread 0's release
  if (t == 0) {
    __threadfence();
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(arrive) : "memory");
  }
  if (j < 0) {
    __syncthreads();  // shared memory is reused by the next item
    return;
  }
  if (t == 0) {
    const uint64_t t0 = attn_global_ns();
    uint32_t rounds = 0;
    while (attn_ld_acquire(arrive) < (uint32_t)nsplit) {
      if ((++rounds & 63u) == 0u && attn_global_ns() - t0 > kMergeWaitNs) {
        if (a.flags) atomicOr(a.flags + (size_t)b * a.flags_stride, kFlagTimeout);
        break;
      }
    }
  }
  __syncthreads();
  uint32_t left = 0;
  if (t == 0) left = atomicAdd(leave, 1u);  // its value is needed only at the end
  float* ws = reinterpret_cast<float*>(&sh.vst[0][0]);  // [8 groups][32] float4, then [8] max, [8] sum
  float4* ws4 = reinterpret_cast<float4*>(ws);
  const int f = t & 31, g = t >> 5;
  const float* pr = a.proj + (size_t)b * kAttnProj;
#pragma unroll 1
  for (int sl = j; sl < kSpread; sl += nm) {
    const int hs = sl >> 1, dd = (sl & 1) * 128 + 4 * f, h = kvh * kQPerKv + hs;
    float4 gate = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g == 0) gate = *reinterpret_cast<const float4*>(pr + 2048 + h * kHeadDim + dd);
    float mv[8], lv[8];
    float4 av[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int u = g + 8 * q;
      mv[q] = -INFINITY;
      lv[q] = 0.f;
      av[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (u < nsplit) {
        const float* ml = S.ml + ((sk * kMaxSplits + u) * kQPerKv + hs) * 2;
        mv[q] = __ldcg(ml);
        lv[q] = __ldcg(ml + 1);
        av[q] = __ldcg(reinterpret_cast<const float4*>(S.acc + (sk * kMaxSplits + u) * kPart + hs * kHeadDim + dd));
      }
    }
    float Mg = -INFINITY;
#pragma unroll
    for (int q = 0; q < 8; ++q) Mg = fmaxf(Mg, mv[q]);
    float Lg = 0.f;
    float4 og = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float w = (mv[q] == -INFINITY) ? 0.f : expf(mv[q] - Mg);
      Lg = fmaf(w, lv[q], Lg);
      og.x = fmaf(w, av[q].x, og.x);
      og.y = fmaf(w, av[q].y, og.y);
      og.z = fmaf(w, av[q].z, og.z);
      og.w = fmaf(w, av[q].w, og.w);
    }
    ws4[g * 32 + f] = og;
    if (f == 0) {
      ws[1024 + g] = Mg;
      ws[1032 + g] = Lg;
    }
    __syncthreads();
    if (g == 0) {
      float M = -INFINITY;
#pragma unroll
      for (int q = 0; q < 8; ++q) M = fmaxf(M, ws[1024 + q]);
      float L = 0.f;
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float mq = ws[1024 + q];
        const float w = (mq == -INFINITY) ? 0.f : expf(mq - M);
        const float4 x = ws4[q * 32 + f];
        L = fmaf(w, ws[1032 + q], L);
        o.x = fmaf(w, x.x, o.x);
        o.y = fmaf(w, x.y, o.y);
        o.z = fmaf(w, x.z, o.z);
        o.w = fmaf(w, x.w, o.w);
      }
      float4 r;
      r.x = o.x / L / (1.0f + expf(-gate.x));
      r.y = o.y / L / (1.0f + expf(-gate.y));
      r.z = o.z / L / (1.0f + expf(-gate.z));
      r.w = o.w / L / (1.0f + expf(-gate.w));
      *reinterpret_cast<float4*>(a.out + (size_t)b * kMixerOut + h * kHeadDim + dd) = r;
      attn_store_planes(a, b, h * kHeadDim + dd, r);
    }
    __syncthreads();  // ws is rewritten by the next slice / the next item
  }
  if (t == 0 && left == (uint32_t)nm - 1) {  // every merger has passed its wait
    *arrive = 0u;
    *leave = 0u;
  }
}

// Writes a split's partial for (sequence b, KV head kvh) -- thread t holds the unnormalized sums
// o of head t / 64, dims 4 (t % 64) .. +3, and sh.run_m / run_l hold the running max and sum per
// head -- then merges partials: spread (attn_spread_merge) when the launch allows it, else in two
// ticketed levels (groups of kGroup splits, then groups), where the CTA that completes the last
// merge applies the output gate and stores. Ends with __syncthreads.
// col0: the first of the item's 4 columns (query heads) of sequence row b in sh.run_m / run_l
// (items with two query rows hold them at columns 0-3 and 4-7).
template <class SH>
__device__ __forceinline__ void attn_merge_store(const AttnArgs& a, SH& sh, int b, int kvh, int split, int nsplit,
                                               float4 o, int col0 = 0, bool spread = false) {
  const int t = threadIdx.x;
  const int hh = t >> 6, d0 = (t & 63) * 4;
  const float* pr = a.proj + (size_t)b * kAttnProj;
  // The output gate, requested before the ticket round trips (only the last merger uses it).
  const int h = kvh * kQPerKv + hh;
  const float4 gate = *reinterpret_cast<const float4*>(pr + 2048 + h * kHeadDim + d0);
  Scratch S = carve(a.scratch, a.scratch_rows > 0 ? a.scratch_rows : a.batch);
  const size_t sk = (size_t)b * kKvHeads + kvh;  // (sequence, KV head)
  const int group = split / kGroup, ngroups = (nsplit + kGroup - 1) / kGroup;
  const int gsize = min(kGroup, nsplit - group * kGroup);
  float* gacc = S.gacc + (sk * kMaxGroups) * kPart;
  float* gml = S.gml + (sk * kMaxGroups) * kQPerKv * 2;
  float L = sh.run_l[col0 + hh];
  bool done = nsplit == 1;  // a single split needs no merge
  if (!done) {
    float* pacc = S.acc + (sk * kMaxSplits + split) * kPart;
    float* pml = S.ml + (sk * kMaxSplits + split) * kQPerKv * 2;
    *reinterpret_cast<float4*>(pacc + hh * kHeadDim + d0) = o;
    if (t < kQPerKv) {
      pml[t * 2 + 0] = sh.run_m[col0 + t];
      pml[t * 2 + 1] = sh.run_l[col0 + t];
    }
    if (spread) {
      attn_spread_merge(a, sh, b, kvh, split, nsplit, S, sk);
      return;
    }
    // Merge level 1: the last split of each group of 8 merges the group; level 2: the last
    // group to finish merges the groups. Each level is entered by one CTA only.
#pragma unroll 1
    for (int level = 0; level < 2 && !done; ++level) {
      const int n = level == 0 ? gsize : ngroups;
      uint32_t* ticket = level == 0 ? S.gticket + sk * kMaxGroups + group : S.ticket + sk;
      __threadfence();
      __syncthreads();
      if (t == 0) sh.flag = (atomicAdd(ticket, 1u) == (uint32_t)n - 1) ? 1u : 0u;
      __syncthreads();
      if (!sh.flag) {
        __syncthreads();  // shared memory is reused by the next item
        return;
      }
      __threadfence();
      float M;
      merge_parts(level == 0 ? S.acc + (sk * kMaxSplits + group * kGroup) * kPart : gacc,
                  level == 0 ? S.ml + (sk * kMaxSplits + group * kGroup) * kQPerKv * 2 : gml, n, hh, d0, M, L, o);
      if (t == 0) *ticket = 0u;
      if (level == 0 && ngroups > 1) {
        *reinterpret_cast<float4*>(gacc + (size_t)group * kPart + hh * kHeadDim + d0) = o;
        if ((t & 63) == 0) {
          gml[((size_t)group * kQPerKv + hh) * 2 + 0] = M;
          gml[((size_t)group * kQPerKv + hh) * 2 + 1] = L;
        }
      } else {
        done = true;
      }
    }
  }
  float4 r;
  r.x = o.x / L / (1.0f + expf(-gate.x));
  r.y = o.y / L / (1.0f + expf(-gate.y));
  r.z = o.z / L / (1.0f + expf(-gate.z));
  r.w = o.w / L / (1.0f + expf(-gate.w));
  *reinterpret_cast<float4*>(a.out + (size_t)b * kMixerOut + h * kHeadDim + d0) = r;
  attn_store_planes(a, b, h * kHeadDim + d0, r);
  __syncthreads();  // shared memory is reused by the next item
}

// The prologue's per-thread constants (thread t = dim t): q_norm[t], k_norm[t] and, for the
// rotated dims (t < 64), the cosine and sine of the pair's angle at pos. Nothing a previous
// kernel writes, so items load them with their staging, before the dependency wait.
__device__ __forceinline__ float4 attn_consts(const AttnArgs& a, uint32_t pos) {
  const int t = threadIdx.x;
  float4 c;
  c.x = a.norms[t];
  c.y = a.norms[kHeadDim + t];
  c.z = c.w = 0.f;
  if (t < 2 * kRopeHalf) {
    const int i = t & (kRopeHalf - 1);
    c.z = a.rope[(size_t)pos * kRopeHalf + i];
    c.w = a.rope[(size_t)kMaxContext * kRopeHalf + (size_t)pos * kRopeHalf + i];
  }
  return c;
}

// Prologue of a work item: q of the 4 heads of KV head kvh (RMSNorm with q_norm, RoPE at pos,
// times 1/16) into sh.q_s; for the item that holds pos (owner), the current key (RMSNorm with
// k_norm, RoPE) and value rounded to f16, appended to the cache page and kept in sh.kc_s /
// sh.vc_s; running max / sum reset. cst = attn_consts(a, pos). Ends with __syncthreads.
template <class SH>
__device__ __forceinline__ void attn_prologue(const KernelArgs& ka, SH& sh, int b, int kvh, uint32_t pos, bool owner,
                                              const uint32_t* pt, float4 cst, int col0 = 0) {
  const AttnArgs& a = ka.a;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float* pr = a.proj + (size_t)b * kAttnProj;
  // ---- q of the 4 heads (and the current k): RMSNorm, RoPE ----
  {
    float xq[kQPerKv];
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) {
      xq[hh] = pr[(kvh * kQPerKv + hh) * kHeadDim + t];
      const float ss = warp_sum(xq[hh] * xq[hh]);
      if (lane == 0) sh.red[warp][hh] = ss;
    }
    const float xk = owner ? pr[4096 + kvh * kHeadDim + t] : 0.f;
    const float ssk = warp_sum(xk * xk);
    if (lane == 0) sh.redk[warp] = ssk;
    __syncthreads();
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sum += sh.red[w][hh];
      sh.q_s[col0 + hh][t] = xq[hh] * rsqrtf(sum / (float)kHeadDim + 1e-6f) * cst.x;
    }
    if (owner) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sum += sh.redk[w];
      sh.kc_s[t] = xk * rsqrtf(sum / (float)kHeadDim + 1e-6f) * cst.y;
    }
  }
  __syncthreads();
  {
    float qr[kQPerKv];
    float kr = 0.f;
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) qr[hh] = sh.q_s[col0 + hh][t];
    if (owner) kr = sh.kc_s[t];
    if (t < 2 * kRopeHalf) {
      const float c = cst.z, sn = cst.w;
#pragma unroll
      for (int hh = 0; hh < kQPerKv; ++hh)
        qr[hh] = (t < kRopeHalf) ? sh.q_s[col0 + hh][t] * c - sh.q_s[col0 + hh][t + kRopeHalf] * sn
                                 : sh.q_s[col0 + hh][t] * c + sh.q_s[col0 + hh][t - kRopeHalf] * sn;
      if (owner)
        kr = (t < kRopeHalf) ? sh.kc_s[t] * c - sh.kc_s[t + kRopeHalf] * sn : sh.kc_s[t] * c + sh.kc_s[t - kRopeHalf] * sn;
    }
    __syncthreads();
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) sh.q_s[col0 + hh][t] = qr[hh] * 0.0625f;  // 1/sqrt(256), exact
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
        sh.kc_s[t] = __half2float(kh);
        sh.vc_s[t] = __half2float(vh);
      } else {
        sh.kc_s[t] = 0.f;
        sh.vc_s[t] = 0.f;
      }
    }
    if (t < kQPerKv) {
      sh.run_m[col0 + t] = -INFINITY;
      sh.run_l[col0 + t] = 0.f;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void cp_async16_attn(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}

struct AttnItem {
  int split, kvh, b, len, nsplit, l0, l1;
  uint32_t pos;
  bool valid, owner;
  const uint32_t* pt;
  float4 cst;  // attn_consts at pos

  // Stages K (kind 0) or V (kind 1) of tokens sb + 8w .. sb + 8w + 7 (this warp's share of a
  // sub-block) and commits them as one cp.async group: one 16-byte cp.async per row and lane.
  // Tokens outside [l0, l1), the current token when this item appends it (taken from kc_s / vc_s
  // instead) and rows of an out-of-range page are zero-filled. A lane later reads only the
  // chunks it staged itself, so a group needs no barrier beyond the lane's own wait. The warp's
  // 8 rows lie in one page, whose id is read once.
  __device__ __forceinline__ void stage(const KernelArgs& ka, AttnShared& sh, int sb, int kind) const {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (sb < l1) {
      const uint32_t pg = pt[(sb + warp * 8) / kPageTokens];
#pragma unroll 1
      for (int i = 0; i < 8; ++i) {
        const int t = warp * 8 + i, l = sb + t;
        uint4* d = reinterpret_cast<uint4*>(kind == 0 ? &sh.kst[t][lane * 8] : &sh.vst[t][lane * 8]);
        const uint32_t page = (l < l1 && !(owner && l == (int)pos)) ? pg : 0xFFFFFFFFu;
        if (page < ka.pool_pages) cp_async16_attn(d, kv_row(ka.a.kv, page, kind, kvh, l % kPageTokens) + lane * 8);
        else *d = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");  // an empty group past the split's end
  }

  // Item geometry and the first sub-block's K/V staging. Reads the position, the page table and
  // rows of earlier tokens only.
  __device__ __forceinline__ void prefetch(const KernelArgs& ka, AttnShared& sh, int item) {
    const AttnArgs& a = ka.a;
    split = item % ka.max_splits;
    kvh = (item / ka.max_splits) % kKvHeads;
    b = item / (ka.max_splits * kKvHeads);
    pos = a.pos[(size_t)b * a.pos_stride];
    if (pos >= (uint32_t)kMaxContext) {
      if (a.flags && threadIdx.x == 0 && split == 0 && kvh == 0)
        atomicOr(a.flags + (size_t)b * a.flags_stride, kFlagPosClamped);
      pos = kMaxContext - 1;
    }
    len = (int)pos + 1;
    nsplit = (len + ka.split - 1) / ka.split;
    valid = split < nsplit;
    if (!valid) return;
    l0 = split * ka.split;
    l1 = min(l0 + ka.split, len);
    owner = !a.kv_appended && (int)pos >= l0 && (int)pos < l1;
    pt = a.page_table + (size_t)b * a.page_table_stride;
    cst = attn_consts(a, pos);
    stage(ka, sh, l0, 0);
    stage(ka, sh, l0, 1);
  }

  __device__ __forceinline__ void run(const KernelArgs& ka, AttnShared& sh) {
    const AttnArgs& a = ka.a;
    if (!valid) return;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    attn_prologue(ka, sh, b, kvh, pos, owner, pt, cst);

    // This lane's 8 dims of q for the 4 heads stay in registers for the whole split.
    float q[kQPerKv][8];
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) {
      *reinterpret_cast<float4*>(&q[hh][0]) = *reinterpret_cast<const float4*>(&sh.q_s[hh][lane * 8]);
      *reinterpret_cast<float4*>(&q[hh][4]) = *reinterpret_cast<const float4*>(&sh.q_s[hh][lane * 8 + 4]);
    }
    float acc[kQPerKv][8];
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[hh][e] = 0.f;

    // K and V of a sub-block are separate cp.async groups, committed in the order K0 V0 K1 V1 ...:
    // K of the next sub-block streams in during this one's softmax and PV, V of the next during
    // its scores. At each wait the one newer group may stay in flight.
#pragma unroll 1
    for (int sb = l0; sb < l1; sb += kSub) {
      asm volatile("cp.async.wait_group 1;" ::: "memory");  // K(sb) has landed
      // Scores of this warp's 8 tokens (each lane reads only the chunks it staged).
#pragma unroll 1
      for (int i = 0; i < 8; ++i) {
        const int tk = warp * 8 + i, l = sb + tk;
        float kf[8];
        if (owner && l == (int)pos) {
          *reinterpret_cast<float4*>(kf) = *reinterpret_cast<const float4*>(&sh.kc_s[lane * 8]);
          *reinterpret_cast<float4*>(kf + 4) = *reinterpret_cast<const float4*>(&sh.kc_s[lane * 8 + 4]);
        } else {
          unpack8(*reinterpret_cast<const uint4*>(&sh.kst[tk][lane * 8]), kf);
        }
        float d[kQPerKv];
#pragma unroll
        for (int hh = 0; hh < kQPerKv; ++hh) {
          float p0 = q[hh][0] * kf[0], p1 = q[hh][4] * kf[4];
          p0 = fmaf(q[hh][1], kf[1], p0);
          p1 = fmaf(q[hh][5], kf[5], p1);
          p0 = fmaf(q[hh][2], kf[2], p0);
          p1 = fmaf(q[hh][6], kf[6], p1);
          p0 = fmaf(q[hh][3], kf[3], p0);
          p1 = fmaf(q[hh][7], kf[7], p1);
          d[hh] = warp_sum(p0 + p1);
        }
        if (lane == 0) {
#pragma unroll
          for (int hh = 0; hh < kQPerKv; ++hh) sh.sc[hh][tk] = (l < l1) ? d[hh] : -INFINITY;
        }
      }
      stage(ka, sh, sb + kSub, 0);  // this lane's K chunks are read: refill them with the next block
      __syncthreads();
      // Block max per head: thread (hh = t / 64, j = t % 64).
      {
        const int hh = t >> 6, j = t & 63;
        const float sval = sh.sc[hh][j];
        const float m = warp_max(sval);
        if (lane == 0) sh.red[warp][0] = m;
        __syncthreads();
        if (j == 0) {
          const float mb = fmaxf(sh.red[2 * hh][0], sh.red[2 * hh + 1][0]);
          const float mnew = fmaxf(sh.run_m[hh], mb);
          sh.blk_scale[hh] = (sh.run_m[hh] == -INFINITY) ? 0.f : expf(sh.run_m[hh] - mnew);
          sh.run_m[hh] = mnew;
        }
        __syncthreads();
        const float p = (sval == -INFINITY) ? 0.f : expf(sval - sh.run_m[hh]);
        sh.sc[hh][j] = p;
        const float ps = warp_sum(p);
        if (lane == 0) sh.red[warp][1] = ps;
        __syncthreads();
        if (j == 0) sh.run_l[hh] = sh.run_l[hh] * sh.blk_scale[hh] + sh.red[2 * hh][1] + sh.red[2 * hh + 1][1];
      }
#pragma unroll
      for (int hh = 0; hh < kQPerKv; ++hh) {
        const float f = sh.blk_scale[hh];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[hh][e] *= f;
      }
      asm volatile("cp.async.wait_group 1;" ::: "memory");  // V(sb) has landed
#pragma unroll 1
      for (int i = 0; i < 8; ++i) {
        const int tk = warp * 8 + i, l = sb + tk;
        if (l < l1) {
          float vf[8];
          if (owner && l == (int)pos) {
            *reinterpret_cast<float4*>(vf) = *reinterpret_cast<const float4*>(&sh.vc_s[lane * 8]);
            *reinterpret_cast<float4*>(vf + 4) = *reinterpret_cast<const float4*>(&sh.vc_s[lane * 8 + 4]);
          } else {
            unpack8(*reinterpret_cast<const uint4*>(&sh.vst[tk][lane * 8]), vf);
          }
#pragma unroll
          for (int hh = 0; hh < kQPerKv; ++hh) {
            const float p = sh.sc[hh][tk];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[hh][e] = fmaf(p, vf[e], acc[hh][e]);
          }
        }
      }
      stage(ka, sh, sb + kSub, 1);  // and the V chunks
      __syncthreads();  // sh.sc is rewritten by the next sub-block
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // (only empty groups remain)
    __syncthreads();  // accw reuses the K area

    // Merge the 8 warps' accumulators and write this split's partial.
#pragma unroll
    for (int hh = 0; hh < kQPerKv; ++hh) {
      *reinterpret_cast<float4*>(sh.accw(warp) + hh * kHeadDim + lane * 8) = *reinterpret_cast<float4*>(&acc[hh][0]);
      *reinterpret_cast<float4*>(sh.accw(warp) + hh * kHeadDim + lane * 8 + 4) = *reinterpret_cast<float4*>(&acc[hh][4]);
    }
    __syncthreads();
    const int hh = t >> 6, d0 = (t & 63) * 4;  // merge mapping
    float4 o;
    o.x = o.y = o.z = o.w = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float4 v = *reinterpret_cast<const float4*>(sh.accw(w) + hh * kHeadDim + d0);
      o.x += v.x;
      o.y += v.y;
      o.z += v.z;
      o.w += v.w;
    }
    attn_merge_store(a, sh, b, kvh, split, nsplit, o, 0, ka.spread != 0);
  }
};

}  // namespace dev
}  // namespace qne
