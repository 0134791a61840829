// Device-side building blocks of the B = 1 GEMV kernels, shared by the per-kernel path
// (gemv.cu) and the persistent decode kernel (persist.cu): input staging with the fused
// prologues, chunk dot products, the pipelined register-streaming f16 GEMV, and the greedy-pick
// reduction across CTAs.
#pragma once

#include <math.h>

#include "common.cuh"
#include "gemv.cuh"

namespace qne {
namespace dev {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kPrefetchBytes = 96u << 10;  // per CTA, issued before the dependency wait
constexpr uint32_t kPrefetchPiece = 8u << 10;

template <int KIND>
struct Fmt;
template <>
struct Fmt<kF16> {
  static constexpr int CV = 8;  // values per 16-byte chunk
  static __host__ __device__ size_t row_bytes(int k) { return (size_t)k * 2; }
};
template <>
struct Fmt<kQ4> {
  static constexpr int CV = 32;
  static __host__ __device__ size_t row_bytes(int k) { return (size_t)k / 2; }
};
template <>
struct Fmt<kQ4G64> {
  static constexpr int CV = 32;
  static __host__ __device__ size_t row_bytes(int k) { return (size_t)k / 2; }
};

// Dequantized value of element (row, i) - the unpack used by dequant_rows and the embedding.
__device__ __forceinline__ float deq_elem(const Mat& m, long row, int i) {
  if (m.kind == kF16) {
    return h2f(__ldg((const uint16_t*)m.w + row * m.k + i));
  }
  const uint32_t word = __ldg((const uint32_t*)m.w + row * (m.k / 8) + i / 8);
  const float q = nib_f(word, 4 * (i % 8));
  float scale, zp;
  if (m.kind == kQ4) {
    q4_scale_zp((const uint32_t*)m.s, (const uint32_t*)m.z, row, m.k, i / 32, scale, zp);
  } else {
    q4g64_scale_zp((const uint16_t*)m.s, (const uint16_t*)m.z, row, m.k, i / 64, scale, zp);
  }
  return (q - zp) * scale;
}

// Issues L2 prefetches of rows [r0, r1) (up to `budget` bytes); called by one warp.
__device__ __forceinline__ void prefetch_rows(const uint8_t* base, size_t row_bytes, long r0,
                                              long r1, uint32_t budget, int lane) {
  if (r1 <= r0) return;
  size_t bytes = (size_t)(r1 - r0) * row_bytes;
  if (bytes > budget) bytes = budget;
  bytes &= ~(size_t)15;
  const uint8_t* p = base + (size_t)r0 * row_bytes;
#pragma unroll 1
  for (size_t off = (size_t)lane * kPrefetchPiece; off < bytes; off += 32 * kPrefetchPiece) {
    const size_t n = bytes - off < kPrefetchPiece ? bytes - off : kPrefetchPiece;
    prefetch_l2(p + off, (uint32_t)n);
  }
}

// Barrier over the 256 threads that stage x: the whole CTA (register kernel) or the consumer
// warps only (bulk-copy kernel, whose producer warp never joins).
struct CtaSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};
struct ConsumerSync {
  __device__ __forceinline__ void operator()() const { asm volatile("bar.sync 1, 256;" ::: "memory"); }
};

template <typename Sync>
__device__ __forceinline__ float sum256(float v, float* red, Sync sync) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  sync();
  if (l == 0) red[w] = v;
  sync();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) t += red[i];
  return t;
}

// ------------------------------------------------------------------------------------------
// Prologues: stage the f32 input vector of length k in shared memory.
// ------------------------------------------------------------------------------------------
template <int PRO, typename Sync = CtaSync>
__device__ __forceinline__ void stage_x(const GemvArgs& a, float* xs, float* red, Sync sync = Sync()) {
  const int k = a.m.k;
  const int tid = threadIdx.x;
  if (PRO == kProCopy) {
    for (int i = tid * 4; i < k; i += kThreads * 4)
      *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(a.x + i);
  } else if (PRO == kProRmsNorm || PRO == kProEmbedNorm) {
    float ss = 0.f;
    if (PRO == kProRmsNorm) {
      for (int i = tid * 4; i < k; i += kThreads * 4) {
        const float4 v = *reinterpret_cast<const float4*>(a.x + i);
        *reinterpret_cast<float4*>(xs + i) = v;
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
    } else {
      // Embedding row of the token the previous step picked (or the host wrote).
      uint32_t token = a.ctl->token;
      if (token >= (uint32_t)a.embed.rows) token = (uint32_t)a.embed.rows - 1;
      for (int i = tid; i < k; i += kThreads) {
        const float v = deq_elem(a.embed, token, i);
        xs[i] = v;
        ss += v * v;
      }
      if (blockIdx.x == 0) {
        for (int i = tid; i < k; i += kThreads) a.h_out[i] = xs[i];
        if (tid == 0) a.ctl->count += 1;  // one more token entered the conv windows
      }
    }
    const float tot = sum256(ss, red, sync);
    const float inv = rsqrtf(tot / (float)k + a.eps);
    for (int i = tid; i < k; i += kThreads) xs[i] = xs[i] * inv * a.norm_w[i];
  } else if (PRO == kProGdnGate) {
    // k == 2048: 16 heads of 128; warp w normalizes heads 2w and 2w+1.
    const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int head = warp * 2 + hh;
      const int base = head * kGdnDim + lane * 4;
      const float4 v = *reinterpret_cast<const float4*>(a.x + base);
      const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
      const float inv = rsqrtf(ss / (float)kGdnDim + a.eps);
      const float4 zz = *reinterpret_cast<const float4*>(a.zgate + base);
      const float4 nw = *reinterpret_cast<const float4*>(a.norm_w + lane * 4);
      xs[base + 0] = v.x * inv * silu(zz.x) * nw.x;
      xs[base + 1] = v.y * inv * silu(zz.y) * nw.y;
      xs[base + 2] = v.z * inv * silu(zz.z) * nw.z;
      xs[base + 3] = v.w * inv * silu(zz.w) * nw.w;
    }
  }
  sync();
}

// ------------------------------------------------------------------------------------------
// One-pass staging (the default kernels). The prologue operand that depends on nothing (the
// norm weight) is loaded into registers before the dependency wait (pre_norm); after the wait
// every thread loads its chunks of x at once, applies the prologue and writes the layout the
// streaming loop reads, so a GEMV pays one round trip to L2 and one barrier between its release
// and its first dot product. RMSNorm is folded: the staged values are x * norm_w and the
// returned factor rsqrt(mean(x^2) + eps) scales the dot products in the epilogue (1 for the
// other prologues, which are applied in full).
// ------------------------------------------------------------------------------------------
constexpr int kStageChunks = 3;  // 8-element chunks per thread loaded together (k <= 6144)

// The norm weight of this thread's first chunk (chunk c = threadIdx.x; the gated GDN norm
// repeats its 128 weights per head).
template <int PRO>
__device__ __forceinline__ void pre_norm(const GemvArgs& a, float (&nw)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) nw[j] = 1.f;
  if (PRO == kProCopy || (int)threadIdx.x >= a.m.k / 8) return;
  const float* src = (PRO == kProGdnGate) ? a.norm_w + ((threadIdx.x * 8) & (kGdnDim - 1)) : a.norm_w + threadIdx.x * 8;
  const float4 p = __ldg(reinterpret_cast<const float4*>(src));
  const float4 q = __ldg(reinterpret_cast<const float4*>(src + 4));
  nw[0] = p.x; nw[1] = p.y; nw[2] = p.z; nw[3] = p.w;
  nw[4] = q.x; nw[5] = q.y; nw[6] = q.z; nw[7] = q.w;
}

__device__ __forceinline__ void ldcg8(float (&v)[8], const float* s) {
  const float4 p = __ldcg(reinterpret_cast<const float4*>(s));
  const float4 q = __ldcg(reinterpret_cast<const float4*>(s + 4));
  v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
  v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  return (uint32_t)__half_as_ushort(__float2half_rn(lo)) | ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
}

// Stages x (prologue applied, RMSNorm folded) in one pass and returns the folded factor.
// OUT = 0: f32 planes, xp[4c ..] = elements 0-3 and xp[k/2 + 4c ..] = elements 4-7 of chunk c.
// OUT = 1: f16 pair planes for the int4 tensor-core kernel, uint4 hi[c] = (v0,v4),(v1,v5),
// (v2,v6),(v3,v7) as f16x2 of f16(v), lo[c] the same of f16(v - f16(v)), lo at hi + k/8; and
// when csum is set, the sums of every `group` consecutive chunks (one quantization block).
// Norm prologues need k <= 8 * kThreads (one chunk per thread; the gated norm k == 2048).
template <int PRO, int OUT, typename Sync>
__device__ __forceinline__ float stage_fold(const GemvArgs& a, void* planes, float* red, const float (&nw)[8],
                                            Sync sync, float* csum = nullptr, int group = 1) {
  const int k = a.m.k, nc = k / 8, tid = threadIdx.x;
  constexpr bool kNorm = PRO == kProRmsNorm || PRO == kProEmbedNorm;
  // chunks per thread and round: the norm prologues stage k <= 2048 (one chunk per thread)
  constexpr int NCH = PRO == kProCopy ? kStageChunks : 1;
  uint32_t token = 0;
  if (PRO == kProEmbedNorm) {
    token = a.ctl->token;
    if (token >= (uint32_t)a.embed.rows) token = (uint32_t)a.embed.rows - 1;
  }
  float ss = 0.f;
#pragma unroll 1
  for (int c0 = 0; c0 < nc; c0 += kThreads * NCH) {
    float v[NCH][8];
    // every load of this round first
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int c = c0 + tid + i * kThreads;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
      if (c < nc) {
        if (PRO == kProEmbedNorm) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = deq_elem(a.embed, token, c * 8 + j);
        } else {
          ldcg8(v[i], a.x + c * 8);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int c = c0 + tid + i * kThreads;
      const bool in = c < nc;
      if (PRO == kProEmbedNorm && in && blockIdx.x == 0) {
        *reinterpret_cast<float4*>(a.h_out + c * 8) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        *reinterpret_cast<float4*>(a.h_out + c * 8 + 4) = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
      }
      float cs = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) cs = fmaf(v[i][j], v[i][j], cs);
      if (kNorm) {
        ss += cs;
        float w[8];
        if (c0 == 0 && i == 0) {
#pragma unroll
          for (int j = 0; j < 8; ++j) w[j] = nw[j];
        } else if (in) {
          ldcg8(w, a.norm_w + c * 8);
        }
        if (in) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] *= w[j];
        }
      } else if (PRO == kProGdnGate) {
        // k == 2048: one chunk per thread, 16 consecutive threads per 128-wide head
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
        const float inv = rsqrtf(cs / (float)kGdnDim + a.eps);
        float z[8];
        ldcg8(z, a.zgate + c * 8);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = v[i][j] * inv * silu(z[j]) * nw[j];
      }
      if (OUT == 0) {
        if (in) {
          float* xp = static_cast<float*>(planes);
          *reinterpret_cast<float4*>(xp + c * 4) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
          *reinterpret_cast<float4*>(xp + k / 2 + c * 4) = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
        }
      } else {
        if (in) {
          uint4* xq = static_cast<uint4*>(planes);
          float lo[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) lo[j] = v[i][j] - __half2float(__float2half_rn(v[i][j]));
          xq[c] = make_uint4(pack_h2(v[i][0], v[i][4]), pack_h2(v[i][1], v[i][5]), pack_h2(v[i][2], v[i][6]),
                             pack_h2(v[i][3], v[i][7]));
          xq[nc + c] = make_uint4(pack_h2(lo[0], lo[4]), pack_h2(lo[1], lo[5]), pack_h2(lo[2], lo[6]), pack_h2(lo[3], lo[7]));
        }
        if (csum) {
          // chunks of one block sit in consecutive lanes (c0 and i * kThreads are multiples of 32)
          float s = ((v[i][0] + v[i][1]) + (v[i][2] + v[i][3])) + ((v[i][4] + v[i][5]) + (v[i][6] + v[i][7]));
          for (int o = 1; o < group; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          if (in && (c % group) == 0) csum[c / group] = s;
        }
      }
    }
  }
  if (PRO == kProEmbedNorm && blockIdx.x == 0 && tid == 0) a.ctl->count += 1;  // conv windows
  if (kNorm) {
    const float t = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = t;
  }
  sync();
  if (!kNorm) return 1.f;
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) t += red[w];
  return rsqrtf(t / (float)k + a.eps);
}

// ------------------------------------------------------------------------------------------
// Chunk dot products: 16 bytes of one row against the matching slice of x in shared memory.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float dot_f16(const uint4& w, const float* x) {
  const float2 a = h2f2(w.x), b = h2f2(w.y), c = h2f2(w.z), d = h2f2(w.w);
  float p0 = a.x * x[0];
  float p1 = b.x * x[2];
  float p2 = c.x * x[4];
  float p3 = d.x * x[6];
  p0 = fmaf(a.y, x[1], p0);
  p1 = fmaf(b.y, x[3], p1);
  p2 = fmaf(c.y, x[5], p2);
  p3 = fmaf(d.y, x[7], p3);
  return (p0 + p1) + (p2 + p3);
}

// sum_n q_n x_n over the 32 nibbles of a chunk (q exact as floats).
__device__ __forceinline__ float dot_q4_raw(const uint4& w, const float* x) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  float p[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float s = nib_f(ws[e], 0) * x[8 * e];
#pragma unroll
    for (int n = 1; n < 8; ++n) s = fmaf(nib_f(ws[e], 4 * n), x[8 * e + n], s);
    p[e] = s;
  }
  return (p[0] + p[1]) + (p[2] + p[3]);
}


// Shared memory a GEMV CTA needs besides the staged input.
struct GemvShared {
  float red[kWarps];
  float bval[kWarps];
  uint32_t bidx[kWarps];
  uint32_t is_last;
};

// f16 GEMV, pipelined register streaming.
//
// Rows are dealt round-robin to every warp of the grid (warp w takes rows w, w + W, ...), so
// all warps get the same number of rows within one. A row is processed in segments of at most
// 2048 elements (1024 for SwiGLU, whose unit is a gate row plus its up row); while one segment
// is multiplied, the next segment's 16-byte loads are already in flight in a second register
// buffer. prefetch() issues the first segment's loads: it touches weights only, so callers run
// it before waiting on the producer of x.
template <int PRO, int EPI>
struct Pipe {
  static constexpr bool SW = (EPI == kSwiGlu);
  static constexpr int CPL = SW ? 4 : 8;  // chunks per lane per segment (max)
  static constexpr int R = SW ? 2 : 1;    // rows per unit
  int k, seg, nseg, cpl, out_rows, gw, nw, my_rows, units, lane;
  long half;
  size_t rb;
  const uint8_t* W;
  uint4 cur[R][CPL];
  float normw[8];  // norm weight of this thread's chunk of x, loaded before the dependency wait

  __device__ __forceinline__ void init(const GemvArgs& a, int cta, int ncta) {
    k = a.m.k;
    cpl = CPL;  // segment = 256 * d elements, d the largest divisor of k / 256 not above CPL
    while ((k / 256) % cpl) --cpl;
    seg = cpl * 256;
    nseg = k / seg;
    out_rows = SW ? a.m.rows / 2 : a.m.rows;
    half = SW ? a.m.rows / 2 : 0;
    rb = (size_t)k * 2;
    W = static_cast<const uint8_t*>(a.m.w);
    lane = threadIdx.x & 31;
    gw = cta * kWarps + (threadIdx.x >> 5);
    nw = ncta * kWarps;
    my_rows = (out_rows > gw) ? (out_rows - gw + nw - 1) / nw : 0;
    units = my_rows * nseg;
  }

  __device__ __forceinline__ void load(uint4 (&buf)[R][CPL], int u) const {
    const long row = gw + (long)(u / nseg) * nw;
    const int sg = u % nseg;
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      const uint8_t* base = W + (size_t)(rr ? half + row : row) * rb + (size_t)sg * seg * 2;
#pragma unroll
      for (int c = 0; c < CPL; ++c)
        buf[rr][c] = (c < cpl) ? ld_stream(base + (size_t)(lane + 32 * c) * 16) : make_uint4(0u, 0u, 0u, 0u);
    }
  }

  // First unit into registers, and the norm weight of the prologue. (A bulk L2 prefetch of the
  // warp's next rows here was measured and makes the decode step slower: it competes with the
  // demand stream instead of filling gaps.)
  __device__ __forceinline__ void prefetch(const GemvArgs& a) {
    if (units > 0) load(cur, 0);
    pre_norm<PRO>(a, normw);
  }

  // Stages x (prologue, one pass), then streams every unit. For kArgmax the lane-0 best
  // candidate of each warp lands in sh.bval / sh.bidx.
  __device__ __forceinline__ void run(const GemvArgs& a, float* xs, GemvShared& sh) {
    const int warp = threadIdx.x >> 5;
    float* xp = xs;  // planes: elements 0-3 and 4-7 of every 8-element chunk
    const float inv = stage_fold<PRO, 0>(a, xp, sh.red, normw, CtaSync());
    float best_v = -INFINITY;
    uint32_t best_i = 0xFFFFFFFFu;
    float acc[R];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) acc[rr] = 0.f;
    uint4 nxt[R][CPL];
    for (int u = 0; u < units; ++u) {
      if (u + 1 < units) load(nxt, u + 1);
      const int sg = u % nseg;
      const float* xlo = xp + (size_t)sg * (seg / 2);
      const float* xhi = xp + k / 2 + (size_t)sg * (seg / 2);
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        if (c < cpl) {
          const int ci = lane + 32 * c;
          float xv[8];
          *reinterpret_cast<float4*>(xv) = *reinterpret_cast<const float4*>(xlo + ci * 4);
          *reinterpret_cast<float4*>(xv + 4) = *reinterpret_cast<const float4*>(xhi + ci * 4);
#pragma unroll
          for (int rr = 0; rr < R; ++rr) acc[rr] += dot_f16(cur[rr][c], xv);
        }
      }
      if (sg == nseg - 1) {
        const long row = gw + (long)(u / nseg) * nw;
        float v[R];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          v[rr] = warp_sum(acc[rr]) * inv;
          acc[rr] = 0.f;
        }
        if (EPI == kArgmax && v[0] > -INFINITY && (v[0] > best_v || (v[0] == best_v && (uint32_t)row < best_i))) {
          best_v = v[0];
          best_i = (uint32_t)row;
        }
        if (lane == 0) {
          if (SW) a.y[row] = silu(v[0]) * v[R - 1];
          else if (EPI == kAccumulate) a.y[row] += v[0];
          else a.y[row] = v[0];
        }
      }
#pragma unroll
      for (int rr = 0; rr < R; ++rr)
#pragma unroll
        for (int c = 0; c < CPL; ++c) cur[rr][c] = nxt[rr][c];
    }
    if (EPI == kArgmax && lane == 0) {
      sh.bval[warp] = best_v;
      sh.bidx[warp] = best_i;
    }
  }
};

// Prologue of the fused-kernel GEMV, chosen at run time: stages x of length k directly in the
// plane layout the streaming loop reads (for every 8-element chunk c, elements 0-3 at
// xp[4c..4c+3] and 4-7 at xp[k/2 + 4c..]), applying the copy, RMSNorm, embedding + RMSNorm or
// gated GDN RMSNorm prologue. One code path for all four keeps the fused kernels small.
__device__ __forceinline__ void stage_planes(const GemvArgs& a, int pro, float* xp, float* red) {
  const int k = a.m.k, tid = threadIdx.x, nc = k / 8;
  float ss = 0.f;
  uint32_t token = 0;
  if (pro == kProEmbedNorm) {
    token = a.ctl->token;
    if (token >= (uint32_t)a.embed.rows) token = (uint32_t)a.embed.rows - 1;
  }
#pragma unroll 1
  for (int c = tid; c < nc; c += kThreads) {
    float v[8];
    if (pro == kProEmbedNorm) {
#pragma unroll 1
      for (int j = 0; j < 8; ++j) v[j] = deq_elem(a.embed, token, c * 8 + j);
      if (blockIdx.x == 0) {
        *reinterpret_cast<float4*>(a.h_out + c * 8) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(a.h_out + c * 8 + 4) = make_float4(v[4], v[5], v[6], v[7]);
      }
    } else {
      *reinterpret_cast<float4*>(v) = *reinterpret_cast<const float4*>(a.x + c * 8);
      *reinterpret_cast<float4*>(v + 4) = *reinterpret_cast<const float4*>(a.x + c * 8 + 4);
    }
    float cs = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) cs = fmaf(v[j], v[j], cs);
    if (pro == kProGdnGate) {
      // k == 2048: one chunk per thread, 16 chunks (16 aligned lanes) per 128-wide head.
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
      const float inv = rsqrtf(cs / (float)kGdnDim + a.eps);
      const int d = (c * 8) & (kGdnDim - 1);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = v[j] * inv * silu(a.zgate[c * 8 + j]) * a.norm_w[d + j];
    }
    ss += cs;
    *reinterpret_cast<float4*>(xp + c * 4) = *reinterpret_cast<const float4*>(v);
    *reinterpret_cast<float4*>(xp + k / 2 + c * 4) = *reinterpret_cast<const float4*>(v + 4);
  }
  if (pro == kProRmsNorm || pro == kProEmbedNorm) {
    if (pro == kProEmbedNorm && blockIdx.x == 0 && tid == 0) a.ctl->count += 1;  // conv windows
    const float inv = rsqrtf(sum256(ss, red, CtaSync()) / (float)k + a.eps);
#pragma unroll 1
    for (int c = tid; c < nc; c += kThreads) {
      const float4 w0 = *reinterpret_cast<const float4*>(a.norm_w + c * 8);
      const float4 w1 = *reinterpret_cast<const float4*>(a.norm_w + c * 8 + 4);
      float4 lo = *reinterpret_cast<float4*>(xp + c * 4), hi = *reinterpret_cast<float4*>(xp + k / 2 + c * 4);
      lo.x *= inv * w0.x; lo.y *= inv * w0.y; lo.z *= inv * w0.z; lo.w *= inv * w0.w;
      hi.x *= inv * w1.x; hi.y *= inv * w1.y; hi.z *= inv * w1.z; hi.w *= inv * w1.w;
      *reinterpret_cast<float4*>(xp + c * 4) = lo;
      *reinterpret_cast<float4*>(xp + k / 2 + c * 4) = hi;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// f16 GEMV for the fused layer kernels: one code path for every prologue and epilogue (chosen
// at run time), so a fused kernel holds a single streaming loop. A unit is two rows times one
// segment of at most 1024 elements: a gate row and its up row for SwiGLU, else two rows of the
// warp's round-robin share (rows gw + t * nw). Each warp streams its units through a ring of
// kSlots unit-sized slots in shared memory with 16-byte cp.async copies; every lane later reads
// exactly the bytes it copied, so the ring needs no synchronization beyond cp.async groups.
// prefetch() fills the ring before the caller waits for x, so the next phase's first 8 KB per
// warp (19 MB over the grid) stream from DRAM across the grid barrier and the prologue.
struct RingPipe {
  static constexpr int CPL = 4;
  static constexpr int kSlots = 2;
  static constexpr int kSlotBytes = 2 * CPL * 512;  // two row segments of up to 1024 f16
  static constexpr int kRingBytes = kWarps * kSlots * kSlotBytes;  // per CTA
  int k, seg, nseg, cpl, gw, nw, my_rows, pairs, units, lane, epi, pro;
  long half;
  size_t rb;
  const uint8_t* W;
  uint8_t* ring;

  __device__ __forceinline__ void init(const GemvArgs& a, int cta, int ncta, uint8_t* ring_base) {
    pro = a.pro;
    epi = a.epi;
    k = a.m.k;
    cpl = CPL;
    while ((k / 256) % cpl) --cpl;
    seg = cpl * 256;
    nseg = k / seg;
    const bool sw = epi == kSwiGlu;
    const int out_rows = sw ? a.m.rows / 2 : a.m.rows;
    half = sw ? a.m.rows / 2 : 0;
    rb = (size_t)k * 2;
    W = static_cast<const uint8_t*>(a.m.w);
    lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    gw = cta * kWarps + warp;
    nw = ncta * kWarps;
    my_rows = (out_rows > gw) ? (out_rows - gw + nw - 1) / nw : 0;
    pairs = sw ? my_rows : (my_rows + 1) / 2;
    units = pairs * nseg;
    ring = ring_base + (size_t)warp * kSlots * kSlotBytes;
  }

  // Row of slot rr (0, 1) of pair j, or -1 when the pair has a single row.
  __device__ __forceinline__ long row_of(int j, int rr) const {
    if (epi == kSwiGlu) return (long)gw + (long)j * nw + (rr ? half : 0);
    const int t = 2 * j + rr;
    return t < my_rows ? (long)gw + (long)t * nw : -1;
  }

  // Copies unit u into its slot (nothing past the last unit) and commits one group.
  __device__ __forceinline__ void issue(int u) const {
    if (u < units) {
      uint8_t* slot = ring + (u % kSlots) * kSlotBytes;
      const int j = u / nseg, sg = u % nseg;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const long row = row_of(j, rr);
        if (row >= 0) {
          const uint8_t* src = W + (size_t)row * rb + (size_t)sg * seg * 2;
#pragma unroll
          for (int c = 0; c < CPL; ++c)
            if (c < cpl) cp_async16(slot + rr * seg * 2 + (lane + 32 * c) * 16, src + (size_t)(lane + 32 * c) * 16);
        }
      }
    }
    cp_async_commit();
  }

  __device__ __forceinline__ void prefetch() const {
#pragma unroll
    for (int u = 0; u < kSlots; ++u) issue(u);
  }

  __device__ __forceinline__ void run(const GemvArgs& a, float* xs, GemvShared& sh) {
    const int warp = threadIdx.x >> 5;
    stage_planes(a, pro, xs, sh.red);
    const float* xp = xs;
    float best_v = -INFINITY;
    uint32_t best_i = 0xFFFFFFFFu;
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 1
    for (int u = 0; u < units; ++u) {
      cp_async_wait<kSlots - 1>();
      const uint8_t* slot = ring + (u % kSlots) * kSlotBytes;
      const int j = u / nseg, sg = u % nseg;
      const bool two = row_of(j, 1) >= 0;
      const float* xlo = xp + (size_t)sg * (seg / 2);
      const float* xhi = xp + k / 2 + (size_t)sg * (seg / 2);
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        if (c < cpl) {
          const int ci = lane + 32 * c;
          float xv[8];
          *reinterpret_cast<float4*>(xv) = *reinterpret_cast<const float4*>(xlo + ci * 4);
          *reinterpret_cast<float4*>(xv + 4) = *reinterpret_cast<const float4*>(xhi + ci * 4);
          acc0 += dot_f16(*reinterpret_cast<const uint4*>(slot + ci * 16), xv);
          if (two) acc1 += dot_f16(*reinterpret_cast<const uint4*>(slot + seg * 2 + ci * 16), xv);
        }
      }
      issue(u + kSlots);  // the slot just read is refilled (each lane reuses only its own bytes)
      if (sg == nseg - 1) {
        const float v0 = warp_sum(acc0), v1 = warp_sum(acc1);
        acc0 = acc1 = 0.f;
        if (epi == kSwiGlu) {
          if (lane == 0) a.y[gw + (long)j * nw] = silu(v0) * v1;
        } else {
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const long row = row_of(j, rr);
            const float v = rr ? v1 : v0;
            if (row >= 0) {
              if (epi == kArgmax && v > -INFINITY && (v > best_v || (v == best_v && (uint32_t)row < best_i))) {
                best_v = v;
                best_i = (uint32_t)row;
              }
              if (lane == 0) {
                if (epi == kAccumulate) a.y[row] += v;
                else a.y[row] = v;
              }
            }
          }
        }
      }
    }
    cp_async_wait<0>();
    if (epi == kArgmax && lane == 0) {
      sh.bval[warp] = best_v;
      sh.bidx[warp] = best_i;
    }
  }
};

// ------------------------------------------------------------------------------------------
// int4 GEMV (block-32 and group-64 layouts), B = 1.
//
// A chunk is 16 bytes of one row: 32 nibbles, the values k = 32c .. 32c + 31. Rows are dealt
// round-robin to the warps of the grid like the f16 pipeline; a unit is `rpu` output rows (their
// gate and up rows for SwiGLU) packed into kSlots chunk slots per lane, lane l holding chunks
// l, l + 32, ... of each row. At the decode shapes one unit is a warp's whole share of a layer
// matrix (3-6 KB), so prefetch() - issued before the wait on the previous kernel - loads all of
// it, with the chunks' scales and zero points, in a single DRAM round trip. Longer shares (an
// int4 LM head) stream unit by unit (one buffer: a second one costs spills at 128 registers).
// ------------------------------------------------------------------------------------------

// sum_n q_n x_n over the 32 nibbles of chunk c. x is staged transposed in shared memory as
// xt[q][c] = x[32c + 4q .. 32c + 4q + 3] (float4), so the 32 lanes of a warp, which hold 32
// consecutive chunks, read 32 consecutive float4 for each q: no bank conflicts.
__device__ __forceinline__ float dot_q4_chunk(const uint4& w, const float4* xt, int nch, int c) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  float p[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float4 a = xt[(size_t)(2 * e) * nch + c];
    const float4 b = xt[(size_t)(2 * e + 1) * nch + c];
    float t = nib_f(ws[e], 0) * a.x;
    t = fmaf(nib_f(ws[e], 4), a.y, t);
    t = fmaf(nib_f(ws[e], 8), a.z, t);
    t = fmaf(nib_f(ws[e], 12), a.w, t);
    t = fmaf(nib_f(ws[e], 16), b.x, t);
    t = fmaf(nib_f(ws[e], 20), b.y, t);
    t = fmaf(nib_f(ws[e], 24), b.z, t);
    p[e] = fmaf(nib_f(ws[e], 28), b.w, t);
  }
  return (p[0] + p[1]) + (p[2] + p[3]);
}

template <int KIND, int PRO, int EPI>
struct Q4Pipe {
  static constexpr bool SW = (EPI == kSwiGlu);
  static constexpr int PH = SW ? 2 : 1;  // physical rows per output row
  static constexpr int kSlots = 8;       // 16-byte chunks per lane per unit
  int k, nch, cpl, rpu, out_rows, gw, nw, my_rows, units, lane;
  long half;
  size_t rb;
  const uint8_t* W;
  uint32_t meta;  // per slot s, bits 4s..4s+3: output row in the unit (3 bits) | up row (bit 3)
  uint32_t cj;    // per slot s, bits 4s..4s+3: chunk column j (chunk = 32 j + lane)
  uint4 cur[kSlots];
  uint32_t cs[kSlots], cz[kSlots];  // raw scale / zero-point words of each slot's chunk

  __device__ __forceinline__ void init(const GemvArgs& a, int cta, int ncta) {
    k = a.m.k;
    nch = k / 32;
    cpl = (nch + 31) / 32;  // chunks per lane per row (the launcher guarantees cpl * PH <= kSlots)
    rpu = kSlots / (cpl * PH);
    out_rows = SW ? a.m.rows / 2 : a.m.rows;
    half = SW ? a.m.rows / 2 : 0;
    rb = (size_t)k / 2;
    W = static_cast<const uint8_t*>(a.m.w);
    lane = threadIdx.x & 31;
    gw = cta * kWarps + (threadIdx.x >> 5);
    nw = ncta * kWarps;
    my_rows = (out_rows > gw) ? (out_rows - gw + nw - 1) / nw : 0;
    units = (my_rows + rpu - 1) / rpu;
    meta = 0u;
    cj = 0u;
#pragma unroll 1
    for (int s = 0; s < kSlots; ++s) {  // the only divisions by the runtime row geometry
      const int q = s / (cpl * PH), which = (s / cpl) % PH, j = s % cpl;
      meta |= (uint32_t)((q > 7 ? 7 : q) | (which << 3)) << (4 * s);
      cj |= (uint32_t)j << (4 * s);
    }
  }

  __device__ __forceinline__ int slot_q(int s) const { return (int)((meta >> (4 * s)) & 7u); }
  __device__ __forceinline__ bool slot_up(int s) const { return (meta >> (4 * s + 3)) & 1u; }

  // Slot s of unit u: output row t (or -1), physical row, chunk index c (or -1 past the row).
  __device__ __forceinline__ void slot(int u, int s, int& t, long& row, int& c) const {
    const int q = slot_q(s), which = slot_up(s) ? 1 : 0, j = (int)((cj >> (4 * s)) & 15u);
    t = u * rpu + q;
    c = j * 32 + lane;
    if (q >= rpu || t >= my_rows || c >= nch) {
      t = -1;
      c = -1;
      row = 0;
      return;
    }
    row = (long)gw + (long)t * nw + (which ? half : 0);
  }

  __device__ __forceinline__ void load(const GemvArgs& a, int u) {
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
      int t, c;
      long row;
      slot(u, s, t, row, c);
      cur[s] = make_uint4(0u, 0u, 0u, 0u);
      cs[s] = 0u;
      cz[s] = 0u;
      if (t >= 0) {
        cur[s] = ld_stream(W + (size_t)row * rb + (size_t)c * 16);
        if (KIND == kQ4) {  // block-32: f16 scale pair per 64 values, zero-point nibbles per 256
          cs[s] = __ldg(static_cast<const uint32_t*>(a.m.s) + row * (k / 64) + c / 2);
          cz[s] = __ldg(static_cast<const uint32_t*>(a.m.z) + row * (k / 256) + c / 8);
        } else {  // group-64: f16 scale and f16 zero point per 64 values
          cs[s] = __ldg(static_cast<const uint16_t*>(a.m.s) + row * (k / 64) + c / 2);
          cz[s] = __ldg(static_cast<const uint16_t*>(a.m.z) + row * (k / 64) + c / 2);
        }
      }
    }
  }

  // The first unit (at decode shapes the warp's whole share) into registers: weights and their
  // quantization parameters only, so callers issue it before waiting on the producer of x.
  __device__ __forceinline__ void prefetch(const GemvArgs& a) {
    if (units > 0) load(a, 0);
  }

  __device__ __forceinline__ void decode(uint32_t sw, uint32_t zw, int c, float& scale, float& zp) const {
    if (KIND == kQ4) {
      scale = h2f((uint16_t)((c & 1) ? (sw >> 16) : (sw & 0xFFFFu)));
      zp = (float)((zw >> (4 * (c % 8))) & 15u);
    } else {
      scale = h2f((uint16_t)sw);
      zp = h2f((uint16_t)zw);
    }
  }

  // Stages x (prologue) transposed plus its per-chunk sums, then every unit: per chunk
  // scale * (sum q x - zp * sum x), summed per output row and reduced over the warp. For kArgmax
  // the lane-0 best candidate of each warp lands in sh.bval / sh.bidx.
  __device__ __forceinline__ void run(const GemvArgs& a, float* xs, GemvShared& sh) {
    const int warp = threadIdx.x >> 5;
    stage_x<PRO>(a, xs, sh.red);
    float4* xt = reinterpret_cast<float4*>(xs + k);  // [8][nch] float4, then [nch] chunk sums
    float* xsum = xs + 2 * k;
    for (int c = threadIdx.x; c < nch; c += kThreads) {
      float t = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(xs + c * 32 + 4 * q);
        xt[(size_t)q * nch + c] = v;
        t += (v.x + v.y) + (v.z + v.w);
      }
      xsum[c] = t;
    }
    __syncthreads();
    float best_v = -INFINITY;
    uint32_t best_i = 0xFFFFFFFFu;
    for (int u = 0; u < units; ++u) {
      if (u > 0) load(a, u);  // unit 0 came from prefetch()
      float acc[kSlots];
#pragma unroll
      for (int s = 0; s < kSlots; ++s) {
        int t, c;
        long row;
        slot(u, s, t, row, c);
        acc[s] = 0.f;
        if (t >= 0) {
          float scale, zp;
          decode(cs[s], cz[s], c, scale, zp);
          acc[s] = scale * (dot_q4_chunk(cur[s], xt, nch, c) - zp * xsum[c]);
        }
      }
#pragma unroll
      for (int q = 0; q < kSlots; ++q) {
        const int t = u * rpu + q;
        if (q < rpu && t < my_rows) {  // warp-uniform
          float g = 0.f, up = 0.f;
#pragma unroll
          for (int s = 0; s < kSlots; ++s) {
            if (slot_q(s) == q && s < rpu * cpl * PH) {
              if (slot_up(s)) up += acc[s];
              else g += acc[s];
            }
          }
          const float v = warp_sum(g);
          const float vu = SW ? warp_sum(up) : 0.f;
          const long row = (long)gw + (long)t * nw;
          if (EPI == kArgmax && v > -INFINITY && (v > best_v || (v == best_v && (uint32_t)row < best_i))) {
            best_v = v;
            best_i = (uint32_t)row;
          }
          if (lane == 0) {
            if (SW) a.y[row] = silu(v) * vu;
            else if (EPI == kAccumulate) a.y[row] += v;
            else a.y[row] = v;
          }
        }
      }
    }
    if (EPI == kArgmax && lane == 0) {
      sh.bval[warp] = best_v;
      sh.bidx[warp] = best_i;
    }
  }
};

__device__ __forceinline__ bool better(float ov, uint32_t oi, float v, uint32_t ix) {
  return oi != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || ov > v || (ov == v && oi < ix));
}

// Greedy pick across the CTAs of a GEMV: per-CTA best from sh.bval / sh.bidx, then the last
// CTA to finish reduces the per-CTA picks (lowest index among equal maxima; NaN never wins),
// writes the pick to ctl->token and advances ctl->pos when a.update_token is set.
__device__ __forceinline__ void argmax_finish(const GemvArgs& a, int cta, int ncta, GemvShared& sh) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    uint32_t ix = 0xFFFFFFFFu;
    for (int w = 0; w < kWarps; ++w)
      if (better(sh.bval[w], sh.bidx[w], v, ix)) {
        v = sh.bval[w];
        ix = sh.bidx[w];
      }
    a.part_val[cta] = v;
    a.part_idx[cta] = ix;
    __threadfence();
    sh.is_last = (atomicAdd(a.ticket, 1u) == (uint32_t)ncta - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (sh.is_last && warp == 0) {
    __threadfence();
    float v = -INFINITY;
    uint32_t ix = 0xFFFFFFFFu;
#pragma unroll 1
    for (int b = lane; b < ncta; b += 32) {
      const float bv = __ldcg(a.part_val + b);
      const uint32_t bi = __ldcg(a.part_idx + b);
      if (better(bv, bi, v, ix)) {
        v = bv;
        ix = bi;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, ix, o);
      if (better(ov, oi, v, ix)) {
        v = ov;
        ix = oi;
      }
    }
    if (lane == 0) {
      if (a.update_token) {
        a.ctl->token = (ix == 0xFFFFFFFFu) ? 0u : ix;
        a.ctl->pos += 1;
      }
      *a.ticket = 0u;
    }
  }
}

}  // namespace dev
}  // namespace qne
