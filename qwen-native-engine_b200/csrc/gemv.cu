// Batch-1 GEMV for the decode step: f16, MatMulNBits block-32 int4 and group-64 int4 weights.
//
// Follows gemv / gemv_f16 / gemv_split_f16 (kernels/src/shaders.rs:48-376) in what it computes:
// y[r] (=, +=, silu-gated) sum_k deq(W[r, k]) x[k], accumulated in f32. The B200 design differs:
//  * one warp owns NR output rows at a time; every lane streams 16-byte chunks of those rows
//    with L1-bypassing loads, U chunks per row in flight, and reduces with warp shuffles;
//  * the CTA stages x in shared memory once, through a fused prologue: plain copy, RMSNorm
//    (rmsnorm_width, kernels/src/shaders.rs:380-403), the gated per-head RMSNorm that ends the
//    GDN step (kernels/src/shaders.rs:512-516), or embedding gather + RMSNorm
//    (embed_width, kernels/src/shaders.rs:409-434);
//  * the epilogue stores, accumulates into the residual stream, applies SwiGLU, or stores logits
//    and runs the greedy pick (argmax_partial + argmax_final, kernels/src/shaders.rs:636-699) in
//    the last CTA to finish;
//  * launches use programmatic dependent launch: the CTA first asks the TMA unit to prefetch its
//    weight rows into L2, then waits for the previous kernel, so weight streaming overlaps the
//    previous kernel's tail and the launch gap.
#include <math.h>

#include <atomic>

#include "gemv.cuh"
#include "gemv_dev.cuh"
#include "tma.cuh"

namespace qne {

using namespace dev;

static std::atomic<uint64_t> g_launches{0};
uint64_t launches_issued() { return g_launches.load(std::memory_order_relaxed); }
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {

// ------------------------------------------------------------------------------------------
// f16 GEMV streamed by the bulk-copy (TMA) unit.
//
// A CTA owns a contiguous range of output rows [r0, r1), so its share of the matrix is one
// contiguous byte range (two for SwiGLU: its gate rows and its up rows). The range is cut into
// pieces of `per` whole rows (SwiGLU: per gate rows, then the per matching up rows), at most
// 16 KB, and one producer thread bulk-copies the pieces in order into a ring of shared-memory
// slots (one or two copies per piece, completing on the slot's mbarrier). Consumer warp w owns
// slot w and takes every NS-th piece (NS = the slot count, 5 or 6 by k; the other consumer warps
// only stage x): wait for the slot, dot its rows with x (staged once in shared memory as two
// planes), release the slot, and lane r applies the epilogue to output row r of the piece. A
// slot has one consumer, so a warp waits on a slot's fills in order and a parity wait cannot
// mistake an earlier, not yet completed fill for the one it wants. The producer starts before the programmatic-launch wait, since weights depend on
// nothing: the first ring's worth of weights (~90 KB per SM) streams while the previous kernel
// finishes. A CTA takes at most ~110 KB of shared memory and 32 K registers, so the next GEMV's
// CTA fits beside it on the same SM and starts streaming as early.
// ------------------------------------------------------------------------------------------
constexpr int kRingConsumers = 8;
constexpr int kThreadsT = (kRingConsumers + 1) * 32;
constexpr uint32_t kPieceB = 16u << 10;    // ring slot
constexpr int kMaxSlots = 8;  // at most one slot per consumer warp
constexpr size_t kRingSmemCap = 110u << 10;  // per CTA: two CTAs share an SM
constexpr int kRingHead = 256;               // barriers and reduction scratch before the ring
constexpr int kRingMaxK = 6144;

// Ring slots for a given k: what fits beside the x planes (k floats) under the per-CTA cap.
__host__ __device__ inline int ring_slots(int k) {
  const size_t left = kRingSmemCap - kRingHead - (size_t)k * 4;
  const int s = (int)(left / kPieceB);
  return s > kMaxSlots ? kMaxSlots : s;
}
__host__ __device__ inline size_t ring_smem_bytes(int k) {
  return kRingHead + (size_t)ring_slots(k) * kPieceB + (size_t)k * 4;
}

struct RingHead {
  unsigned long long full[kMaxSlots];
  unsigned long long empty[kMaxSlots];
  float red[kRingConsumers];
  float bval[kRingConsumers];
  uint32_t bidx[kRingConsumers];
  uint32_t is_last;
};
static_assert(sizeof(RingHead) <= kRingHead, "ring header fits its reserved bytes");

// This CTA's rows and their cut into pieces. `per` is the largest power of two (up to 8 rows, 4
// for SwiGLU) that a slot holds and that still gives every slot's warp a piece when the CTA has
// few rows.
struct RingGeo {
  int out_rows, r0, r1, per, R, npieces;
  uint32_t rb;
  __host__ __device__ void init(int rows, int k, bool sw, int cta, int ncta, int nslots) {
    out_rows = sw ? rows / 2 : rows;
    rb = (uint32_t)k * 2u;
    r0 = (int)((long)out_rows * cta / ncta);
    r1 = (int)((long)out_rows * (cta + 1) / ncta);
    const int cap = (int)(kPieceB / (sw ? 2u * rb : rb));
    const int want = (r1 - r0 + nslots - 1) / nslots;
    const int mx = sw ? 4 : 8;
    per = 1;
    while (per * 2 <= cap && per * 2 <= want && per * 2 <= mx) per *= 2;
    R = sw ? 2 * per : per;
    npieces = r1 > r0 ? (r1 - r0 + per - 1) / per : 0;
  }
};

// Stages x for the consumer warps as two planes (elements 0-3 and 4-7 of every 8-element
// chunk; a lane's 16-byte reads of consecutive chunks are then conflict-free) with the prologue
// applied. RMSNorm is folded: the planes hold x * norm_w and the returned factor
// rsqrt(mean(x^2) + eps) scales the dot products in the epilogue (1 for the other prologues).
// `nw` holds this thread's chunk of the norm weight, loaded before the dependency wait.
template <int PRO>
__device__ __forceinline__ float ring_stage(const GemvArgs& a, float* xs, RingHead& hd, const float (&nw)[8]) {
  const int k = a.m.k, tid = threadIdx.x, nc = k / 8;
  float* xlo = xs;
  float* xhi = xs + k / 2;
  constexpr bool kNorm = PRO == kProRmsNorm || PRO == kProEmbedNorm;
  float ss = 0.f;
  if (PRO == kProCopy) {
#pragma unroll 1
    for (int c = tid; c < nc; c += kRingConsumers * 32) {
      *reinterpret_cast<float4*>(xlo + c * 4) = __ldcg(reinterpret_cast<const float4*>(a.x + c * 8));
      *reinterpret_cast<float4*>(xhi + c * 4) = __ldcg(reinterpret_cast<const float4*>(a.x + c * 8 + 4));
    }
  } else {
    // Norm prologues run on k <= 2048: one chunk per thread at most.
    const int c = tid;
    if (c < nc) {
      float v[8];
      if (PRO == kProEmbedNorm) {
        uint32_t token = a.ctl->token;
        if (token >= (uint32_t)a.embed.rows) token = (uint32_t)a.embed.rows - 1;
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = deq_elem(a.embed, token, c * 8 + j);
        if (blockIdx.x == 0) {
          *reinterpret_cast<float4*>(a.h_out + c * 8) = make_float4(v[0], v[1], v[2], v[3]);
          *reinterpret_cast<float4*>(a.h_out + c * 8 + 4) = make_float4(v[4], v[5], v[6], v[7]);
        }
      } else {
        const float4 p = __ldcg(reinterpret_cast<const float4*>(a.x + c * 8));
        const float4 q = __ldcg(reinterpret_cast<const float4*>(a.x + c * 8 + 4));
        v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
        v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
      }
      float cs = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) cs = fmaf(v[j], v[j], cs);
      ss = cs;
      if (kNorm) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] *= nw[j];
      } else if (PRO == kProGdnGate) {
        // k == 2048 and 256 threads: one chunk per thread, 16 consecutive threads per 128-wide head.
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
        const float inv = rsqrtf(cs / (float)kGdnDim + a.eps);
        const float4 z0 = __ldcg(reinterpret_cast<const float4*>(a.zgate + c * 8));
        const float4 z1 = __ldcg(reinterpret_cast<const float4*>(a.zgate + c * 8 + 4));
        const float z[8] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = v[j] * inv * silu(z[j]) * nw[j];
      }
      *reinterpret_cast<float4*>(xlo + c * 4) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(xhi + c * 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (PRO == kProEmbedNorm && blockIdx.x == 0 && tid == 0) a.ctl->count += 1;  // conv windows
    if (kNorm) {
      const float t = warp_sum(ss);
      if ((tid & 31) == 0) hd.red[tid >> 5] = t;
    }
  }
  ConsumerSync()();
  if (!kNorm) return 1.f;
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kRingConsumers; ++w) t += hd.red[w];
  return rsqrtf(t / (float)k + a.eps);
}

// Dot products of the R rows of one piece with x; every lane ends with the R sums.
template <int R>
__device__ __forceinline__ void ring_dot(const uint8_t* piece, const float* xs, int k, uint32_t rb, int lane,
                                         float (&acc)[R]) {
  float s[R];
#pragma unroll
  for (int r = 0; r < R; ++r) s[r] = 0.f;
  const float* xlo = xs;
  const float* xhi = xs + k / 2;
  constexpr int U = R >= 4 ? 2 : 4;
#pragma unroll U
  for (int c = lane; c < k / 8; c += 32) {
    float xv[8];
    *reinterpret_cast<float4*>(xv) = *reinterpret_cast<const float4*>(xlo + c * 4);
    *reinterpret_cast<float4*>(xv + 4) = *reinterpret_cast<const float4*>(xhi + c * 4);
#pragma unroll
    for (int r = 0; r < R; ++r)
      s[r] += dot_f16(*reinterpret_cast<const uint4*>(piece + (size_t)r * rb + (size_t)c * 16), xv);
  }
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = warp_sum(s[r]);
}

template <int N>
__device__ __forceinline__ float ring_pick(const float (&v)[N], int i) {
  float r = 0.f;
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (j == i) r = v[j];
  return r;
}

__device__ __forceinline__ bool ring_better(float v, uint32_t i, float bv, uint32_t bi) {
  return i != 0xFFFFFFFFu && (bi == 0xFFFFFFFFu || v > bv || (v == bv && i < bi));
}

// The pieces of consumer warp w < NS (w, w + NS, ...: every fill of slot w), R rows each.
template <int EPI, int R>
__device__ __forceinline__ void ring_consume(const GemvArgs& a, const RingGeo& geo, uint8_t* ring, int NS,
                                             const float* xs, RingHead& hd, float inv, float& best_v,
                                             uint32_t& best_i) {
  constexpr bool SW = (EPI == kSwiGlu);
  constexpr int OUT = SW ? R / 2 : R;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k = a.m.k;
#pragma unroll 1
  for (int j = warp; j < geo.npieces; j += NS) {
    const int slot = warp;
    const int row0 = geo.r0 + j * geo.per;
    const int n = min(geo.per, geo.r1 - row0);
    const float resid = (EPI == kAccumulate && lane < n) ? __ldcg(a.y + row0 + lane) : 0.f;
    if (!mbar_wait(smem_u32(&hd.full[slot]), (uint32_t)(j / NS) & 1u, a.err)) return;
    float acc[R];
    ring_dot<R>(ring + (size_t)slot * kPieceB, xs, k, geo.rb, lane, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&hd.empty[slot]));
    if (lane < n) {
      const int row = row0 + lane;
      const float v = ring_pick<R>(acc, lane) * inv;
      if (SW) {
        a.y[row] = silu(v) * (ring_pick<R>(acc, OUT + lane) * inv);
      } else if (EPI == kAccumulate) {
        a.y[row] = resid + v;
      } else {
        a.y[row] = v;
        if (EPI == kArgmax && v > -INFINITY && ring_better(v, (uint32_t)row, best_v, best_i)) {
          best_v = v;
          best_i = (uint32_t)row;
        }
      }
    }
  }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(kThreadsT, 2) gemv_tma_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  RingHead& hd = *reinterpret_cast<RingHead*>(smem_raw);
  uint8_t* ring = smem_raw + kRingHead;
  const int k = a.m.k;
  const int NS = ring_slots(k);
  float* xs = reinterpret_cast<float*>(ring + (size_t)NS * kPieceB);
  constexpr bool SW = (EPI == kSwiGlu);
  RingGeo geo;
  geo.init(a.m.rows, k, SW, blockIdx.x, gridDim.x, NS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(smem_u32(&hd.full[i]), 1);
      mbar_init(smem_u32(&hd.empty[i]), 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch();

  if (warp == kRingConsumers) {
    // ---------------- producer: lane 0 ----------------
    if (lane != 0) return;
    const uint8_t* W = static_cast<const uint8_t*>(a.m.w);
    int issued = 0;
#pragma unroll 1
    for (int j = 0; j < geo.npieces; ++j, ++issued) {
      const int slot = j % NS;
      if (j >= NS && !mbar_wait(smem_u32(&hd.empty[slot]), (uint32_t)(j / NS - 1) & 1u, a.err)) break;
      const int row0 = geo.r0 + j * geo.per;
      const int n = min(geo.per, geo.r1 - row0);
      const uint32_t bytes = (uint32_t)n * geo.rb;
      const uint32_t fb = smem_u32(&hd.full[slot]);
      const uint32_t dst = smem_u32(ring + (size_t)slot * kPieceB);
      mbar_arrive_expect_tx(fb, SW ? 2u * bytes : bytes);
      bulk_g2s(dst, W + (size_t)row0 * geo.rb, bytes, fb);
      if (SW) bulk_g2s(dst + (uint32_t)geo.per * geo.rb, W + (size_t)(geo.out_rows + row0) * geo.rb, bytes, fb);
    }
    // Every copy lands before the CTA exits (bounded; normally the consumers saw them all).
#pragma unroll 1
    for (int s = 0; s < NS && s < issued; ++s) {
      const int fills = (issued - s + NS - 1) / NS;
      mbar_wait(smem_u32(&hd.full[s]), (uint32_t)(fills - 1) & 1u, a.err);
    }
    return;
  }

  // ---------------- consumers ----------------
  float nw[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) nw[j] = 1.f;
  if (PRO != kProCopy && threadIdx.x < k / 8) {
    // The norm weight depends on nothing: load it before the dependency wait.
    const float* src = (PRO == kProGdnGate) ? a.norm_w + ((threadIdx.x * 8) & (kGdnDim - 1)) : a.norm_w + threadIdx.x * 8;
    const float4 p = __ldg(reinterpret_cast<const float4*>(src));
    const float4 q = __ldg(reinterpret_cast<const float4*>(src + 4));
    nw[0] = p.x; nw[1] = p.y; nw[2] = p.z; nw[3] = p.w;
    nw[4] = q.x; nw[5] = q.y; nw[6] = q.z; nw[7] = q.w;
  }
  pdl_wait();
  const float inv = ring_stage<PRO>(a, xs, hd, nw);

  float best_v = -INFINITY;
  uint32_t best_i = 0xFFFFFFFFu;
  if (warp < NS) switch (geo.R) {
    case 1: ring_consume<EPI, 1>(a, geo, ring, NS, xs, hd, inv, best_v, best_i); break;
    case 2: ring_consume<EPI, 2>(a, geo, ring, NS, xs, hd, inv, best_v, best_i); break;
    case 4: ring_consume<EPI, 4>(a, geo, ring, NS, xs, hd, inv, best_v, best_i); break;
    default: ring_consume<EPI, 8>(a, geo, ring, NS, xs, hd, inv, best_v, best_i); break;
  }

  if (EPI == kArgmax) {
    // Greedy pick: warp best, CTA best, then the last CTA reduces across CTAs.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ring_better(ov, oi, best_v, best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    if (lane == 0) {
      hd.bval[warp] = best_v;
      hd.bidx[warp] = best_i;
    }
    ConsumerSync()();
    if (threadIdx.x == 0) {
      float v = -INFINITY;
      uint32_t ix = 0xFFFFFFFFu;
      for (int w = 0; w < kRingConsumers; ++w)
        if (ring_better(hd.bval[w], hd.bidx[w], v, ix)) {
          v = hd.bval[w];
          ix = hd.bidx[w];
        }
      a.part_val[blockIdx.x] = v;
      a.part_idx[blockIdx.x] = ix;
      __threadfence();
      hd.is_last = (atomicAdd(a.ticket, 1u) == gridDim.x - 1) ? 1u : 0u;
    }
    ConsumerSync()();
    if (hd.is_last && warp == 0) {
      __threadfence();
      float v = -INFINITY;
      uint32_t ix = 0xFFFFFFFFu;
      for (int b = lane; b < (int)gridDim.x; b += 32) {
        const float bv = __ldcg(a.part_val + b);
        const uint32_t bi = __ldcg(a.part_idx + b);
        if (ring_better(bv, bi, v, ix)) {
          v = bv;
          ix = bi;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, ix, o);
        if (ring_better(ov, oi, v, ix)) {
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
}

// f16 GEMV, pipelined register streaming (the default f16 kernel): see dev::Pipe.
template <int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 2) gemv_pipe_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) float xs[];
  __shared__ GemvShared sh;
  Pipe<PRO, EPI> p;
  p.init(a, blockIdx.x, gridDim.x);
  pdl_launch();
  p.prefetch(a);
  pdl_wait();
  p.run(a, xs, sh);
  if (EPI == kArgmax) argmax_finish(a, blockIdx.x, gridDim.x, sh);
}

// ------------------------------------------------------------------------------------------
// int4 GEMV on the tensor cores (B = 1).
//
// A warp owns a tile of 16 weight rows (plus the 16 matching up rows for SwiGLU) and a slice of
// k cut into 128-wide segments (64 bytes of a row). For every segment lane (g, t) holds one
// 16-byte load of rows g and g + 8: nibbles k = 128S + 32t .. +31, i.e. lane t's own
// quantization block (block-32) or half of one (group-64). The warp's whole slice (up to 6
// segments, 2-3 for SwiGLU), with each block's scale and zero-point words, is loaded into
// registers before the wait on the previous kernel. (w >> 4i) & 0x000F000F | 0x64006400 turns
// nibbles i and i + 4 into the f16 pair (1024 + n_i, 1024 + n_{i+4}); subtracting 1024 leaves the
// exact integers. Each word of a lane feeds two mma.m16n8k16 (A slots 2t, 2t + 1, 2t + 8, 2t + 9
// of lane t are its own nibbles, so no data moves between lanes; the k order inside an MMA is
// permuted identically for weights and x). The 8 MMA columns keep the blocks apart: column
// 2b + 0 / 1 carries f16(x) / f16(x - f16(x)) of the k values in block b of the segment and zero
// elsewhere, so lane t ends each segment holding block t's exact sum_k n_k x_k for rows g and
// g + 8 (columns 2t, 2t + 1), and applies scale * (sum - zp * sum_k x_k) in f32. Warps of a CTA
// split k when the matrix has few rows; partial sums meet in shared memory.
// ------------------------------------------------------------------------------------------
constexpr int kQtSeg = 128;  // k per segment
// Segments a warp holds in registers (block-32 SwiGLU keeps two: its scale and zero-point words
// do not fit three within 128 registers).
__host__ __device__ constexpr int qt_batch(int kind, bool swiglu) { return swiglu ? (kind == kQ4 ? 2 : 3) : 6; }

__device__ __forceinline__ uint32_t nib_pair_f16(uint32_t w, int i) {
  uint32_t r;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(r) : "r"(w >> (4 * i)));  // (a & b) | c
  uint32_t out;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(out) : "r"(r), "r"(0x64006400u));
  return out;
}

__device__ __forceinline__ void mma_f16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// int4 GEMV through registers (Q4Pipe): the warp's share of weights, scales and zero points is
// loaded before the wait on the previous kernel.
template <int KIND, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 2) gemv_q4pipe_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) float xs[];
  __shared__ GemvShared sh;
  Q4Pipe<KIND, PRO, EPI> p;
  p.init(a, blockIdx.x, gridDim.x);
  pdl_launch();
  p.prefetch(a);
  pdl_wait();
  p.run(a, xs, sh);
  if (EPI == kArgmax) argmax_finish(a, blockIdx.x, gridDim.x, sh);
}

template <int KIND, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 2) gemv_q4_mma_kernel(const GemvArgs a) {
  // the hi and lo f16 pair planes of x ([2][k / 8] uint4), then [k / QB] block sums
  extern __shared__ __align__(16) float xs[];
  __shared__ GemvShared sh;
  __shared__ float part[kWarps][2][16];

  constexpr bool SW = (EPI == kSwiGlu);
  constexpr int PH = SW ? 2 : 1;
  constexpr int PF = qt_batch(KIND, SW);       // segments held in registers per batch
  constexpr int QB = (KIND == kQ4) ? 32 : 64;  // values per quantization block
  const int k = a.m.k;
  const int out_rows = SW ? a.m.rows / 2 : a.m.rows;
  const long half = SW ? a.m.rows / 2 : 0;
  const int tiles = (out_rows + 15) / 16;
  const int RG = a.row_groups, KG = kWarps / RG;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rg = warp % RG, kg = warp / RG;
  const int nseg = k / kQtSeg;
  const int s0 = kg * nseg / KG, s1 = (kg + 1) * nseg / KG;
  const uint8_t* W = static_cast<const uint8_t*>(a.m.w);
  const size_t rb = (size_t)k / 2;
  // Lane t's quantization block within a segment (block-32: t; group-64: t / 2, lanes 0-1 hold
  // the two groups' sums) and whether it feeds x to the MMA: column g carries block g / 2,
  // hi (g even) or lo (g odd).
  const int qblk = (KIND == kQ4) ? t : (t >> 1);
  const bool feeds = (g >> 1) == qblk;
  const bool sums = (KIND == kQ4) || t < 2;

  uint4 w[PF][PH][2];        // [segment][gate / up][row g, row g + 8]: 32 nibbles each
  uint32_t sq[PF][PH][2];    // scale word of lane t's block
  uint32_t zq[PF][PH][2];    // zero-point word of lane t's block

  // Loads segments [sb, min(sb + PF, s1)) of tile `tile` (rows clamped into the matrix).
  auto load = [&](int tile, int sb) {
    const long rA = min((long)tile * 16 + g, (long)out_rows - 1);
    const long rB = min((long)tile * 16 + g + 8, (long)out_rows - 1);
#pragma unroll
    for (int i = 0; i < PF; ++i) {
      const int S = sb + i;
#pragma unroll
      for (int p = 0; p < PH; ++p)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          w[i][p][r] = make_uint4(0u, 0u, 0u, 0u);
          sq[i][p][r] = 0u;
          zq[i][p][r] = 0u;
        }
      if (S >= s1) continue;
#pragma unroll
      for (int p = 0; p < PH; ++p)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const long row = (r ? rB : rA) + (p ? half : 0);
          w[i][p][r] = ld_stream(W + (size_t)row * rb + (size_t)S * (kQtSeg / 2) + (size_t)t * 16);
          if (sums) {
            if (KIND == kQ4) {  // f16 scale pair per 64 values, 8 zero-point nibbles per 256
              sq[i][p][r] = __ldg(static_cast<const uint32_t*>(a.m.s) + row * (k / 64) + 2 * S + (t >> 1));
              zq[i][p][r] = __ldg(static_cast<const uint32_t*>(a.m.z) + row * (k / 256) + (S >> 1));
            } else {            // f16 scale and f16 zero point per 64 values
              sq[i][p][r] = __ldg(static_cast<const uint16_t*>(a.m.s) + row * (k / 64) + 2 * S + t);
              zq[i][p][r] = __ldg(static_cast<const uint16_t*>(a.m.z) + row * (k / 64) + 2 * S + t);
            }
          }
        }
    }
  };

  pdl_launch();
  const int first = blockIdx.x * RG + rg;
  if (first < tiles) load(first, s0);  // weights depend on nothing: before the dependency wait
  float nw[8];
  pre_norm<PRO>(a, nw);
  pdl_wait();

  // x (prologue applied, RMSNorm folded into `inv`) as hi / lo f16 pair planes and block sums
  uint4* xq = reinterpret_cast<uint4*>(xs);  // [2][k / 8]: hi plane, then lo plane
  float* xsum = xs + k;
  const float inv = stage_fold<PRO, 1>(a, xq, sh.red, nw, CtaSync(), xsum, QB / 8);
  const uint2* xplane = reinterpret_cast<const uint2*>(xq + (g & 1) * (k / 8));

  float best_v = -INFINITY;
  uint32_t best_i = 0xFFFFFFFFu;
  bool loaded = true;
  // CTA-uniform loop (every warp runs the same iterations: the k-slice reduction synchronizes)
  for (int base = blockIdx.x * RG; base < tiles; base += gridDim.x * RG) {
    const int tile = base + rg;
    const bool tile_ok = tile < tiles;
    float tot[PH][2];
#pragma unroll
    for (int p = 0; p < PH; ++p) tot[p][0] = tot[p][1] = 0.f;
    for (int sb = s0; sb < s1; sb += PF) {
      if (!loaded && tile_ok) load(tile, sb);
      loaded = false;
      if (!tile_ok) continue;
#pragma unroll
      for (int i = 0; i < PF; ++i) {
        const int S = sb + i;
        if (S >= s1) break;
        float c[PH][4];
#pragma unroll
        for (int p = 0; p < PH; ++p) c[p][0] = c[p][1] = c[p][2] = c[p][3] = 0.f;
#pragma unroll
        for (int wd = 0; wd < 4; ++wd) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            // x of chunk (segment S, block t, word wd): elements 2h, 2h + 4 and 2h + 1, 2h + 5
            uint2 xb = make_uint2(0u, 0u);
            if (feeds) xb = xplane[(size_t)(S * 16 + t * 4 + wd) * 2 + h];
#pragma unroll
            for (int p = 0; p < PH; ++p) {
              const uint32_t wa = (&w[i][p][0].x)[wd], wb = (&w[i][p][1].x)[wd];
              mma_f16(c[p], nib_pair_f16(wa, 2 * h), nib_pair_f16(wb, 2 * h), nib_pair_f16(wa, 2 * h + 1),
                      nib_pair_f16(wb, 2 * h + 1), xb.x, xb.y);
            }
          }
        }
        if (sums) {
          // lane t holds columns 2t (hi) and 2t + 1 (lo): block qblk of the segment, rows g, g + 8
          const int blk = (KIND == kQ4) ? 4 * S + t : 2 * S + t;
          const float xsb = xsum[blk];
#pragma unroll
          for (int p = 0; p < PH; ++p)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              float scale, zp;
              if (KIND == kQ4) {
                scale = h2f((uint16_t)((t & 1) ? (sq[i][p][r] >> 16) : (sq[i][p][r] & 0xFFFFu)));
                zp = (float)((zq[i][p][r] >> (4 * (4 * (S & 1) + t))) & 15u);
              } else {
                scale = h2f((uint16_t)sq[i][p][r]);
                zp = h2f((uint16_t)zq[i][p][r]);
              }
              tot[p][r] = fmaf(scale, (c[p][2 * r] + c[p][2 * r + 1]) - zp * xsb, tot[p][r]);
            }
        }
      }
    }
    // blocks of the quad, then the k-slices of the CTA's warps (shared memory)
#pragma unroll
    for (int p = 0; p < PH; ++p)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        tot[p][r] += __shfl_xor_sync(0xffffffffu, tot[p][r], 1);
        tot[p][r] += __shfl_xor_sync(0xffffffffu, tot[p][r], 2);
      }
    if (KG > 1) {
      __syncthreads();
      if (t == 0) {
#pragma unroll
        for (int p = 0; p < PH; ++p) {
          part[warp][p][g] = tot[p][0];
          part[warp][p][g + 8] = tot[p][1];
        }
      }
      __syncthreads();
      if (kg == 0 && t == 0) {
        for (int q = 1; q < KG; ++q)
#pragma unroll
          for (int p = 0; p < PH; ++p) {
            tot[p][0] += part[rg + q * RG][p][g];
            tot[p][1] += part[rg + q * RG][p][g + 8];
          }
      }
    }
    if (tile_ok && kg == 0 && t == 0) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const long o = (long)tile * 16 + g + 8 * r;
        if (o >= out_rows) continue;
        const float v = SW ? silu(tot[0][r] * inv) * (tot[PH - 1][r] * inv) : tot[0][r] * inv;
        if (EPI == kAccumulate) a.y[o] += v;
        else a.y[o] = v;
        if (EPI == kArgmax && v > -INFINITY && better(v, (uint32_t)o, best_v, best_i)) {
          best_v = v;
          best_i = (uint32_t)o;
        }
      }
    }
  }
  if (EPI == kArgmax) {
    // lanes without rows hold no candidate; reduce the warp, then the CTA and the grid
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (better(ov, oi, best_v, best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    if (lane == 0) {
      sh.bval[warp] = best_v;
      sh.bidx[warp] = best_i;
    }
    argmax_finish(a, blockIdx.x, gridDim.x, sh);
  }
}

template <int KIND, int PRO, int EPI, int NR>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[kWarps];
  __shared__ float bval[kWarps];
  __shared__ uint32_t bidx[kWarps];
  __shared__ uint32_t is_last;

  constexpr int CV = Fmt<KIND>::CV;
  constexpr int PHYS = (EPI == kSwiGlu) ? 2 * NR : NR;
  constexpr int U = (KIND == kF16) ? (PHYS == 1 ? 8 : 16 / PHYS) : (PHYS == 1 ? 4 : 8 / PHYS);
  const int k = a.m.k;
  const int nch = k / CV;
  const int out_rows = (EPI == kSwiGlu) ? a.m.rows / 2 : a.m.rows;
  const long half = (EPI == kSwiGlu) ? a.m.rows / 2 : 0;
  const size_t rb = Fmt<KIND>::row_bytes(k);
  const int groups = (out_rows + NR - 1) / NR;
  const int g0 = (int)((long)blockIdx.x * groups / gridDim.x);
  const int g1 = (int)((long)(blockIdx.x + 1) * groups / gridDim.x);
  const uint8_t* W = static_cast<const uint8_t*>(a.m.w);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  pdl_launch();
  if (warp == 0) {
    const long r0 = (long)g0 * NR;
    const long r1 = min((long)g1 * NR, (long)out_rows);
    const uint32_t budget = (EPI == kSwiGlu) ? kPrefetchBytes / 2 : kPrefetchBytes;
    prefetch_rows(W, rb, r0, r1, budget, lane);
    if (EPI == kSwiGlu) prefetch_rows(W, rb, half + r0, half + r1, budget, lane);
  }
  pdl_wait();
  stage_x<PRO>(a, xs, red);

  float best_v = -INFINITY;
  uint32_t best_i = 0xFFFFFFFFu;

  for (int g = g0 + warp; g < g1; g += kWarps) {
    long rows[PHYS];
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const long r = min((long)g * NR + i, (long)out_rows - 1);
      rows[i] = r;
      if (EPI == kSwiGlu) rows[NR + i] = half + r;
    }
    float acc[PHYS];
#pragma unroll
    for (int i = 0; i < PHYS; ++i) acc[i] = 0.f;

    for (int base = 0; base < nch; base += 32 * U) {
      uint4 wv[PHYS][U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = base + u * 32 + lane;
#pragma unroll
        for (int i = 0; i < PHYS; ++i)
          wv[i][u] = (c < nch) ? ld_stream(W + (size_t)rows[i] * rb + (size_t)c * 16)
                               : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = base + u * 32 + lane;
        if (c < nch) {
          const float* xc = xs + c * CV;
          if (KIND == kF16) {
            float xv[8];
            *reinterpret_cast<float4*>(xv) = *reinterpret_cast<const float4*>(xc);
            *reinterpret_cast<float4*>(xv + 4) = *reinterpret_cast<const float4*>(xc + 4);
#pragma unroll
            for (int i = 0; i < PHYS; ++i) acc[i] += dot_f16(wv[i][u], xv);
          } else {
            float xv[32];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<float4*>(xv + 4 * j) = *reinterpret_cast<const float4*>(xc + 4 * j);
            float xsum = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) xsum += xv[j];
#pragma unroll
            for (int i = 0; i < PHYS; ++i) {
              float scale, zp;
              if (KIND == kQ4)
                q4_scale_zp((const uint32_t*)a.m.s, (const uint32_t*)a.m.z, rows[i], k, c, scale, zp);
              else
                q4g64_scale_zp((const uint16_t*)a.m.s, (const uint16_t*)a.m.z, rows[i], k, c / 2,
                               scale, zp);
              const float raw = dot_q4_raw(wv[i][u], xv);
              acc[i] = fmaf(scale, raw - zp * xsum, acc[i]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < PHYS; ++i) acc[i] = warp_sum(acc[i]);

#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const long r = (long)g * NR + i;
      if (r < out_rows) {
        if (EPI == kArgmax) {
          const float v = acc[i];
          if (v > -INFINITY && (v > best_v || (v == best_v && (uint32_t)r < best_i))) {
            best_v = v;
            best_i = (uint32_t)r;
          }
        }
        if (lane == i) {
          if (EPI == kStore || EPI == kArgmax) a.y[r] = acc[i];
          else if (EPI == kAccumulate) a.y[r] += acc[i];
          else if (EPI == kSwiGlu) a.y[r] = silu(acc[i]) * acc[NR + i];
        }
      }
    }
  }

  if (EPI == kArgmax) {
    // Per-CTA pick, then the last CTA to finish reduces the per-CTA picks.
    if (lane == 0) {
      bval[warp] = best_v;
      bidx[warp] = best_i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = bval[0];
      uint32_t ix = bidx[0];
      for (int w = 1; w < kWarps; ++w) {
        if (bidx[w] != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || bval[w] > v || (bval[w] == v && bidx[w] < ix))) {
          v = bval[w];
          ix = bidx[w];
        }
      }
      a.part_val[blockIdx.x] = v;
      a.part_idx[blockIdx.x] = ix;
      __threadfence();
      const uint32_t t = atomicAdd(a.ticket, 1u);
      is_last = (t == gridDim.x - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (is_last && warp == 0) {
      __threadfence();
      float v = -INFINITY;
      uint32_t ix = 0xFFFFFFFFu;
      for (int b = lane; b < (int)gridDim.x; b += 32) {
        const float bv = __ldcg(a.part_val + b);
        const uint32_t bi = __ldcg(a.part_idx + b);
        if (bi != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || bv > v || (bv == v && bi < ix))) {
          v = bv;
          ix = bi;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, ix, o);
        if (oi != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || ov > v || (ov == v && oi < ix))) {
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
}

template <int KIND>
__global__ void dequant_rows_kernel(const Mat m, int row0, int nrows, float* out) {
  const long total = (long)nrows * m.k;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long)gridDim.x * blockDim.x) {
    const long r = e / m.k;
    const int i = (int)(e % m.k);
    out[e] = deq_elem(m, row0 + r, i);
  }
}

// Standalone greedy pick over n logits (argmax_partial + argmax_final).
__global__ void __launch_bounds__(256) argmax_kernel(const float* logits, uint32_t n, SeqCtl* ctl,
                                                     float* part_val, uint32_t* part_idx,
                                                     uint32_t* ticket) {
  __shared__ float bv[8];
  __shared__ uint32_t bi[8];
  __shared__ uint32_t is_last;
  pdl_launch();
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float v = -INFINITY;
  uint32_t ix = 0xFFFFFFFFu;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float x = logits[i];
    if (x > -INFINITY && (ix == 0xFFFFFFFFu || x > v)) {  // indices ascend: ties keep the first
      v = x;
      ix = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, ix, o);
    if (oi != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || ov > v || (ov == v && oi < ix))) {
      v = ov;
      ix = oi;
    }
  }
  if (lane == 0) {
    bv[warp] = v;
    bi[warp] = ix;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    v = -INFINITY;
    ix = 0xFFFFFFFFu;
    for (int w = 0; w < 8; ++w)
      if (bi[w] != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || bv[w] > v || (bv[w] == v && bi[w] < ix))) {
        v = bv[w];
        ix = bi[w];
      }
    part_val[blockIdx.x] = v;
    part_idx[blockIdx.x] = ix;
    __threadfence();
    is_last = (atomicAdd(ticket, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (is_last && warp == 0) {
    __threadfence();
    v = -INFINITY;
    ix = 0xFFFFFFFFu;
    for (int b = lane; b < (int)gridDim.x; b += 32) {
      const float ov = __ldcg(part_val + b);
      const uint32_t oi = __ldcg(part_idx + b);
      if (oi != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || ov > v || (ov == v && oi < ix))) {
        v = ov;
        ix = oi;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, ix, o);
      if (oi != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || ov > v || (ov == v && oi < ix))) {
        v = ov;
        ix = oi;
      }
    }
    if (lane == 0) {
      ctl->token = (ix == 0xFFFFFFFFu) ? 0u : ix;
      ctl->pos += 1;
      *ticket = 0u;
    }
  }
}

template <typename Kernel>
cudaError_t launch_ex(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      bool pdl, const GemvArgs& a) {
  if (grid.x > (unsigned)kMaxGrid) return cudaErrorInvalidConfiguration;  // argmax slots
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kernel, a);
}

template <int KIND, int PRO, int EPI, int NR>
cudaError_t launch_t(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  auto kernel = gemv_kernel<KIND, PRO, EPI, NR>;
  const size_t smem = (size_t)a.m.k * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int out_rows = (EPI == kSwiGlu) ? a.m.rows / 2 : a.m.rows;
  const int groups = (out_rows + NR - 1) / NR;
  int grid = (groups + kWarps - 1) / kWarps;
  const int max_grid = kNumSms * (a.ctas_per_sm == 1 ? 1 : 2);
  if (grid > max_grid) grid = max_grid;
  if (grid < 1) grid = 1;
  return launch_ex(kernel, dim3(grid), dim3(kThreads), smem, stream, pdl, a);
}

template <int KIND, int PRO, int EPI>
cudaError_t launch_nr(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  // Few output rows: one row per warp so more SMs take part.
  const int out_rows = (EPI == kSwiGlu) ? a.m.rows / 2 : a.m.rows;
  if ((out_rows + 1) / 2 < kNumSms * kWarps) return launch_t<KIND, PRO, EPI, 1>(a, stream, pdl);
  return launch_t<KIND, PRO, EPI, 2>(a, stream, pdl);
}

template <int PRO, int EPI>
cudaError_t launch_pipe(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  auto kernel = gemv_pipe_kernel<PRO, EPI>;
  const size_t smem = (size_t)a.m.k * sizeof(float);  // the two planes of x
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int out_rows = (EPI == kSwiGlu) ? a.m.rows / 2 : a.m.rows;
  int grid = (out_rows + kWarps - 1) / kWarps;  // at least one row per warp
  if (grid > 2 * kNumSms) grid = 2 * kNumSms;
  if (grid < 1) grid = 1;
  return launch_ex(kernel, dim3(grid), dim3(kThreads), smem, stream, pdl, a);
}

// Q4Pipe holds 8 chunks of 32 values per lane and unit: one output row (its gate and up rows
// for SwiGLU) must fit, i.e. k <= 8192 (4096 with SwiGLU).
bool q4pipe_fits(const GemvArgs& a) {
  const int cpl = (a.m.k / 32 + 31) / 32;
  return a.m.k % 256 == 0 && cpl * (a.epi == kSwiGlu ? 2 : 1) <= 8;
}

template <int KIND, int PRO, int EPI>
cudaError_t launch_q4pipe(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  auto kernel = gemv_q4pipe_kernel<KIND, PRO, EPI>;
  const size_t smem = ((size_t)2 * a.m.k + a.m.k / 32) * sizeof(float);  // x, transposed x, chunk sums
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int out_rows = (EPI == kSwiGlu) ? a.m.rows / 2 : a.m.rows;
  int grid = (out_rows + kWarps - 1) / kWarps;  // at least one row per warp
  if (grid > 2 * kNumSms) grid = 2 * kNumSms;
  if (grid < 1) grid = 1;
  return launch_ex(kernel, dim3(grid), dim3(kThreads), smem, stream, pdl, a);
}

template <int KIND, int PRO, int EPI>
cudaError_t launch_q4_mma(GemvArgs a, cudaStream_t stream, bool pdl) {
  auto kernel = gemv_q4_mma_kernel<KIND, PRO, EPI>;
  const int k = a.m.k;
  const size_t smem = ((size_t)k + k / 32) * sizeof(float);  // pair planes, block sums
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int out_rows = (EPI == kSwiGlu) ? a.m.rows / 2 : a.m.rows;
  const int tiles = (out_rows + 15) / 16;
  const int nseg = k / kQtSeg;
  const int pf = qt_batch(KIND, EPI == kSwiGlu);
  const int max_grid = 2 * kNumSms;
  // k-slices per tile: of the splits that keep every warp's slice within one register batch and
  // the grid within two CTAs per SM, the one with the most CTAs; 8 when none does (the CTAs
  // then loop over tiles and batches).
  int kg = 8;
  long most = -1;
  for (int q = 1; q <= kWarps; q *= 2) {
    const long ctas = (tiles + kWarps / q - 1) / (kWarps / q);
    if ((nseg + q - 1) / q <= pf && ctas <= max_grid && ctas > most) {
      most = ctas;
      kg = q;
    }
  }
  const int rg = kWarps / kg;
  a.row_groups = rg;
  int grid = (tiles + rg - 1) / rg;
  if (grid > max_grid) grid = max_grid;
  if (grid < 1) grid = 1;
  return launch_ex(kernel, dim3(grid), dim3(kThreads), smem, stream, pdl, a);
}

// Whether the bulk-copy kernel takes this shape: a piece slot holds a row (SwiGLU: a gate and an
// up row), x fits beside the ring, and the norm prologues stage one chunk per consumer thread.
bool ring_fits(const GemvArgs& a) {
  const int k = a.m.k;
  if (a.m.kind != kF16 || k % 256 || k > kRingMaxK) return false;
  if (a.epi == kSwiGlu && 4 * k > (int)kPieceB) return false;
  if (a.pro != kProCopy && k > 8 * kRingConsumers * 32) return false;
  return true;
}

template <int PRO, int EPI>
cudaError_t launch_tma(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  auto kernel = gemv_tma_kernel<PRO, EPI>;
  const size_t smem = ring_smem_bytes(a.m.k);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int out_rows = (EPI == kSwiGlu) ? a.m.rows / 2 : a.m.rows;
  int grid = out_rows < kNumSms ? out_rows : kNumSms;  // one CTA per SM, at least a row each
  if (grid < 1) grid = 1;
  return launch_ex(kernel, dim3(grid), dim3(kThreadsT), smem, stream, pdl, a);
}

template <int KIND>
cudaError_t launch_kind(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  // Variant 2 (bulk-copy ring) on request; auto picks the register-streamed kernel, which
  // measures faster on B200 for every decode shape.
  if (KIND == kF16 && a.variant == 2 && ring_fits(a)) {
#define QNE_TCOMBO(P, E) \
    if (a.pro == P && a.epi == E) return launch_tma<P, E>(a, stream, pdl);
    QNE_TCOMBO(kProCopy, kStore)
    QNE_TCOMBO(kProCopy, kAccumulate)
    QNE_TCOMBO(kProCopy, kSwiGlu)
    QNE_TCOMBO(kProRmsNorm, kStore)
    QNE_TCOMBO(kProRmsNorm, kAccumulate)
    QNE_TCOMBO(kProRmsNorm, kSwiGlu)
    QNE_TCOMBO(kProRmsNorm, kArgmax)
    QNE_TCOMBO(kProEmbedNorm, kStore)
    QNE_TCOMBO(kProGdnGate, kAccumulate)
#undef QNE_TCOMBO
  }
  if (KIND == kF16 && a.variant == 0 && a.m.k % 256 == 0) {
#define QNE_PCOMBO(P, E) \
    if (a.pro == P && a.epi == E) return launch_pipe<P, E>(a, stream, pdl);
    QNE_PCOMBO(kProCopy, kStore)
    QNE_PCOMBO(kProCopy, kAccumulate)
    QNE_PCOMBO(kProCopy, kSwiGlu)
    QNE_PCOMBO(kProRmsNorm, kStore)
    QNE_PCOMBO(kProRmsNorm, kAccumulate)
    QNE_PCOMBO(kProRmsNorm, kSwiGlu)
    QNE_PCOMBO(kProRmsNorm, kArgmax)
    QNE_PCOMBO(kProEmbedNorm, kStore)
    QNE_PCOMBO(kProGdnGate, kAccumulate)
#undef QNE_PCOMBO
  }
  if constexpr (KIND != kF16) {
    // int4: the tensor-core kernel by default (k % 128 == 0), the register pipeline on request
    // (variant 4) or for the other widths.
    if ((a.variant == 4 || (a.variant == 0 && a.m.k % kQtSeg)) && q4pipe_fits(a)) {
#define QNE_Q4P(P, E) \
    if (a.pro == P && a.epi == E) return launch_q4pipe<KIND, P, E>(a, stream, pdl);
      QNE_Q4P(kProCopy, kStore)
      QNE_Q4P(kProCopy, kAccumulate)
      QNE_Q4P(kProCopy, kSwiGlu)
      QNE_Q4P(kProRmsNorm, kStore)
      QNE_Q4P(kProRmsNorm, kAccumulate)
      QNE_Q4P(kProRmsNorm, kSwiGlu)
      QNE_Q4P(kProRmsNorm, kArgmax)
      QNE_Q4P(kProEmbedNorm, kStore)
      QNE_Q4P(kProGdnGate, kAccumulate)
#undef QNE_Q4P
    }
  }
  if (KIND != kF16 && (a.variant == 0 || a.variant == 3) && a.m.k % kQtSeg == 0) {
#define QNE_QCOMBO(P, E) \
    if (a.pro == P && a.epi == E) return launch_q4_mma<KIND, P, E>(a, stream, pdl);
    QNE_QCOMBO(kProCopy, kStore)
    QNE_QCOMBO(kProCopy, kAccumulate)
    QNE_QCOMBO(kProCopy, kSwiGlu)
    QNE_QCOMBO(kProRmsNorm, kStore)
    QNE_QCOMBO(kProRmsNorm, kAccumulate)
    QNE_QCOMBO(kProRmsNorm, kSwiGlu)
    QNE_QCOMBO(kProRmsNorm, kArgmax)
    QNE_QCOMBO(kProEmbedNorm, kStore)
    QNE_QCOMBO(kProGdnGate, kAccumulate)
#undef QNE_QCOMBO
  }
#define QNE_COMBO(P, E) \
  if (a.pro == P && a.epi == E) return launch_nr<KIND, P, E>(a, stream, pdl);
  QNE_COMBO(kProCopy, kStore)
  QNE_COMBO(kProCopy, kAccumulate)
  QNE_COMBO(kProCopy, kSwiGlu)
  QNE_COMBO(kProRmsNorm, kStore)
  QNE_COMBO(kProRmsNorm, kAccumulate)
  QNE_COMBO(kProRmsNorm, kSwiGlu)
  QNE_COMBO(kProRmsNorm, kArgmax)
  QNE_COMBO(kProEmbedNorm, kStore)
  QNE_COMBO(kProGdnGate, kAccumulate)
#undef QNE_COMBO
  return cudaErrorInvalidValue;
}

}  // namespace

// Per-CTA slots of the greedy-pick reduction: every GEMV / argmax grid is capped at kMaxGrid.
size_t argmax_scratch_bytes() { return 2 * 4 * kMaxGrid + 256; }
void argmax_scratch_carve(void* scratch, float** part_val, uint32_t** part_idx, uint32_t** ticket) {
  uint8_t* p = static_cast<uint8_t*>(scratch);
  *part_val = reinterpret_cast<float*>(p);
  *part_idx = reinterpret_cast<uint32_t*>(p + 4 * kMaxGrid);
  *ticket = reinterpret_cast<uint32_t*>(p + 8 * kMaxGrid);
}

const char* check_gemv(const GemvArgs& a) {
  const Mat& m = a.m;
  if (a.variant < 0 || a.variant > 4) return "unknown GEMV variant";
  if (a.variant == 4 && (m.kind == kF16 || !q4pipe_fits(a)))
    return "the int4 register pipeline needs int4 weights, k % 256 == 0 and k <= 8192 (4096 with SwiGLU)";
  if (a.variant == 3 && (m.kind == kF16 || m.k % kQtSeg)) return "the tensor-core GEMV needs int4 weights and k % 128 == 0";
  if (a.variant == 2 && !ring_fits(a))
    return "the bulk-copy GEMV needs f16 weights, k % 256 == 0 and k <= 6144 (4096 with SwiGLU, 2048 with a norm prologue)";
  if (!m.w || m.rows <= 0 || m.k <= 0) return "matrix has no data or an empty shape";
  if (m.kind == kF16) {
    if (m.k % 256) return "f16 GEMV needs k % 256 == 0";
  } else if (m.kind == kQ4) {
    if (m.k % 256) return "block-32 int4 GEMV needs k % 256 == 0";
    if (!m.s || !m.z) return "int4 matrix without scales or zero points";
  } else if (m.kind == kQ4G64) {
    if (m.k % 64) return "group-64 int4 GEMV needs k % 64 == 0";
    if (!m.s || !m.z) return "int4 matrix without scales or zero points";
  } else {
    return "unknown weight kind";
  }
  if (m.k > 16384) return "k above 16384";
  if (a.epi == kSwiGlu && (m.rows % 2)) return "SwiGLU needs an even row count";
  if (a.pro == kProGdnGate && m.k != kMixerOut) return "the GDN gate prologue needs k == 2048";
  if (!a.y) return "null output";
  if ((a.pro == kProCopy || a.pro == kProRmsNorm || a.pro == kProGdnGate) && !a.x) return "null input";
  if ((a.pro == kProRmsNorm || a.pro == kProEmbedNorm || a.pro == kProGdnGate) && !a.norm_w)
    return "null norm weight";
  if (a.pro == kProGdnGate && !a.zgate) return "null gate";
  if (a.pro == kProEmbedNorm && (!a.embed.w || a.embed.k != m.k || !a.ctl || !a.h_out))
    return "embedding prologue needs an embedding of width k, control words and h";
  if (a.epi == kArgmax && (!a.part_val || !a.part_idx || !a.ticket || (a.update_token && !a.ctl)))
    return "argmax epilogue needs scratch";
  return nullptr;
}

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  switch (a.m.kind) {
    case kF16: return launch_kind<kF16>(a, stream, pdl);
    case kQ4: return launch_kind<kQ4>(a, stream, pdl);
    case kQ4G64: return launch_kind<kQ4G64>(a, stream, pdl);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_dequant_rows(const Mat& m, int row0, int nrows, float* out, cudaStream_t stream) {
  const long total = (long)nrows * m.k;
  int grid = (int)((total + 255) / 256);
  if (grid > 4 * kNumSms) grid = 4 * kNumSms;
  if (grid < 1) grid = 1;
  count_launch();
  switch (m.kind) {
    case kF16: dequant_rows_kernel<kF16><<<grid, 256, 0, stream>>>(m, row0, nrows, out); break;
    case kQ4: dequant_rows_kernel<kQ4><<<grid, 256, 0, stream>>>(m, row0, nrows, out); break;
    case kQ4G64: dequant_rows_kernel<kQ4G64><<<grid, 256, 0, stream>>>(m, row0, nrows, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float* logits, uint32_t n, SeqCtl* ctl, void* scratch,
                          cudaStream_t stream, bool pdl) {
  float* pv;
  uint32_t *pi, *ticket;
  argmax_scratch_carve(scratch, &pv, &pi, &ticket);
  int grid = (int)((n + 1023) / 1024);
  if (grid > kNumSms) grid = kNumSms;
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  return cudaLaunchKernelEx(&cfg, argmax_kernel, logits, n, ctl, pv, pi, ticket);
}

}  // namespace qne
