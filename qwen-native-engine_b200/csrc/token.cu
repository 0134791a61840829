// The token kernel: the per-token dispatch list of kernels/src/model.rs:220-269 (per layer
// in-projection, GDN, out-projection, gate_up, down; then final norm + LM head + greedy pick) run
// as phases of one grid, between the attention layers.
//
// Why: a decode token is a chain of ~120 dependent steps, and as separate kernels each step pays
// a launch boundary and its own ramp and tail, during which HBM idles (the per-operation graph
// measured 1.1 ms per 2B token against 0.58 ms of weight streaming). Here the weight streaming
// does not wait for the dependencies:
//   * one CTA per SM (148), 8 consumer warps + 1 producer warp;
//   * the producer warp walks the launch's GEMV phases in order and bulk-copies (TMA,
//     cp.async.bulk, no multicast) this CTA's rows of every matrix into a ring of 8 x 24 KB
//     shared-memory slots, guarded by full/empty mbarriers. Weights depend on nothing, so the
//     producer runs ahead across phase boundaries until the ring is full: while the consumers
//     wait at a grid barrier for the previous phase's output, the next phase's first 192 KB per
//     SM (28 MB over the GPU) are already streaming. It starts before the launch's dependency
//     wait, so a launch's first weights stream while the kernel before it finishes;
//   * consumer warp w owns ring slot w and takes every 8th slot of the CTA's sequence. A slot
//     holds whole rows (2, 3, 6 or 12 by row length; SwiGLU: gate rows then the matching up
//     rows); the warp dots them with x (staged once per phase in shared memory with its prologue:
//     copy, RMSNorm, gated GDN RMSNorm, or embedding gather + RMSNorm), reduces across lanes and
//     applies the epilogue (store, residual add, SwiGLU, greedy-pick candidate);
//   * phases that read what the previous phase wrote start behind a grid barrier (an arrival
//     counter; release reduction to arrive, acquire polls, bounded in time with an error flag);
//   * GDN: one dev::GdnItem (16 value columns of one head) per CTA for CTAs 0..127, its state
//     slice loaded before the barrier.
// A token is one launch per stretch of layers between attention mixers; each attention layer's
// mixer is the paged attention kernel (attention.cu) between two such launches, chained by
// programmatic dependent launch. Results match the per-operation kernels within the logit
// tolerance (f32 accumulation, other summation order).
#include <math.h>

#include "gemv_dev.cuh"
#include "tma.cuh"
#include "token.cuh"

namespace qne {
namespace {

using namespace dev;

constexpr int kTkConsumerWarps = 8;
constexpr int kTkConsumers = kTkConsumerWarps * 32;
constexpr int kTkThreads = kTkConsumers + 32;  // + the producer warp
constexpr int kTkSlots = kTkConsumerWarps;     // one ring slot per consumer warp
constexpr uint32_t kTkSlotBytes = 24u << 10;
constexpr int kTkMaxK = 6144;

struct TkShared {
  uint8_t ring[kTkSlots][kTkSlotBytes];
  float xs[kTkMaxK];  // the GEMV input (two planes); scratch of the mixer phases
  unsigned long long full[kTkSlots];
  unsigned long long empty[kTkSlots];
  float red[kTkConsumerWarps];
  float bval[kTkConsumerWarps];
  uint32_t bidx[kTkConsumerWarps];
  uint32_t flag;
};
static_assert(sizeof(GdnShared) <= sizeof(float) * kTkMaxK, "GDN scratch aliases xs");
static_assert((kTkSlotBytes % 128) == 0, "ring slots stay 128-byte aligned");

struct ConsumerBar {
  __device__ __forceinline__ void operator()() const { asm volatile("bar.sync 1, 256;" ::: "memory"); }
};

__device__ __forceinline__ unsigned long long tk_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned long long tk_ld_acquire64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t tk_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void tk_red_release64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Grid barrier among the consumer warps of all CTAs (the producer warps never join), split into
// arrive (right after a phase's last write) and wait (before the next phase's first read), so the
// next phase's prefetch loads go out in between without delaying the arrival. The counter is zero
// at launch, barrier n completes at n * (grid + extra) arrivals, the last CTA to exit clears it.
// The consumer barrier orders the CTA's writes before thread 0's release reduction, which
// publishes them; the acquire polls make the other CTAs' writes visible. Bounded in time; once any
// CTA gave up (kFlagTimeout), the others stop waiting.
struct TkBarrier {
  unsigned long long* count;
  unsigned long long target;  // consumer thread 0 only
  uint64_t limit_ns;
  uint32_t extra;

  __device__ __forceinline__ void arrive() {
    ConsumerBar()();
    if (threadIdx.x == 0) {
      target += gridDim.x + extra;
      tk_red_release64(count, 1ull);
    }
  }

  __device__ __forceinline__ void wait(uint32_t* err) {
    if (threadIdx.x == 0) {
      const unsigned long long t0 = tk_now();
      uint32_t rounds = 0;
      while (tk_ld_acquire64(count) < target) {
        if ((++rounds & 63u) == 0u) {
          if (tk_ld_acquire(err) & kFlagTimeout) break;
          if (tk_now() - t0 > limit_ns) {
            atomicOr(err, kFlagTimeout);
            break;
          }
        }
      }
    }
    ConsumerBar()();
  }

  __device__ __forceinline__ void exit() {
    ConsumerBar()();
    if (threadIdx.x == 0 && atomicAdd(count + 1, 1ull) == gridDim.x - 1) {
      count[0] = 0ull;
      count[1] = 0ull;
      __threadfence();
    }
  }
};

// This CTA's share of a GEMV phase: output rows [r0, r1), `per` output rows per ring slot (a
// slot holds R = per rows, or per gate rows then per up rows for SwiGLU; R in {2, 3, 6, 12}).
// `per` is the smallest size that still spreads the CTA's rows over all 8 consumer warps (many
// small slots when a matrix has few rows), up to what a 24 KB slot holds.
struct Geo {
  int k, out_rows, r0, r1, per, R, nslots;
  uint32_t rb;  // bytes per row
  bool sw;
  __device__ __forceinline__ void init(const TkPhase& p, int cta, int ncta) {
    sw = p.epi == kSwiGlu;
    k = p.k;
    out_rows = sw ? p.rows / 2 : p.rows;
    rb = (uint32_t)k * 2u;
    r0 = (int)((long)out_rows * cta / ncta);
    r1 = (int)((long)out_rows * (cta + 1) / ncta);
    const int want = (r1 - r0 + kTkSlots - 1) / kTkSlots;  // rows per warp if every warp gets one slot
    int cap = (int)(kTkSlotBytes / rb);
    if (sw) {
      cap /= 2;
      const int mx = cap >= 6 ? 6 : cap >= 3 ? 3 : 1;
      per = want <= 1 ? 1 : want <= 3 ? 3 : 6;
      if (per > mx) per = mx;
      R = 2 * per;
    } else {
      const int mx = cap >= 12 ? 12 : cap >= 6 ? 6 : cap >= 3 ? 3 : 2;
      per = want <= 2 ? 2 : want <= 3 ? 3 : want <= 6 ? 6 : 12;
      if (per > mx) per = mx;
      R = per;
    }
    nslots = r1 > r0 ? (r1 - r0 + per - 1) / per : 0;
  }
};

// ------------------------------------------------------------------------------------------
// Producer: lane 0 of the last warp.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tk_produce(const TkArgs& A, TkShared& sh) {
  uint32_t g = 0;
#pragma unroll 1
  for (int p = 0; p < A.nphases; ++p) {
    const TkPhase& ph = A.phases[p];
    if (ph.kind != kTkGemv) continue;
    Geo geo;
    geo.init(ph, blockIdx.x, gridDim.x);
    const uint8_t* W = reinterpret_cast<const uint8_t*>(ph.w);
#pragma unroll 1
    for (int i = 0; i < geo.nslots; ++i, ++g) {
      const int s = (int)(g % kTkSlots);
      const uint32_t j = g / kTkSlots;
      mbar_wait(smem_u32(&sh.empty[s]), (j & 1u) ^ 1u, A.err);
      const int a = geo.r0 + i * geo.per;
      const int n = min(geo.per, geo.r1 - a);
      const uint32_t bytes = (uint32_t)n * geo.rb;
      const uint32_t full = smem_u32(&sh.full[s]);
      mbar_arrive_expect_tx(full, geo.sw ? 2u * bytes : bytes);
      bulk_g2s(smem_u32(sh.ring[s]), W + (size_t)a * geo.rb, bytes, full);
      if (geo.sw)
        bulk_g2s(smem_u32(sh.ring[s]) + (uint32_t)geo.per * geo.rb, W + (size_t)(geo.out_rows + a) * geo.rb, bytes,
                 full);
    }
  }
  // Every copy lands before the CTA can exit (bounded; the consumers normally saw them all).
#pragma unroll 1
  for (uint32_t s = 0; s < (uint32_t)kTkSlots && s < g; ++s) {
    const uint32_t fills = (g - s + kTkSlots - 1) / kTkSlots;
    mbar_wait(smem_u32(&sh.full[s]), (fills - 1u) & 1u, A.err);
  }
}

// ------------------------------------------------------------------------------------------
// Consumers
// ------------------------------------------------------------------------------------------

constexpr int kTkMaxChunks = kTkMaxK / 8 / kTkConsumers;  // 8-element chunks of x per thread (3)

// Prologue operands that do not depend on the previous phase (the norm weight, and for the gated
// GDN norm the gate z, written two phases earlier), loaded before the grid barrier.
struct TkPre {
  float w[kTkMaxChunks][8];
  float z[kTkMaxChunks][8];
};

__device__ __forceinline__ void ld8(float* d, const float* s) {
  const float4 a = __ldcg(reinterpret_cast<const float4*>(s));
  const float4 b = __ldcg(reinterpret_cast<const float4*>(s + 4));
  d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w;
  d[4] = b.x; d[5] = b.y; d[6] = b.z; d[7] = b.w;
}

__device__ __forceinline__ void tk_prefetch(const TkPhase& p, TkPre& pre) {
  const int nc = p.k / 8;
#pragma unroll
  for (int i = 0; i < kTkMaxChunks; ++i) {
    const int c = threadIdx.x + i * kTkConsumers;
    if (c < nc) {
      if (p.pro == kProRmsNorm || p.pro == kProEmbedNorm) ld8(pre.w[i], p.norm_w + c * 8);
      if (p.pro == kProGdnGate) {
        ld8(pre.z[i], p.zgate + c * 8);
        ld8(pre.w[i], p.norm_w + ((c * 8) & (kGdnDim - 1)));
      }
    }
  }
}

// Stages x of a GEMV phase as two planes (elements 0-3 and 4-7 of every 8-element chunk), so a
// lane's 16-byte reads of consecutive chunks are conflict-free, applying the prologue. RMSNorm is
// folded: the planes hold x * norm_w and the returned factor rsqrt(mean(x^2) + eps) scales the
// dot products in the epilogue (1 for the other prologues). One consumer barrier.
__device__ __forceinline__ float tk_stage(const TkPhase& p, const TkArgs& A, TkShared& sh, const TkPre& pre) {
  const int k = p.k, tid = threadIdx.x, nc = k / 8;
  float* xlo = sh.xs;
  float* xhi = sh.xs + k / 2;
  const bool norm = p.pro == kProRmsNorm || p.pro == kProEmbedNorm;
  float ss = 0.f;
  uint32_t token = 0;
  if (p.pro == kProEmbedNorm) {
    token = A.ctl->token;
    if (token >= (uint32_t)A.embed.rows) token = (uint32_t)A.embed.rows - 1;
  }
#pragma unroll
  for (int i = 0; i < kTkMaxChunks; ++i) {
    const int c = tid + i * kTkConsumers;
    if (c >= nc) break;
    float v[8];
    if (p.pro == kProEmbedNorm) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = deq_elem(A.embed, token, c * 8 + j);
      if (blockIdx.x == 0) {
        *reinterpret_cast<float4*>(A.h_out + c * 8) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(A.h_out + c * 8 + 4) = make_float4(v[4], v[5], v[6], v[7]);
      }
    } else {
      ld8(v, p.x + c * 8);
    }
    float cs = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) cs = fmaf(v[j], v[j], cs);
    ss += cs;
    if (norm) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] *= pre.w[i][j];
    } else if (p.pro == kProGdnGate) {
      // k == 2048 and 256 threads: one chunk per thread, 16 consecutive threads per 128-wide head.
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
      const float inv = rsqrtf(cs / (float)kGdnDim + 1e-6f);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = v[j] * inv * silu(pre.z[i][j]) * pre.w[i][j];
    }
    *reinterpret_cast<float4*>(xlo + c * 4) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(xhi + c * 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
  if (p.pro == kProEmbedNorm && blockIdx.x == 0 && tid == 0) A.ctl->count += 1;  // conv windows
  if (norm) {
    const float t = warp_sum(ss);
    if ((tid & 31) == 0) sh.red[tid >> 5] = t;
  }
  ConsumerBar()();
  if (!norm) return 1.f;
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kTkConsumerWarps; ++w) t += sh.red[w];
  return rsqrtf(t / (float)k + 1e-6f);
}

// Dot products of the R rows of one ring slot with x; every lane ends with the R sums.
template <int R>
__device__ __forceinline__ void tk_dot(const uint8_t* slot, const float* xs, int k, uint32_t rb, int lane,
                                       float (&acc)[R]) {
  float a[R];
#pragma unroll
  for (int r = 0; r < R; ++r) a[r] = 0.f;
  const float* xlo = xs;
  const float* xhi = xs + k / 2;
  constexpr int U = R >= 6 ? 2 : 4;  // 2 R (or 4 R) independent 16-byte loads in flight
#pragma unroll U
  for (int c = lane; c < k / 8; c += 32) {
    float xv[8];
    *reinterpret_cast<float4*>(xv) = *reinterpret_cast<const float4*>(xlo + c * 4);
    *reinterpret_cast<float4*>(xv + 4) = *reinterpret_cast<const float4*>(xhi + c * 4);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint4 w = *reinterpret_cast<const uint4*>(slot + (size_t)r * rb + (size_t)c * 16);
      a[r] += dot_f16(w, xv);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = warp_sum(a[r]);
}

template <int N>
__device__ __forceinline__ float pick(const float (&v)[N], int i) {
  float r = 0.f;
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (j == i) r = v[j];
  return r;
}

// The warp's slots of one GEMV phase (every 8th of the CTA's sequence), R rows per slot: wait for
// the slot, dot, release the slot to the producer; lane r applies the epilogue to output row r of
// the slot (the residual it adds is loaded before the dot). For SwiGLU the slot's rows are
// per = R / 2 gate rows, then the matching up rows. Each lane keeps its best greedy-pick candidate.
template <int R, bool SW>
__device__ __forceinline__ void tk_slots(const TkPhase& ph, const Geo& geo, const TkArgs& A, TkShared& sh, uint32_t g,
                                         float inv, float& best_v, uint32_t& best_i) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int OUT = SW ? R / 2 : R;
#pragma unroll 1
  for (int i = 0; i < geo.nslots; ++i) {
    const uint32_t gi = g + (uint32_t)i;
    if ((int)(gi % kTkSlots) != warp) continue;
    const uint32_t j = gi / kTkSlots;
    const int a = geo.r0 + i * geo.per;
    const int n = min(geo.per, geo.r1 - a);
    const float resid = (ph.epi == kAccumulate && lane < n) ? __ldcg(ph.y + a + lane) : 0.f;
    mbar_wait(smem_u32(&sh.full[warp]), j & 1u, A.err);
    float acc[R];
    tk_dot<R>(sh.ring[warp], sh.xs, geo.k, geo.rb, lane, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&sh.empty[warp]));
    if (lane < n) {
      const int row = a + lane;
      const float v = pick<R>(acc, lane) * inv;
      if (SW) {
        ph.y[row] = silu(v) * (pick<R>(acc, OUT + lane) * inv);
      } else if (ph.epi == kAccumulate) {
        ph.y[row] = resid + v;
      } else {
        ph.y[row] = v;
        if (ph.epi == kArgmax && v > -INFINITY && better(v, (uint32_t)row, best_v, best_i)) {
          best_v = v;
          best_i = (uint32_t)row;
        }
      }
    }
  }
}

__device__ __forceinline__ void tk_gemv(const TkPhase& ph, const TkArgs& A, TkShared& sh, uint32_t& g, float inv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Geo geo;
  geo.init(ph, blockIdx.x, gridDim.x);
  float best_v = -INFINITY;
  uint32_t best_i = 0xFFFFFFFFu;
  if (geo.sw) {
    switch (geo.R) {
      case 2: tk_slots<2, true>(ph, geo, A, sh, g, inv, best_v, best_i); break;
      case 6: tk_slots<6, true>(ph, geo, A, sh, g, inv, best_v, best_i); break;
      default: tk_slots<12, true>(ph, geo, A, sh, g, inv, best_v, best_i); break;
    }
  } else {
    switch (geo.R) {
      case 2: tk_slots<2, false>(ph, geo, A, sh, g, inv, best_v, best_i); break;
      case 3: tk_slots<3, false>(ph, geo, A, sh, g, inv, best_v, best_i); break;
      case 6: tk_slots<6, false>(ph, geo, A, sh, g, inv, best_v, best_i); break;
      default: tk_slots<12, false>(ph, geo, A, sh, g, inv, best_v, best_i); break;
    }
  }
  g += (uint32_t)geo.nslots;
  if (ph.epi != kArgmax) return;
  // Greedy pick: warp best, CTA best, then the last CTA reduces across CTAs and updates the
  // control words.
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
  ConsumerBar()();
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    uint32_t ix = 0xFFFFFFFFu;
    for (int w = 0; w < kTkConsumerWarps; ++w)
      if (better(sh.bval[w], sh.bidx[w], v, ix)) {
        v = sh.bval[w];
        ix = sh.bidx[w];
      }
    A.part_val[blockIdx.x] = v;
    A.part_idx[blockIdx.x] = ix;
    __threadfence();
    sh.flag = (atomicAdd(A.ticket, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  ConsumerBar()();
  if (sh.flag && warp == 0) {
    __threadfence();
    float v = -INFINITY;
    uint32_t ix = 0xFFFFFFFFu;
#pragma unroll 1
    for (int b = lane; b < (int)gridDim.x; b += 32) {
      const float bv = __ldcg(A.part_val + b);
      const uint32_t bi = __ldcg(A.part_idx + b);
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
      if (A.update_token) {
        A.ctl->token = (ix == 0xFFFFFFFFu) ? 0u : ix;
        A.ctl->pos += 1;
      }
      *A.ticket = 0u;
    }
  }
}

__device__ __forceinline__ void tk_consume(const TkArgs& A, TkShared& sh) {
  TkBarrier bar{A.barrier, 0ull, A.wait_limit_ns, A.wait_extra};
  uint32_t g = 0;
  pdl_wait();  // the previous token's control words and states are complete
#pragma unroll 1
  for (int p = 0; p < A.nphases; ++p) {
    const TkPhase& ph = A.phases[p];
    if (ph.kind == kTkGemv) {
      TkPre pre;
      tk_prefetch(ph, pre);
      if (p > 0) bar.wait(A.err);
      const float inv = tk_stage(ph, A, sh, pre);
      tk_gemv(ph, A, sh, g, inv);
    } else if (ph.kind == kTkGdn) {
      const bool mine = (int)blockIdx.x < kGdnItemsPerSeq;
      GdnItem it;
      if (mine) it.prefetch(ph.gdn, blockIdx.x);  // the state slice, before the barrier
      bar.wait(A.err);
      if (mine) it.run_with(ph.gdn, *reinterpret_cast<GdnShared*>(sh.xs), ConsumerBar());
    }
    if (p + 1 < A.nphases) bar.arrive();
  }
  bar.exit();
}

__global__ void __launch_bounds__(kTkThreads, 1) token_kernel(const __grid_constant__ TkArgs A) {
  extern __shared__ __align__(128) uint8_t tk_smem[];
  TkShared& sh = *reinterpret_cast<TkShared*>(tk_smem);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTkSlots; ++s) {
      mbar_init(smem_u32(&sh.full[s]), 1);
      mbar_init(smem_u32(&sh.empty[s]), 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch();
  if ((threadIdx.x >> 5) == kTkConsumerWarps) {
    if ((threadIdx.x & 31) == 0) tk_produce(A, sh);
    return;
  }
  tk_consume(A, sh);
}

}  // namespace

bool token_gemv_ok(int rows, int k, int epi) {
  if (k < 256 || k > kTkMaxK || k % 256 || rows < 1) return false;
  if (epi == kSwiGlu && (rows % 2 || (size_t)4 * k > kTkSlotBytes)) return false;
  return true;
}

int token_ctas() {
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  const int smem = (int)sizeof(TkShared);
  if (cudaFuncSetAttribute(token_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, token_kernel, kTkThreads, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  // One CTA per SM, all co-resident (the grid barriers need it); the GDN phase needs a CTA per item.
  if (per_sm < 1 || sms < kGdnItemsPerSeq || sms > kMaxGrid) return 0;
  return sms;
}

cudaError_t launch_token(const TkArgs& args, int ctas, cudaStream_t stream, bool pdl) {
  const int smem = (int)sizeof(TkShared);
  cudaError_t e = cudaFuncSetAttribute(token_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kTkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  return cudaLaunchKernelEx(&cfg, token_kernel, args);
}

}  // namespace qne
