// Batched linear layers on the 5th-generation tensor cores: Y[b] (=, +=, SwiGLU) W X[b] for up
// to 64 activation rows (batched decode sequences or the tokens of a prompt chunk).
//
// Same arithmetic as gemm.cu (the per-token GEMV of kernels/src/shaders.rs:48-250 applied to B
// rows; the reference's prompt GEMM is batch::gemm, kernels/src/batch.rs:16-99): f16 weights,
// activations as two f16 planes hi = f16(x), lo = f16(x - hi), both multiplied into one f32
// accumulator.
//
// B200 design (tcgen05 + TMA + TMEM, one CTA of 4 warps per tile):
//  * a tile is 128 weight rows (SwiGLU: 64 gate rows and the matching 64 up rows) by the whole
//    activation batch (N = 16, 32 or 64 columns of the MMA, zero-filled past the batch);
//  * warp 0 lane 0 streams 64-wide k-blocks of the weight tile and of both activation planes
//    with TMA (128-byte swizzle, the canonical K-major layout of the MMA operands) into a 6-stage
//    ring guarded by mbarriers (3 stages, three CTAs per SM, when the tiles fill more than two
//    waves, as in the batched LM head); weight loads of the first stages are issued before
//    waiting on the previous kernel, whose output the activations are;
//  * warp 1 lane 0 issues tcgen05.mma (M = 128, K = 16, f32 accumulators in tensor memory), one
//    of width 2N per k-step over the hi and lo tiles together, and frees each stage with
//    tcgen05.commit;
//  * split-K runs across the CTAs of a thread-block cluster, each CTA owning a slice of the
//    tile's output rows. Where a receive area fits beside the ring (N <= 32), every CTA stores
//    each accumulator row from tensor memory straight into the receive area of the row's owner
//    (st.shared::cluster, posted), and after one cluster barrier the owner sums its slice over
//    the ranks in rank order from its own shared memory; otherwise (N = 64) every CTA moves its
//    accumulator to its own shared memory and the owners read the other ranks' partials through
//    the cluster window. Either way the sum is deterministic, and the owner applies the epilogue
//    (store, accumulate, or SwiGLU written as the next GEMM's hi/lo planes).
// No load uses cluster multicast: every CTA fetches its own tiles.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <map>
#include <mutex>
#include <tuple>

#include "batch.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace qne {
namespace {

constexpr int kTcThreads = 128;
constexpr int kTcStages = 6;      // ring depth of one CTA per SM (most GEMMs: one wave of tiles)
constexpr int kTcStagesWide = 3;  // many waves of tiles (the batched LM head): three CTAs per SM,
                                  // so CTAs' epilogues overlap the others' weight streams
constexpr int kBK = 64;                 // k per stage: one 128-byte swizzle span of f16
constexpr int kTileA = 128 * kBK * 2;   // 16 KB of weights per stage
constexpr int kMaxCluster = 8;
constexpr int kSumsqLd = kGemmMaxRows;  // folded-norm partials: [16-row block][kGemmMaxRows columns]
constexpr int kCtaSlots = kNumSms;  // one CTA per SM fits (about 145 KB of shared memory)

struct TcArgs {
  int out_rows;     // output rows (SwiGLU: rows / 2)
  int batch;
  int kblocks;      // ceil(k / 64)
  int kb_per_rank;  // k-blocks per cluster rank
  int half;         // SwiGLU: first up row
  int epi;
  float* y;
  uint16_t* yh;
  uint16_t* yl;
  int ldy;
  uint32_t* err;
  // folded RMSNorm (see GemmArgs)
  const float* norm_w_out;
  uint16_t* out_xh;
  uint16_t* out_xl;
  int out_ldx;
  float* sumsq_out;
  const float* sumsq_in;
  int sumsq_slots, norm_k;
  float eps;
  int w_after_wait;  // weights written by the previous kernel: no weight loads before the wait
  // int4 weights (kernel instances with Q != kF16): the packed nibbles come through `tw`, the
  // scales and zero points are read directly.
  int rows;       // physical rows
  int k;
  const void* ws;
  const void* wz;
};

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  // K-major operand, 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart.
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

template <int N>
__host__ __device__ constexpr uint32_t instr_desc_f16() {
  // f32 accumulator, f16 A and B, both K-major, M = 128.
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void tmem_load_row(uint32_t taddr, float* v);

template <>
__device__ __forceinline__ void tmem_load_row<16>(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <>
__device__ __forceinline__ void tmem_load_row<32>(uint32_t taddr, float* v) {
  tmem_load_row<16>(taddr, v);
  tmem_load_row<16>(taddr + 16, v + 16);
}

template <>
__device__ __forceinline__ void tmem_load_row<64>(uint32_t taddr, float* v) {
  tmem_load_row<32>(taddr, v);
  tmem_load_row<32>(taddr + 32, v + 32);
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  return remote;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
// Volatile keeps the loads after the cluster barrier; callers issue the loads of all ranks
// before the sums that consume them, so they are in flight together.
__device__ __forceinline__ float4 ld_cluster_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}

// f16x2 helpers of the int4 converters (round to nearest, subnormals kept).
__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t prmt_u(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// Nibbles i and i + 4 of w as the f16 pair (1024 + n_i, 1024 + n_{i+4}).
__device__ __forceinline__ uint32_t nib_pair_1024(uint32_t w, int i) {
  uint32_t r;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(r) : "r"(w >> (4 * i)));  // (a & b) | c
  return r;
}

__device__ __forceinline__ void split_hilo_tc(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

// Push mode (split-K partials sent to their owners' receive areas) when the receive area fits
// beside the stage ring; the other instances read the partials through the cluster window.
template <int N, int ST, int Q>
__host__ __device__ constexpr int stage_bytes() {
  return kTileA + 2 * N * kBK * 2 + (Q != kF16 ? 128 * kBK / 2 : 0);
}
template <int N>
__host__ __device__ constexpr int recv_bytes() {
  return 128 * (N + 4) * 4;
}
template <int N, int ST, int Q>
__host__ __device__ constexpr bool push_mode() {
  return ST == kTcStages && ST * stage_bytes<N, ST, Q>() + 1024 + recv_bytes<N>() + 4096 <= 232448;
}

template <int N, bool SW, int ST, int Q>
__global__ void __launch_bounds__(Q != kF16 ? 2 * kTcThreads : kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap txh,
                   const __grid_constant__ CUtensorMap txl, const __grid_constant__ TcArgs a) {
  extern __shared__ uint8_t dsm_raw[];
  constexpr bool kQ = Q != kF16;  // int4 weights, widened to f16 in shared memory
  __shared__ __align__(8) uint64_t full[ST], empty[ST], accb, rawf[kQ ? ST : 1], conv[kQ ? ST : 1];
  __shared__ uint32_t tmem_slot;
  __shared__ float inv_s[kGemmMaxRows];
  constexpr int kTileB = N * kBK * 2;  // one activation plane per stage
  constexpr int kLoadF16 = kTileA + 2 * kTileB;  // bytes of one stage's TMA loads (f16 weights)
  constexpr int kRaw = kQ ? 128 * kBK / 2 : 0;   // int4: the stage's packed nibbles (4 KB)
  constexpr int kStage = kTileA + 2 * kTileB + kRaw;
  static_assert(kStage == stage_bytes<N, ST, Q>(), "stage layout");
  constexpr int kTmemCols = 2 * N < 32 ? 32 : 2 * N;  // accumulator columns: N of hi, then N of lo
  constexpr int kPitch = N + 4;  // partial rows in shared memory: 16-byte aligned, conflict-free v4 stores
  constexpr bool kPush = push_mode<N, ST, Q>();  // split-K partials pushed to their owners
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(base);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int nrank = (int)(gridDim.x);
  const int tile = blockIdx.y;
  const int kb0 = (int)rank * a.kb_per_rank;
  const int nkb = max(0, min(a.kb_per_rank, a.kblocks - kb0));

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "n"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
      if (kQ) {
        mbar_init(smem_u32(&rawf[s]), 1);
        mbar_init(smem_u32(&conv[s]), 4);  // one arrival per converter warp
      }
    }
    mbar_init(smem_u32(&accb), 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // Push mode: the first cluster barrier phase tells each rank that every rank has started, so
  // its receive area may be written; arrive now, wait just before the pushes.
  if (kPush) cluster_arrive_relaxed();
  pdl_launch();

  bool ok = true;
  if (warp == 0 && lane == 0 && nkb > 0) {
    // Producer. Weight tiles do not depend on the previous kernel: the first stages' weights go
    // out before the dependency wait, their activation tiles after it (unless the previous
    // kernel wrote the weights, w_after_wait).
    const int r0 = SW ? tile * 64 : tile * 128;
    auto load_a = [&](int i) {
      const uint32_t st = sbase + (uint32_t)((i % ST) * kStage);
      const int kx = (kb0 + i) * kBK;
      if (kQ) {
        // packed nibbles: 32 bytes of every row of the tile, into the stage's raw area
        const uint32_t bar = smem_u32(&rawf[i % ST]);
        const uint32_t raw = st + (uint32_t)(kTileA + 2 * kTileB);
        mbar_arrive_expect_tx(bar, (uint32_t)kRaw);
        if (SW) {
          tma_load_2d(raw, &tw, kx / 2, r0, bar);
          tma_load_2d(raw + kRaw / 2, &tw, kx / 2, a.half + r0, bar);
        } else {
          tma_load_2d(raw, &tw, kx / 2, r0, bar);
        }
        return;
      }
      const uint32_t bar = smem_u32(&full[i % ST]);
      mbar_arrive_expect_tx(bar, (uint32_t)kLoadF16);
      if (SW) {
        tma_load_2d(st, &tw, kx, r0, bar);
        tma_load_2d(st + kTileA / 2, &tw, kx, a.half + r0, bar);
      } else {
        tma_load_2d(st, &tw, kx, r0, bar);
      }
    };
    auto load_b = [&](int i) {
      const uint32_t st = sbase + (uint32_t)((i % ST) * kStage);
      const uint32_t bar = smem_u32(&full[i % ST]);
      const int kx = (kb0 + i) * kBK;
      if (kQ) mbar_arrive_expect_tx(bar, (uint32_t)(2 * kTileB));
      tma_load_2d(st + kTileA, &txh, kx, 0, bar);
      tma_load_2d(st + kTileA + kTileB, &txl, kx, 0, bar);
    };
    const int pre = min(ST, nkb);
    if (!a.w_after_wait)
      for (int i = 0; i < pre; ++i) load_a(i);
    pdl_wait();
    if (a.w_after_wait)
      for (int i = 0; i < pre; ++i) load_a(i);
    for (int i = 0; i < pre; ++i) load_b(i);
    for (int i = pre; i < nkb; ++i) {
      if (!mbar_wait(smem_u32(&empty[i % ST]), (uint32_t)((i / ST) + 1) & 1u, a.err)) {
        ok = false;
        break;
      }
      load_a(i);
      load_b(i);
    }
  } else if (warp == 1 && lane == 0 && nkb > 0) {
    // MMA issuer: 4 k-steps of 16 per stage. The hi and lo activation tiles sit back to back in
    // the stage, which is the layout of one operand of 2N rows: one MMA of width 2N per k-step
    // (the tensor core's cost here is per instruction, so this halves the MMA time); accumulator
    // columns [0, N) collect W x_hi and [N, 2N) W x_lo, added in the epilogue.
    constexpr uint32_t idesc = instr_desc_f16<2 * N>();
    for (int i = 0; i < nkb; ++i) {
      const int s = i % ST;
      if (!mbar_wait(smem_u32(&full[s]), (uint32_t)(i / ST) & 1u, a.err) ||
          (kQ && !mbar_wait(smem_u32(&conv[s]), (uint32_t)(i / ST) & 1u, a.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t st = sbase + (uint32_t)(s * kStage);
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        const uint64_t ad = smem_desc_sw128(st + kk * 32);
        mma_f16(tmem, ad, smem_desc_sw128(st + kTileA + kk * 32), idesc, (i | kk) != 0);
      }
      mma_commit(smem_u32(&empty[s]));
    }
    mma_commit(smem_u32(&accb));
  } else if (kQ && warp >= 4 && nkb > 0) {
    // Converters (warps 4-7, int4 instances only): thread t widens row t of every stage's weight
    // tile into the 128-byte-swizzled K-major layout the MMA reads (16-byte chunk c of row r at
    // c ^ (r % 8)). The row's scales and zero points of a stage are loaded four stages ahead.
    const int t = tid - 128;
    const int r0 = SW ? tile * 64 : tile * 128;
    long prow[1];
    {
      const int ar = t;
      const long phys = SW ? (ar < 64 ? (long)r0 + ar : (long)a.half + r0 + ar - 64) : (long)r0 + ar;
      prow[0] = phys < a.rows ? phys : (long)a.rows - 1;  // rows past the matrix: read as zero, never stored
    }
    uint32_t sq[4][1], zq[4][1];
    auto load_sz = [&](int i, uint32_t (&sv)[1], uint32_t (&zv)[1]) {
#pragma unroll
      for (int rr = 0; rr < 1; ++rr) {
        sv[rr] = 0u;
        zv[rr] = 0u;
        if (i < nkb) {
          const int kb = kb0 + i;
          if (Q == kQ4) {  // f16 scale pair per 64 values, 8 zero-point nibbles per 256
            sv[rr] = __ldg(static_cast<const uint32_t*>(a.ws) + prow[rr] * (a.k / 64) + kb);
            zv[rr] = __ldg(static_cast<const uint32_t*>(a.wz) + prow[rr] * (a.k / 256) + kb / 4);
          } else {         // f16 scale and zero point per 64 values
            sv[rr] = __ldg(static_cast<const uint16_t*>(a.ws) + prow[rr] * (a.k / 64) + kb);
            zv[rr] = __ldg(static_cast<const uint16_t*>(a.wz) + prow[rr] * (a.k / 64) + kb);
          }
        }
      }
    };
#pragma unroll
    for (int j = 0; j < 4; ++j) load_sz(j, sq[j], zq[j]);
    for (int i0 = 0; i0 < nkb && ok; i0 += 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = i0 + j;
        if (i >= nkb || !ok) break;  // uniform across the two converter warps
        const int s = i % ST;
        if (!mbar_wait(smem_u32(&rawf[s]), (uint32_t)(i / ST) & 1u, a.err)) {
          ok = false;
          break;
        }
        uint8_t* A = base + (size_t)s * kStage;
        const uint8_t* raw = A + kTileA + 2 * kTileB;
        const int kb = kb0 + i;
#pragma unroll
        for (int rr = 0; rr < 1; ++rr) {
          const int ar = t;
          const uint4 w0 = *reinterpret_cast<const uint4*>(raw + ar * 32);
          const uint4 w1 = *reinterpret_cast<const uint4*>(raw + ar * 32 + 16);
          const uint32_t wd[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
          // Per block (words 0-3 and 4-7: one block-32 block each, one group-64 group), f16x2
          // constants. Block-32 (integer zero point): (1024 + q) - (1024 + zp) is the exact
          // integer q - zp and one f16x2 multiply rounds (q - zp) * scale once, the value the
          // per-token kernels use. Group-64 (f16 zero point): q * scale + f16(-zp * scale) in one
          // f16x2 fma (within an f16 unit of the f32 form).
          uint32_t ca[2], cb[2];
          if (Q == kQ4) {
            const uint32_t z0 = (zq[j][rr] >> (4 * (2 * (kb & 3)))) & 15u, z1 = (zq[j][rr] >> (4 * (2 * (kb & 3) + 1))) & 15u;
            ca[0] = 0x64006400u | z0 | (z0 << 16);
            ca[1] = 0x64006400u | z1 | (z1 << 16);
            cb[0] = prmt_u(sq[j][rr], sq[j][rr], 0x1010u);  // scale of block 2kb in both halves
            cb[1] = prmt_u(sq[j][rr], sq[j][rr], 0x3232u);  // block 2kb + 1
          } else {
            const uint32_t sh = sq[j][rr] & 0xFFFFu;
            const uint32_t cz = __half_as_ushort(__float2half_rn(-h2f((uint16_t)zq[j][rr]) * h2f((uint16_t)sh)));
            ca[0] = ca[1] = cz | (cz << 16);
            cb[0] = cb[1] = sh | (sh << 16);
          }
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t p = nib_pair_1024(wd[c], e);  // (1024 + n_e, 1024 + n_{e+4})
              v[e] = Q == kQ4 ? hmul2_u(hsub2_u(p, ca[c >> 2]), cb[c >> 2])
                              : hfma2_u(hsub2_u(p, 0x64006400u), cb[c >> 2], ca[c >> 2]);
            }
            // v[e] = (value e, value e + 4): back to the natural order (0,1) (2,3) (4,5) (6,7)
            *reinterpret_cast<uint4*>(A + ar * 128 + ((c ^ (ar & 7)) << 4)) =
                make_uint4(prmt_u(v[0], v[1], 0x5410u), prmt_u(v[2], v[3], 0x5410u), prmt_u(v[0], v[1], 0x7632u),
                           prmt_u(v[2], v[3], 0x7632u));
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> the MMA's operand reads
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&conv[s]));
        load_sz(i + 4, sq[j], zq[j]);
      }
    }
  }
  __syncwarp();

  // Epilogue geometry. Thread work item: one output row j and 4 consecutive batch columns;
  // consecutive threads take consecutive rows, so each of the 4 output stores is coalesced, and a
  // half-warp covers one 16-row block of one column group (the unit of the folded-norm partials).
  constexpr int kOutTile = SW ? 64 : 128;
  constexpr int kIt = kOutTile * (N / 4) / kTcThreads;  // work items per thread at most (1 rank, N columns)
  // Residual values prefetched into registers during the MMAs (kIt of them per thread); at
  // N = 64 that would be 64 more registers, so there the epilogue reads them when it stores.
  constexpr int kYv = kIt <= 8 ? kIt : 1;
  const int slice = kOutTile / nrank;  // a power of two (cluster sizes are)
  const int slice_log2 = __ffs(slice) - 1;
  const int o0 = (int)rank * slice;
  const int B = a.batch;
  const int groups = (B + 3) / 4;
  const int total = slice * groups;
  auto item_of = [&](int it, int& b0, int& j) {
    const int e = it * kTcThreads + tid;
    b0 = (e >> slice_log2) * 4;
    j = o0 + (e & (slice - 1));
    return tid < kTcThreads && e < total;  // the converter warps of the int4 instances hold no items
  };

  // What depends only on the previous kernel is fetched while the MMAs run: the consumer's 1/rms
  // per activation row (warps 2-3, unrolled loads, fixed summation order) and the residual values
  // an accumulating epilogue adds to.
  pdl_wait();
  if (a.sumsq_in && tid >= 64 && tid < 64 + B) {
    const int b = tid - 64;
    float ss = 0.f;
    for (int q0 = 0; q0 < a.sumsq_slots; q0 += 32) {  // 32 loads in flight, then the sums in order
      float v[32];
#pragma unroll
      for (int q = 0; q < 32; ++q) v[q] = q0 + q < a.sumsq_slots ? a.sumsq_in[(q0 + q) * kSumsqLd + b] : 0.f;
#pragma unroll
      for (int q = 0; q < 32; ++q) ss += v[q];
    }
    inv_s[b] = rsqrtf(ss / (float)a.norm_k + a.eps);
  }
  float yv[SW ? 1 : kYv][4];
  if (!SW && kYv == kIt && a.epi == kAccumulate) {
#pragma unroll
    for (int it = 0; it < (SW ? 1 : kYv); ++it) {
      int b0, j;
      const bool act = item_of(it, b0, j);
      const int orow = tile * kOutTile + j;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        yv[it][i] = (act && orow < a.out_rows && b0 + i < B) ? a.y[(size_t)(b0 + i) * a.ldy + orow] : 0.f;
    }
  }

  // Accumulator -> shared memory. Pull mode: each rank's own partial goes to its stage ring (free
  // once accb fired: every MMA completed, so every TMA load it consumed had landed), and the
  // owners read the other ranks' partials through the cluster window. Push mode: thread t sends
  // row t of the tile to the receive area of the rank that owns that output row (a region of its
  // own after the ring, so a rank still streaming is not disturbed), at [source rank][row of the
  // owner's slice], and the owners sum in their own shared memory after one cluster barrier.
  // Thread t holds row t of the tile.
  float* part = reinterpret_cast<float*>(base);
  float* recv = reinterpret_cast<float*>(base + (size_t)ST * kStage);
  const int rows_per_src = SW ? 2 * slice : slice;
  if (kPush) cluster_wait();  // every rank has started (first barrier phase)
  if (warp < 4) {  // the tile's 128 accumulator lanes (the int4 converter warps hold none)
    float v[N];
    if (nkb > 0) {
      if (!mbar_wait(smem_u32(&accb), 0u, a.err)) ok = false;
      tc_fence_after();
      const uint32_t row = tmem + ((uint32_t)(warp * 32) << 16);
      float u[N];
      tmem_load_row<N>(row, v);
      tmem_load_row<N>(row + (uint32_t)N, u);
#pragma unroll
      for (int c = 0; c < N; ++c) v[c] += u[c];  // W x_hi + W x_lo
    } else {
#pragma unroll
      for (int c = 0; c < N; ++c) v[c] = 0.f;
    }
    if (!ok) {
#pragma unroll
      for (int c = 0; c < N; ++c) v[c] = 0.f;
    }
    if (kPush) {
      const int orow_t = SW ? (tid & 63) : tid;  // output row of the tile this accumulator row feeds
      const int q = orow_t >> slice_log2;        // its owner rank
      const int lr = (SW ? (tid >> 6) * slice : 0) + (orow_t - q * slice);
      const uint32_t dst =
          cluster_addr(smem_u32(recv) + (uint32_t)(((int)rank * rows_per_src + lr) * kPitch * 4), (uint32_t)q);
#pragma unroll
      for (int c = 0; c < N; c += 4) st_cluster_v4(dst + (uint32_t)(c * 4), v[c], v[c + 1], v[c + 2], v[c + 3]);
    } else {
#pragma unroll
      for (int c = 0; c < N; c += 4)
        *reinterpret_cast<float4*>(part + tid * kPitch + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
    }
  }

  tc_fence_before();
  cluster_sync_all();  // every rank's partial is in its shared memory (and inv_s is visible)

  // Reduction over the cluster's ranks, in rank order: all remote reads first, then this CTA
  // signals that it is done reading, and the epilogue math and stores overlap the other ranks.
  const uint32_t pbase = smem_u32(part);
  float vv[kIt][4], uu[SW ? kIt : 1][4];
#pragma unroll
  for (int it = 0; it < kIt; ++it) {
    int b0, j;
    const bool act = item_of(it, b0, j);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      vv[it][i] = 0.f;
      if (SW) uu[SW ? it : 0][i] = 0.f;
    }
    if (act) {
      float4 pv[kMaxCluster], pu[kMaxCluster];
      if (kPush) {
        const int lr = j - o0;
#pragma unroll
        for (int q = 0; q < kMaxCluster; ++q) {
          if (q < nrank) {
            pv[q] = *reinterpret_cast<const float4*>(recv + (size_t)((q * rows_per_src + lr) * kPitch + b0));
            if (SW) pu[q] = *reinterpret_cast<const float4*>(recv + (size_t)((q * rows_per_src + slice + lr) * kPitch + b0));
          }
        }
      } else {
#pragma unroll
        for (int q = 0; q < kMaxCluster; ++q) {
          if (q < nrank) {
            pv[q] = ld_cluster_v4(cluster_addr(pbase + (uint32_t)((j * kPitch + b0) * 4), (uint32_t)q));
            if (SW) pu[q] = ld_cluster_v4(cluster_addr(pbase + (uint32_t)(((64 + j) * kPitch + b0) * 4), (uint32_t)q));
          }
        }
      }
#pragma unroll
      for (int q = 0; q < kMaxCluster; ++q) {
        if (q < nrank) {
          vv[it][0] += pv[q].x;
          vv[it][1] += pv[q].y;
          vv[it][2] += pv[q].z;
          vv[it][3] += pv[q].w;
          if (SW) {
            uu[SW ? it : 0][0] += pu[q].x;
            uu[SW ? it : 0][1] += pu[q].y;
            uu[SW ? it : 0][2] += pu[q].z;
            uu[SW ? it : 0][3] += pu[q].w;
          }
        }
      }
    }
  }
  if (!kPush) cluster_arrive();

#pragma unroll
  for (int it = 0; it < kIt; ++it) {
    if (it * kTcThreads >= total) break;  // uniform across the CTA
    int b0, j;
    const bool act = item_of(it, b0, j);
    const int orow = tile * kOutTile + j;
    float sq[4] = {0.f, 0.f, 0.f, 0.f};
    if (act && orow < a.out_rows) {
      // The four columns are independent: their arithmetic is unconditional, so it interleaves,
      // and only the stores (and loads) of columns past the batch are predicated off.
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int b = b0 + i;
        const bool in = b < B;
        float v = vv[it][i], u = SW ? uu[SW ? it : 0][i] : 0.f;
        if (a.sumsq_in) {
          const float is = inv_s[b < kGemmMaxRows ? b : kGemmMaxRows - 1];
          v *= is;
          u *= is;
        }
        if (SW) {
          __half hi, lo;
          split_hilo_tc(silu(v) * u, hi, lo);
          if (in) {
            a.yh[(size_t)b * a.ldy + orow] = __half_as_ushort(hi);
            a.yl[(size_t)b * a.ldy + orow] = __half_as_ushort(lo);
          }
        } else if (a.epi == kAccumulate) {
          const float prev = kYv == kIt ? yv[SW || kYv != kIt ? 0 : it][i] : (in ? a.y[(size_t)b * a.ldy + orow] : 0.f);
          const float hn = prev + v;
          if (in) a.y[(size_t)b * a.ldy + orow] = hn;
          if (a.norm_w_out) {
            // producer of a folded RMSNorm: the next GEMM's planes of h * norm_w, and h^2
            __half hi, lo;
            split_hilo_tc(hn * a.norm_w_out[orow], hi, lo);
            if (in) {
              a.out_xh[(size_t)b * a.out_ldx + orow] = __half_as_ushort(hi);
              a.out_xl[(size_t)b * a.out_ldx + orow] = __half_as_ushort(lo);
            }
            sq[i] = in ? hn * hn : 0.f;
          }
        } else if (in) {
          a.y[(size_t)b * a.ldy + orow] = v;
        }
      }
    }
    if (a.sumsq_out) {
      // sums over the 16 rows of this half-warp's block, one partial per (block, column)
#pragma unroll
      for (int o = 1; o < 16; o <<= 1)
#pragma unroll
        for (int i = 0; i < 4; ++i) sq[i] += __shfl_xor_sync(0xffffffffu, sq[i], o);
      const int blk = (tile * kOutTile + j) / 16;
      if (act && (j & 15) == 0 && blk * 16 < a.out_rows) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (b0 + i < B) a.sumsq_out[blk * kSumsqLd + b0 + i] = sq[i];
      }
    }
  }
  if (!kPush) cluster_wait();  // no CTA leaves while another still reads its shared memory
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kTmemCols) : "memory");
  }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

// 2-D f16 tensor [outer][inner] with rows `row_bytes` apart; box = box_inner x box_outer,
// 128-byte swizzle (box_inner = 64 f16). Out-of-range elements read as zero.
bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
              uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)kBK, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D byte tensor [outer][inner] (int4 weights: the packed nibbles of a row), no swizzle; box =
// 32 bytes (one 64-value k-block) x box_outer rows.
bool make_map_u8(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(kBK / 2), box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Clusters of `ranks` CTAs that can be resident at once (cached per device, kernel and size).
template <typename K>
int max_clusters(K kernel, size_t smem, int ranks, int threads) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, reinterpret_cast<const void*>(kernel), ranks);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ranks, 1);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ranks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = kCtaSlots / ranks;  // fall back to the one-CTA-per-SM estimate
  }
  cache[key] = n;
  return n;
}

template <int N, bool SW, int ST, int Q>
cudaError_t launch_tc(const GemmArgs& g, cudaStream_t stream, bool pdl) {
  auto kernel = gemm_tc_kernel<N, SW, ST, Q>;
  constexpr int kStage = stage_bytes<N, ST, Q>();
  const size_t smem = (size_t)ST * kStage + 1024 + (push_mode<N, ST, Q>() ? recv_bytes<N>() : 0);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  TcArgs a;
  a.out_rows = SW ? g.rows / 2 : g.rows;
  a.batch = g.batch;
  a.kblocks = (g.k + kBK - 1) / kBK;
  a.half = SW ? g.rows / 2 : 0;
  a.epi = g.epi;
  a.y = g.y;
  a.yh = g.yh;
  a.yl = g.yl;
  a.ldy = g.ldy;
  a.err = g.err;
  a.norm_w_out = g.norm_w_out;
  a.out_xh = g.out_xh;
  a.out_xl = g.out_xl;
  a.out_ldx = g.out_ldx;
  a.sumsq_out = g.sumsq_out;
  a.sumsq_in = g.sumsq_in;
  a.sumsq_slots = g.sumsq_slots;
  a.norm_k = g.norm_k;
  a.eps = g.eps;
  a.w_after_wait = g.w_after_wait ? 1 : 0;
  a.rows = g.rows;
  a.k = g.k;
  a.ws = g.ws;
  a.wz = g.wz;
  const int out_tile = SW ? 64 : 128;
  const int tiles = (a.out_rows + out_tile - 1) / out_tile;
  // Split k over a cluster: the largest power of two whose clusters (one per tile) all fit on
  // the device at once, with every rank at two k-blocks or more.
  int ranks = 1;
  constexpr int kThreadsLaunch = Q != kF16 ? 2 * kTcThreads : kTcThreads;  // int4: + 4 converter warps
  while (ranks < kMaxCluster && a.kblocks >= ranks * 4 && tiles <= max_clusters(kernel, smem, ranks * 2, kThreadsLaunch))
    ranks *= 2;
  a.kb_per_rank = (a.kblocks + ranks - 1) / ranks;
  const int x_rows = g.x_rows > 0 ? g.x_rows : (g.batch + 7) / 8 * 8;
  CUtensorMap tw, txh, txl;
  const bool wmap = Q != kF16 ? make_map_u8(&tw, g.w, (uint64_t)g.k / 2, (uint64_t)g.rows, (uint64_t)g.k / 2, SW ? 64 : 128)
                              : make_map(&tw, g.w, (uint64_t)g.k, (uint64_t)g.rows, (uint64_t)g.k * 2, SW ? 64 : 128);
  if (!wmap ||
      !make_map(&txh, g.xh, (uint64_t)g.k, (uint64_t)x_rows, (uint64_t)g.ldx * 2, N) ||
      !make_map(&txl, g.xl, (uint64_t)g.k, (uint64_t)x_rows, (uint64_t)g.ldx * 2, N))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ranks, tiles);
  cfg.blockDim = dim3(kThreadsLaunch);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ranks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kernel, tw, txh, txl, a);
}

template <int N, bool SW>
cudaError_t launch_tc_nsw(const GemmArgs& g, cudaStream_t stream, bool pdl) {
  const int out_tile = SW ? 64 : 128;
  const int tiles = ((SW ? g.rows / 2 : g.rows) + out_tile - 1) / out_tile;
  if (g.wkind == kQ4) return launch_tc<N, SW, kTcStages, kQ4>(g, stream, pdl);
  if (g.wkind == kQ4G64) return launch_tc<N, SW, kTcStages, kQ4G64>(g, stream, pdl);
  if (!SW && tiles > 2 * kCtaSlots) return launch_tc<N, SW, kTcStagesWide, kF16>(g, stream, pdl);
  return launch_tc<N, SW, kTcStages, kF16>(g, stream, pdl);
}

}  // namespace

bool gemm_tc_available() { return encode_fn() != nullptr; }

bool gemm_int4_direct(const GemmArgs& g) {
  if (g.wkind != kQ4 && g.wkind != kQ4G64) return false;
  if (g.impl != kGemmTensorCore || !gemm_tc_available() || g.w_after_wait || !g.ws || !g.wz) return false;
  if (g.k % (g.wkind == kQ4 ? 256 : 64) || g.batch < 1 || g.batch > kGemmMaxRows) return false;
  if (reinterpret_cast<uintptr_t>(g.w) % 16 || (size_t)g.k / 2 % 16) return false;
  // the many-wave case (the batched LM head) keeps the f16 route: it runs three CTAs per SM
  const bool sw = g.epi == kSwiGlu;
  const int tiles = ((sw ? g.rows / 2 : g.rows) + (sw ? 63 : 127)) / (sw ? 64 : 128);
  return sw || tiles <= 2 * kCtaSlots;
}

cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t stream, bool pdl) {
  const bool sw = g.epi == kSwiGlu;
  if (g.batch <= 16) return sw ? launch_tc_nsw<16, true>(g, stream, pdl) : launch_tc_nsw<16, false>(g, stream, pdl);
  if (g.batch <= 32) return sw ? launch_tc_nsw<32, true>(g, stream, pdl) : launch_tc_nsw<32, false>(g, stream, pdl);
  return sw ? launch_tc_nsw<64, true>(g, stream, pdl) : launch_tc_nsw<64, false>(g, stream, pdl);
}

}  // namespace qne
