// Batched decode linear layers: Y[b] (=, +=, SwiGLU) W X[b] for B independent sequences.
//
// Same arithmetic as the B=1 GEMV (gemv / gemv_f16, kernels/src/shaders.rs:48-250) applied to
// B activation vectors at once; the reference decodes one sequence at a time and has no such
// kernel, its closest relative is the 16-token prompt GEMM batch::gemm (kernels/src/batch.rs:16-99).
//
// B200 design. With B >= 2 every weight element feeds B multiply-adds, so the work goes to the
// tensor cores (mma.m16n8k16, f16 inputs, f32 accumulators):
//  * activations arrive as two f16 planes, hi = f16(x) and lo = f16(x - hi); both are multiplied
//    into the same f32 accumulator, which keeps the product accurate to ~2^-22 relative, close to
//    the f32 arithmetic of the single-sequence path;
//  * a warp owns 16 weight rows (32 for SwiGLU: gate and up) and a slice of k; each lane streams
//    its own 16-byte weight chunks through a private cp.async ring in shared memory (8 stages in
//    flight) and reads the activation fragments with 16-byte loads: the k order inside every
//    32-wide step is permuted identically for weights and activations, so one 16-byte load per
//    row (and per sequence group) supplies the fragments of two MMAs;
//  * warps of a CTA split k when there are few rows, and reduce through shared memory;
//  * the epilogue stores or accumulates f32 outputs, or applies SwiGLU and writes the result
//    directly as the hi/lo planes the next GEMM reads.
#include <math.h>

#include <algorithm>

#include "batch.cuh"
#include "gemv.cuh"

namespace qne {
namespace {

constexpr int kThreads = 256;
constexpr int kStages = 8;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void split_hilo(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

// NT = number of 8-sequence groups; SW = SwiGLU (gate + up rows per warp); EPI: kStore,
// kAccumulate, kSwiGlu (writes hi/lo planes).
template <int NT, bool SW>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const GemmArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int NL = SW ? 4 : 2;  // 16-byte weight loads per lane per k-step
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int RG = a.row_groups, KG = kThreads / 32 / RG;
  const int rg = warp % RG, kg = warp / RG;
  const int out_rows = SW ? a.rows / 2 : a.rows;
  const long half = SW ? a.rows / 2 : 0;
  const int r0 = (blockIdx.x * RG + rg) * 16;
  const int steps = a.k / 32;
  const int s0 = kg * steps / KG, s1 = (kg + 1) * steps / KG;
  const uint16_t* W = static_cast<const uint16_t*>(a.w);
  const size_t K = (size_t)a.k;

  // Rows of this lane (clamped for the tail; results of clamped rows are discarded).
  long rows[NL];
  rows[0] = min(r0 + g, out_rows - 1);
  rows[1] = min(r0 + g + 8, out_rows - 1);
  if constexpr (SW) {
    rows[2] = half + rows[0];
    rows[3] = half + rows[1];
  }
  uint4* ring = reinterpret_cast<uint4*>(smem);  // [stage][tid][NL]

  pdl_launch();
  // Weights do not depend on the previous kernel: start the ring before waiting on it.
  auto issue = [&](int s, int stage) {
    if (s < s1) {
      const size_t col = (size_t)s * 32 + 8 * t;
#pragma unroll
      for (int l = 0; l < NL; ++l) cp_async16(ring + ((size_t)stage * kThreads + tid) * NL + l, W + rows[l] * K + col);
    }
    cp_commit();
  };
#pragma unroll
  for (int i = 0; i < kStages - 1; ++i) issue(s0 + i, i);
  pdl_wait();

  float acc[NT][4];
  float accu[SW ? NT : 1][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[j][e] = 0.f;
      if constexpr (SW) accu[j][e] = 0.f;
    }
  const uint16_t* Xh = a.xh;
  const uint16_t* Xl = a.xl;
  const size_t ldx = (size_t)a.ldx;

  for (int s = s0; s < s1; ++s) {
    const int i = s - s0;
    issue(s + kStages - 1, (i + kStages - 1) % kStages);
    cp_wait<kStages - 1>();
    const uint4* mine = ring + ((size_t)(i % kStages) * kThreads + tid) * NL;
    uint4 w[NL];
#pragma unroll
    for (int l = 0; l < NL; ++l) w[l] = mine[l];
    const size_t col = (size_t)s * 32 + 8 * t;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const size_t xr = (size_t)(j * 8 + g) * ldx + col;
      const uint4 xh = *reinterpret_cast<const uint4*>(Xh + xr);
      const uint4 xl = *reinterpret_cast<const uint4*>(Xl + xr);
      mma16816(acc[j], w[0].x, w[1].x, w[0].y, w[1].y, xh.x, xh.y);
      mma16816(acc[j], w[0].z, w[1].z, w[0].w, w[1].w, xh.z, xh.w);
      mma16816(acc[j], w[0].x, w[1].x, w[0].y, w[1].y, xl.x, xl.y);
      mma16816(acc[j], w[0].z, w[1].z, w[0].w, w[1].w, xl.z, xl.w);
      if constexpr (SW) {
        mma16816(accu[j], w[2].x, w[3].x, w[2].y, w[3].y, xh.x, xh.y);
        mma16816(accu[j], w[2].z, w[3].z, w[2].w, w[3].w, xh.z, xh.w);
        mma16816(accu[j], w[2].x, w[3].x, w[2].y, w[3].y, xl.x, xl.y);
        mma16816(accu[j], w[2].z, w[3].z, w[2].w, w[3].w, xl.z, xl.w);
      }
    }
  }
  cp_wait<0>();
  __syncthreads();

  // Reduce the k-groups through shared memory: red[rg][kg][which][col][17] (row-minor, padded so
  // the epilogue reads consecutive rows without bank conflicts).
  constexpr int NC = NT * 8;
  constexpr int RP = 17;
  float* red = reinterpret_cast<float*>(smem);
  const int nwhich = SW ? 2 : 1;
  auto slot = [&](int rgi, int kgi, int which, int row, int col) -> float& {
    return red[(((size_t)rgi * KG + kgi) * nwhich + which) * (NC * RP) + col * RP + row];
  };
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int c = j * 8 + 2 * t;
    slot(rg, kg, 0, g, c) = acc[j][0];
    slot(rg, kg, 0, g, c + 1) = acc[j][1];
    slot(rg, kg, 0, g + 8, c) = acc[j][2];
    slot(rg, kg, 0, g + 8, c + 1) = acc[j][3];
    if constexpr (SW) {
      slot(rg, kg, 1, g, c) = accu[j][0];
      slot(rg, kg, 1, g, c + 1) = accu[j][1];
      slot(rg, kg, 1, g + 8, c) = accu[j][2];
      slot(rg, kg, 1, g + 8, c + 1) = accu[j][3];
    }
  }
  __syncthreads();
  const int B = a.batch;
  const int tile_rows = RG * 16;
  const int total = tile_rows * B;
  for (int e = tid; e < total; e += kThreads) {
    // consecutive threads take consecutive rows of one sequence: coalesced stores
    const int b = e / tile_rows;
    const int rr = e % tile_rows;
    const int rgi = rr / 16, row = rr % 16;
    const int orow = blockIdx.x * tile_rows + rr;
    if (orow >= out_rows) continue;
    float v = 0.f, u = 0.f;
    for (int kgi = 0; kgi < KG; ++kgi) {
      v += slot(rgi, kgi, 0, row, b);
      if constexpr (SW) u += slot(rgi, kgi, 1, row, b);
    }
    if constexpr (SW) {
      const float y = silu(v) * u;
      __half hi, lo;
      split_hilo(y, hi, lo);
      a.yh[(size_t)b * a.ldy + orow] = __half_as_ushort(hi);
      a.yl[(size_t)b * a.ldy + orow] = __half_as_ushort(lo);
    } else if (a.epi == kAccumulate) {
      a.y[(size_t)b * a.ldy + orow] += v;
    } else {
      a.y[(size_t)b * a.ldy + orow] = v;
    }
  }
}

template <int NT, bool SW>
cudaError_t launch_nt(const GemmArgs& a, cudaStream_t stream, bool pdl) {
  auto kernel = gemm_kernel<NT, SW>;
  constexpr int NL = SW ? 4 : 2;
  const int RG = a.row_groups, KG = kThreads / 32 / RG;
  const size_t ring = (size_t)kStages * kThreads * NL * 16;
  const size_t red = (size_t)RG * KG * (SW ? 2 : 1) * 17 * NT * 8 * 4;
  const size_t smem = ring > red ? ring : red;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int out_rows = SW ? a.rows / 2 : a.rows;
  const int grid = (out_rows + RG * 16 - 1) / (RG * 16);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
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

template <bool SW>
cudaError_t launch_sw(const GemmArgs& a, cudaStream_t stream, bool pdl) {
  const int nt = (a.batch + 7) / 8;
  switch (nt) {
    case 1: return launch_nt<1, SW>(a, stream, pdl);
    case 2: return launch_nt<2, SW>(a, stream, pdl);
    case 3: return launch_nt<3, SW>(a, stream, pdl);
    case 4: return launch_nt<4, SW>(a, stream, pdl);
  }
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------------------------------
// Prep: RMSNorm / embedding / gated GDN norm / copy, written as hi/lo planes for the GEMM.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float deq_any(const Mat& m, long row, int i) {
  if (m.kind == kF16) return h2f(__ldg((const uint16_t*)m.w + row * m.k + i));
  const uint32_t word = __ldg((const uint32_t*)m.w + row * (m.k / 8) + i / 8);
  const float q = nib_f(word, 4 * (i % 8));
  float scale, zp;
  if (m.kind == kQ4) q4_scale_zp((const uint32_t*)m.s, (const uint32_t*)m.z, row, m.k, i / 32, scale, zp);
  else q4g64_scale_zp((const uint16_t*)m.s, (const uint16_t*)m.z, row, m.k, i / 64, scale, zp);
  return (q - zp) * scale;
}

__global__ void __launch_bounds__(256) prep_kernel(const PrepArgs a) {
  __shared__ float red[8];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int K = a.k;
  pdl_launch();
  pdl_wait();
  uint16_t* xh = a.xh + (size_t)b * a.ldx;
  uint16_t* xl = a.xl + (size_t)b * a.ldx;
  if (a.conv_tail) {
    const uint32_t e = a.conv_ctl->count + (uint32_t)a.conv_n;
    for (int i = b * 256 + tid; i < 3 * kConvChannels; i += gridDim.x * 256) {
      const int j = i / kConvChannels, c = i % kConvChannels;
      a.conv_ring[(size_t)((e - 3u + (uint32_t)j) & 3u) * kConvChannels + c] = a.conv_tail[i];
    }
  }
  if (a.mode == kPrepGdnGate) {
    // K == 2048: 16 heads of 128 (warp w: heads 2w, 2w + 1)
    const int warp = tid >> 5, lane = tid & 31;
    for (int hh = 0; hh < 2; ++hh) {
      const int head = warp * 2 + hh;
      float v[4], ss = 0.f;
      for (int j = 0; j < 4; ++j) {
        v[j] = a.src[(size_t)b * a.lds + head * 128 + lane * 4 + j];
        ss += v[j] * v[j];
      }
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / 128.0f + a.eps);
      for (int j = 0; j < 4; ++j) {
        const int c = head * 128 + lane * 4 + j;
        const float z = a.zgate[(size_t)b * kGdnProj + 6144 + c];  // z block of proj
        __half hi, lo;
        split_hilo(v[j] * inv * silu(z) * a.norm_w[lane * 4 + j], hi, lo);
        xh[c] = __half_as_ushort(hi);
        xl[c] = __half_as_ushort(lo);
      }
    }
    return;
  }
  float ss = 0.f;
  const float* src = a.src + (size_t)b * a.lds;
  if (a.mode == kPrepEmbedNorm) {
    uint32_t token = a.ctl[b].token;
    if (token >= (uint32_t)a.embed.rows) token = (uint32_t)a.embed.rows - 1;
    float* h = a.h + (size_t)b * a.ldh;
    for (int i = tid; i < K; i += 256) {
      const float v = deq_any(a.embed, token, i);
      h[i] = v;
      ss += v * v;
    }
    if (tid == 0) a.ctl[b].count += 1;
    src = h;
    __syncthreads();
  } else if (a.mode == kPrepNorm) {
    for (int i = tid; i < K; i += 256) {
      const float v = src[i];
      ss += v * v;
    }
  }
  float inv = 1.f;
  if (a.mode != kPrepCopy) {
    const float tot = block_sum<256>(ss, red);
    inv = rsqrtf(tot / (float)K + a.eps);
    if (a.sumsq_out) {  // folded into the next GEMM: it applies 1 / rms
      inv = 1.f;
      for (int q = tid; q < a.sumsq_slots; q += 256) a.sumsq_out[q * kGemmMaxRows + b] = q == 0 ? tot : 0.f;
    }
  }
  for (int i = tid; i < K; i += 256) {
    const float v = a.mode == kPrepCopy ? src[i] : src[i] * inv * a.norm_w[i];
    __half hi, lo;
    split_hilo(v, hi, lo);
    xh[i] = __half_as_ushort(hi);
    xl[i] = __half_as_ushort(lo);
  }
}

// Greedy pick per sequence over logits[b][n]; grid (blocks, batch).
__global__ void __launch_bounds__(256) argmax_batched_kernel(const float* logits, uint32_t n, size_t ld,
                                                             SeqCtl* ctl, uint32_t* picks, float* part_val,
                                                             uint32_t* part_idx, uint32_t* ticket, int update) {
  __shared__ float bv[8];
  __shared__ uint32_t bi[8];
  __shared__ uint32_t is_last;
  const int b = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_launch();
  pdl_wait();
  const float* x = logits + (size_t)b * ld;
  float v = -INFINITY;
  uint32_t ix = 0xFFFFFFFFu;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float f = x[i];
    if (f > -INFINITY && (ix == 0xFFFFFFFFu || f > v)) {
      v = f;
      ix = i;
    }
  }
  auto better = [](float ov, uint32_t oi, float v0, uint32_t i0) {
    return oi != 0xFFFFFFFFu && (i0 == 0xFFFFFFFFu || ov > v0 || (ov == v0 && oi < i0));
  };
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
    bv[warp] = v;
    bi[warp] = ix;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    v = -INFINITY;
    ix = 0xFFFFFFFFu;
    for (int w = 0; w < 8; ++w)
      if (better(bv[w], bi[w], v, ix)) {
        v = bv[w];
        ix = bi[w];
      }
    part_val[(size_t)b * gridDim.x + blockIdx.x] = v;
    part_idx[(size_t)b * gridDim.x + blockIdx.x] = ix;
    __threadfence();
    is_last = (atomicAdd(ticket + b, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (is_last && warp == 0) {
    __threadfence();
    v = -INFINITY;
    ix = 0xFFFFFFFFu;
    for (int k = lane; k < (int)gridDim.x; k += 32) {
      const float ov = __ldcg(part_val + (size_t)b * gridDim.x + k);
      const uint32_t oi = __ldcg(part_idx + (size_t)b * gridDim.x + k);
      if (better(ov, oi, v, ix)) {
        v = ov;
        ix = oi;
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
      const uint32_t pick = (ix == 0xFFFFFFFFu) ? 0u : ix;
      if (picks) picks[b] = pick;
      if (update) {
        ctl[b].token = pick;
        ctl[b].pos += 1;
      }
      ticket[b] = 0u;
    }
  }
}

__global__ void hilo_to_f32_kernel(const uint16_t* hi, const uint16_t* lo, float* out, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = h2f(hi[i]) + h2f(lo[i]);
}

// splitmix64-style hash -> uniform in [-1, 1)
__device__ __forceinline__ float hash_uniform(uint64_t seed, uint64_t i) {
  uint64_t z = seed + 0x9E3779B97F4A7C15ull * (i + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 8388608.0f) - 1.0f;
}

__global__ void fill_kv_kernel(uint16_t* kv, const uint32_t* table, uint32_t len, uint64_t seed, uint32_t pool_pages) {
  // one CTA per (position, K/V, kv head); 256 threads = dims
  const uint32_t l = blockIdx.x;
  const int which = blockIdx.y >> 1, kvh = blockIdx.y & 1, d = threadIdx.x;
  if (l >= len) return;
  const uint32_t page = table[l / kPageTokens];
  if (page >= pool_pages) return;
  const uint64_t idx = (((uint64_t)l * 2 + which) * 2 + kvh) * 256 + d;
  kv[(size_t)page * kPageElems + ((size_t)(which * kKvHeads + kvh) * kPageTokens + l % kPageTokens) * kHeadDim + d] =
      __half_as_ushort(__float2half_rn(hash_uniform(seed, idx)));
}

__global__ void fill_f32_kernel(float* p, size_t n, uint64_t seed, float scale) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    p[i] = hash_uniform(seed, i) * scale;
}

cudaLaunchConfig_t cfg_of(dim3 grid, dim3 block, cudaStream_t stream, bool pdl, cudaLaunchAttribute* attr) {
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

// ------------------------------------------------------------------------------------------
// int4 matrices (the reference's block-32 layout or group 64) for the batched GEMMs: the matrix
// is decoded to f16 into a scratch the next GEMM reads (from L2 when the matrix fits). Each thread takes one u32 word, i.e. 8 values of one quantization block, with
// the per-token kernels' arithmetic (float(q) - zp) * scale, rounded to f16 once. The int4 words
// are immutable and load before the dependency wait; the stores overwrite what the previous GEMM
// of the stream read, so they come after it.
// ------------------------------------------------------------------------------------------
template <int KIND>
__global__ void __launch_bounds__(256) dequant_f16_kernel(const Mat m, uint16_t* out) {
  pdl_launch();
  const long words = (long)m.rows * (m.k / 8);
  const long stride = (long)gridDim.x * blockDim.x;
  bool waited = false;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < words; e += stride) {
    const long row = e / (m.k / 8);
    const int i = (int)(e % (m.k / 8)) * 8;
    const uint32_t word = __ldg(static_cast<const uint32_t*>(m.w) + e);
    float scale, zp;
    if (KIND == kQ4)
      q4_scale_zp(static_cast<const uint32_t*>(m.s), static_cast<const uint32_t*>(m.z), row, m.k, i / 32, scale, zp);
    else
      q4g64_scale_zp(static_cast<const uint16_t*>(m.s), static_cast<const uint16_t*>(m.z), row, m.k, i / 64, scale,
                     zp);
    uint32_t h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = __half_as_ushort(__float2half_rn((nib_f(word, 8 * j) - zp) * scale));
      const uint32_t hi = __half_as_ushort(__float2half_rn((nib_f(word, 8 * j + 4) - zp) * scale));
      h[j] = lo | (hi << 16);
    }
    if (!waited) {
      pdl_wait();
      waited = true;
    }
    *reinterpret_cast<uint4*>(out + e * 8) = make_uint4(h[0], h[1], h[2], h[3]);
  }
}

}  // namespace

int gemm_row_groups(int out_rows) {
  for (int rg = 8; rg > 1; rg /= 2)
    if ((out_rows + rg * 16 - 1) / (rg * 16) >= kNumSms) return rg;
  return 1;
}

const char* check_gemm(const GemmArgs& a) {
  if (!a.w || a.rows <= 0 || a.k <= 0) return "empty matrix";
  if (a.k % 32) return "batched GEMM needs k % 32 == 0";
  if (a.batch < 1 || a.batch > kGemmMaxRows) return "batch must be 1..64";
  if (a.impl == kGemmMmaSync && a.batch > 32) return "the mma.sync GEMM takes batch 1..32";
  if (a.epi == kSwiGlu && (a.rows % 2)) return "SwiGLU needs an even row count";
  if (!a.xh || !a.xl || a.ldx < a.k || a.ldx % 8) return "bad activation planes";
  if (a.epi == kSwiGlu ? (!a.yh || !a.yl) : !a.y) return "null output";
  if (a.row_groups != 1 && a.row_groups != 2 && a.row_groups != 4 && a.row_groups != 8) return "bad row groups";
  if (a.norm_w_out && (a.epi != kAccumulate || !a.out_xh || !a.out_xl || !a.sumsq_out || a.rows % 16))
    return "a folded-norm producer accumulates, writes planes and partials, rows % 16 == 0";
  if (a.sumsq_in && (a.sumsq_slots < 1 || a.norm_k < 1)) return "a folded-norm consumer needs its partials";
  if ((a.norm_w_out || a.sumsq_in) && (a.impl != kGemmTensorCore || !gemm_tc_available()))
    return "the folded RMSNorm needs the tensor-core GEMM";
  if (a.w_after_wait && (a.impl != kGemmTensorCore || !gemm_tc_available() || reinterpret_cast<uintptr_t>(a.w) % 16))
    return "weights written by the previous kernel need the tensor-core GEMM";
  if (a.wkind != kF16 && !gemm_int4_direct(a))
    return "int4 weights need the tensor-core GEMM, k % 64 == 0 (block-32: k % 256), scales and zero points";
  return nullptr;
}

cudaError_t launch_dequant_f16(const Mat& m, uint16_t* out, cudaStream_t stream, bool pdl) {
  if ((m.kind != kQ4 && m.kind != kQ4G64) || m.k % 64 || m.rows < 1) return cudaErrorInvalidValue;
  const long words = (long)m.rows * (m.k / 8);
  const int grid = (int)std::min<long>((words + 255) / 256, 8L * kNumSms);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cfg_of(dim3(grid), dim3(256), stream, pdl, attr);
  count_launch();
  return m.kind == kQ4 ? cudaLaunchKernelEx(&cfg, dequant_f16_kernel<kQ4>, m, out)
                       : cudaLaunchKernelEx(&cfg, dequant_f16_kernel<kQ4G64>, m, out);
}

cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream, bool pdl) {
  if (a.wkind != kF16) return gemm_int4_direct(a) ? launch_gemm_tc(a, stream, pdl) : cudaErrorInvalidValue;
  if (a.impl == kGemmTensorCore && gemm_tc_available() && reinterpret_cast<uintptr_t>(a.w) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(a.xh) % 16 == 0 && reinterpret_cast<uintptr_t>(a.xl) % 16 == 0)
    return launch_gemm_tc(a, stream, pdl);
  if (a.w_after_wait) return cudaErrorInvalidValue;  // the mma.sync kernel prefetches weights early
  return a.epi == kSwiGlu ? launch_sw<true>(a, stream, pdl) : launch_sw<false>(a, stream, pdl);
}

cudaError_t launch_prep(const PrepArgs& a, int batch, cudaStream_t stream, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cfg_of(dim3(batch), dim3(256), stream, pdl, attr);
  count_launch();
  return cudaLaunchKernelEx(&cfg, prep_kernel, a);
}

size_t argmax_batched_scratch_bytes(int batch) { return (size_t)batch * (64 * 8 + 4) + 256; }

cudaError_t launch_argmax_batched(const float* logits, uint32_t n, size_t ld, int batch, SeqCtl* ctl,
                                  uint32_t* picks, void* scratch, int update, cudaStream_t stream, bool pdl) {
  const int blocks = 64;
  uint8_t* p = static_cast<uint8_t*>(scratch);
  float* pv = reinterpret_cast<float*>(p);
  uint32_t* pi = reinterpret_cast<uint32_t*>(p + (size_t)batch * blocks * 4);
  uint32_t* ticket = reinterpret_cast<uint32_t*>(p + (size_t)batch * blocks * 8);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cfg_of(dim3(blocks, batch), dim3(256), stream, pdl, attr);
  count_launch();
  return cudaLaunchKernelEx(&cfg, argmax_batched_kernel, logits, n, ld, ctl, picks, pv, pi, ticket, update);
}

cudaError_t launch_fill_kv(uint16_t* kv, const uint32_t* table, uint32_t len, uint64_t seed, uint32_t pool_pages,
                           cudaStream_t stream) {
  if (len == 0) return cudaSuccess;
  count_launch();
  fill_kv_kernel<<<dim3(len, 4), 256, 0, stream>>>(kv, table, len, seed, pool_pages);
  return cudaGetLastError();
}

cudaError_t launch_hilo_to_f32(const uint16_t* hi, const uint16_t* lo, float* out, size_t n, cudaStream_t stream) {
  count_launch();
  hilo_to_f32_kernel<<<kNumSms * 2, 256, 0, stream>>>(hi, lo, out, n);
  return cudaGetLastError();
}

cudaError_t launch_fill_f32(float* p, size_t n, uint64_t seed, float scale, cudaStream_t stream) {
  count_launch();
  fill_f32_kernel<<<kNumSms * 4, 256, 0, stream>>>(p, n, seed, scale);
  return cudaGetLastError();
}

}  // namespace qne
