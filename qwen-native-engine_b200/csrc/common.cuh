// Shared constants and device helpers of the sm_100a decode kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qne {

// Architecture constants of the Qwen3.5 hybrid decoder (kernels/src/lib.rs:21-30).
constexpr int kMaxContext = 4096;
constexpr int kPageTokens = 16;
constexpr int kPagesPerSeq = kMaxContext / kPageTokens;  // 256
constexpr int kGdnHeads = 16;
constexpr int kGdnDim = 128;
constexpr int kGdnProj = 8224;      // q, k, v, z (4 x 2048) + a, b (2 x 16)
constexpr int kConvChannels = 6144; // q, k, v
constexpr int kConvSlots = 4;       // ring of the last 4 conv inputs
constexpr int kAttnHeads = 8;
constexpr int kKvHeads = 2;
constexpr int kHeadDim = 256;
constexpr int kAttnProj = 5120;     // q, gate (2 x 2048) + k, v (2 x 512)
constexpr int kRopeHalf = 32;       // rotate-half pairs (i, i + 32), i < 32
constexpr int kMixerOut = 2048;
constexpr int kVocab = 248320;     // VOCAB, kernels/src/lib.rs (the two Qwen3.5 sizes)
// One KV page: [K, V][kv head][token][dim] f16.
constexpr int kPageElems = 2 * kKvHeads * kPageTokens * kHeadDim;  // 16384 halves = 32 KB
constexpr int kNumSms = 148;
constexpr int kMaxGrid = 512;  // largest 1-D grid of the B=1 kernels (per-CTA reduction slots)

enum WeightKind : int { kF16 = 0, kQ4 = 1, kQ4G64 = 2 };
enum Epi : int { kStore = 0, kAccumulate = 1, kSwiGlu = 2, kArgmax = 3 };
enum Pro : int { kProCopy = 0, kProRmsNorm = 1, kProGdnGate = 2, kProEmbedNorm = 3 };

// Per-sequence control words: token id, position, tokens processed (conv ring counter), flags.
struct SeqCtl {
  uint32_t token;
  uint32_t pos;
  uint32_t count;
  uint32_t flags;
};
constexpr uint32_t kFlagPosClamped = 1u;  // a position at or past the context limit was clamped
constexpr uint32_t kFlagTimeout = 2u;     // a bounded device wait gave up

// ------------------------------------------------------------------------------------------
// Programmatic dependent launch: every kernel issues launch_dependents early (so the next
// kernel's CTAs can start their weight prefetch) and waits before touching data produced by
// the kernel before it.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Asynchronous bulk prefetch of [p, p + bytes) into L2 by the TMA unit (no registers, no
// shared memory). p must be 16-byte aligned and bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// 16-byte streaming load of read-only data (weights): bypasses L1.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ float2 h2f2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}
__device__ __forceinline__ float h2f(uint16_t v) {
  return __half2float(__ushort_as_half(v));
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x == NT (multiple of 32); `red` holds NT / 32 floats.
// Every thread receives the total.
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t += red[i];
  return t;
}

// ------------------------------------------------------------------------------------------
// Weight unpacking. A "chunk" is one 16-byte load of a row: 8 f16 values, or 32 int4 values.
// The int4 formats store values low nibble first, eight per u32 (kernels/src/lib.rs:490).
// ------------------------------------------------------------------------------------------

// Exact float of a nibble 0..15 via the 2^23 exponent trick (no int->float conversion).
__device__ __forceinline__ float nib_f(uint32_t w, int shift) {
  return __uint_as_float(0x4B000000u | ((w >> shift) & 15u)) - 8388608.0f;
}

// Scale and zero point of the 32-value block `blk` of `row` in the MatMulNBits block-32 layout
// (kernels/src/lib.rs:491-493): scale = f16 half (blk & 1) of s[row*k/64 + blk/2],
// zp = nibble (blk % 8) of z[row*k/256 + blk/8].
__device__ __forceinline__ void q4_scale_zp(const uint32_t* s, const uint32_t* z, long row, int k,
                                            int blk, float& scale, float& zp) {
  const uint32_t sw = __ldg(s + row * (k / 64) + blk / 2);
  scale = h2f((uint16_t)((blk & 1) ? (sw >> 16) : (sw & 0xFFFFu)));
  const uint32_t zw = __ldg(z + row * (k / 256) + blk / 8);
  zp = (float)((zw >> (4 * (blk % 8))) & 15u);
}

// Scale and zero point of the 64-value group `grp` of `row` in the group-64 layout.
__device__ __forceinline__ void q4g64_scale_zp(const uint16_t* s, const uint16_t* z, long row,
                                               int k, int grp, float& scale, float& zp) {
  scale = h2f(__ldg(s + row * (k / 64) + grp));
  zp = h2f(__ldg(z + row * (k / 64) + grp));
}

}  // namespace qne
