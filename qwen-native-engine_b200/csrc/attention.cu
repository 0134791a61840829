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
// (context split, KV head, sequence) serves the 4 query heads of the KV head, stages its
// split's K and V rows in shared memory with cp.async, keeps an online softmax per head, and
// writes a partial (max, sum, 4 x 256 accumulator). The partials of each (sequence, KV head) are
// merged in one of two ways: with one sequence whose grid is resident at once, the last 8 splits
// each merge one 128-wide slice of the output over all splits once every split has arrived
// (attn_spread_merge); otherwise by tickets, the last split of each group of 8 merging the group
// and the last group merging the groups. The merger applies the output gate. The default work
// item (attn_tc.cuh)
// computes the scores and the PV product with mma.sync (q and the probabilities as hi + lo f16
// halves); the CUDA-core item (attn_dev.cuh, also used by the fused layer kernels) reduces each
// token's dot products across a warp.
// The CTA whose split holds `pos` normalizes, rotates and appends the current K/V (rounded to
// f16) and uses the rounded values for that position; no other CTA reads that slot.
// RoPE angles come from a host-built table (double precision), identical for every consumer.
#include <math.h>

#include <cmath>

#include "attn_dev.cuh"
#include "attn_tc.cuh"
#include "gdn.cuh"
#include "gemv.cuh"

namespace qne {
namespace {

using namespace dev;

template <class Item, class Shared>
__global__ void __launch_bounds__(256, 2) attention_kernel(const KernelArgs ka) {
  extern __shared__ __align__(128) uint8_t smem[];
  Shared& sh = *reinterpret_cast<Shared*>(smem);
  const int item = (blockIdx.z * kKvHeads + blockIdx.y) * ka.max_splits + blockIdx.x;
  Item it;
  pdl_launch();
  if (!ka.a.kv_appended) {
    // Decode: the positions, the page tables and every cached row a split stages were written
    // before this launch's graph or stream work began (the positions advance in the step's last
    // kernel, the page tables by host copies, and the current token's row is appended by this
    // kernel), so the split is staged under the previous kernel's tail.
    it.prefetch(ka, sh, item);
    pdl_wait();
  } else {
    pdl_wait();  // prompt rows: the previous kernel appended the chunk's keys and values
    it.prefetch(ka, sh, item);
  }
  it.run(ka, sh);
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
                             cudaStream_t stream, bool pdl, int rows_per_item) {
  // A split is whole 64-token sub-blocks, and the scratch holds at most kMaxSplits of them.
  if (split_tokens < kSub || split_tokens % kSub) return cudaErrorInvalidValue;
  if (rows_per_item != 1 && (rows_per_item != 2 || a.impl != 0 || !a.kv_appended || a.page_table_stride != 0))
    return cudaErrorInvalidValue;
  KernelArgs ka;
  ka.a = a;
  ka.split = split_tokens;
  ka.pool_pages = pool_pages;
  const int max_splits = (kMaxContext + split_tokens - 1) / split_tokens;
  ka.max_splits = max_splits;
  const bool tc = a.impl == 0;
  auto kernel = rows_per_item == 2 ? attention_kernel<AttnTcItemT<2>, AttnTcSharedT<8>>
                : tc               ? attention_kernel<AttnTcItem, AttnTcShared>
                                   : attention_kernel<AttnItem, AttnShared>;
  const size_t smem = rows_per_item == 2 ? sizeof(AttnTcSharedT<8>) : tc ? sizeof(AttnTcShared) : sizeof(AttnShared);
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  // Spread merge for one sequence, when every CTA of the grid can be resident at once: its
  // mergers wait for the other splits of their KV head.
  if (a.batch == 1 && rows_per_item == 1) {
    int dev = 0, sms = 0, occ = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, 256, smem) == cudaSuccess)
      ka.spread = (long)max_splits * kKvHeads <= (long)occ * sms ? 1 : 0;
    cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(max_splits, kKvHeads, (a.batch + rows_per_item - 1) / rows_per_item);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kernel, ka);
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
