// Launchers of the Gated DeltaNet and attention kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace qne {

// conv: [batch][4][6144] ring; state: [batch][16][128][128]; counter[b * counter_stride] is the
// number of tokens processed including this one; out_raw: [batch][2048] before the gated norm.
cudaError_t launch_gdn_step(const float* proj, float* conv, const float* conv_w, float* state,
                            const float* params, const uint32_t* counter, int counter_stride,
                            float* out_raw, int batch, cudaStream_t stream, bool pdl);
// Gated per-head RMSNorm: out = raw * rsqrt(mean(raw^2) + 1e-6) * silu(z) * norm_w.
cudaError_t launch_gdn_gate(const float* raw, const float* proj, const float* norm_w, float* out,
                            int batch, cudaStream_t stream, bool pdl);

// Attention over paged f16 KV. pos[b * pos_stride] is the position of the token being decoded.
// Rows are independent sequences (batched decode) or, with page_table_stride 0 and kv_appended,
// consecutive tokens of one sequence whose keys and values were appended beforehand (prefill).
// rope: [4096][32] cos followed by [4096][32] sin (f32).
struct AttnArgs {
  const float* proj = nullptr;  // [batch][5120]
  const float* norms = nullptr; // [512]
  const float* rope = nullptr;  // [2][4096][32]
  uint16_t* kv = nullptr;       // page pool
  const uint32_t* page_table = nullptr;  // [batch][256]
  const uint32_t* pos = nullptr;
  int pos_stride = 1;
  uint32_t* flags = nullptr;    // optional: kFlagPosClamped is or-ed in when pos >= 4096
  int flags_stride = 1;
  float* out = nullptr;         // [batch][2048]
  // Optional: the merged output also as hi = f16(v), lo = f16(v - hi) planes [batch][out_ldx]
  // (the next tensor-core GEMM's activations), so no separate conversion launch is needed.
  uint16_t* out_xh = nullptr;
  uint16_t* out_xl = nullptr;
  int out_ldx = 0;
  int batch = 1;
  void* scratch = nullptr;
  int page_table_stride = kPagesPerSeq;  // 0: every row reads one sequence's page table (prefill)
  int kv_appended = 0;  // 1: every row's own K/V is already in the cache (prefill); no CTA appends
  int scratch_rows = 0;  // rows `scratch` is laid out for (0: batch); fixed when batch varies
  int impl = 0;          // 0: tensor-core kernel (mma.sync QK^T and PV), 1: CUDA-core kernel
};
size_t attention_scratch_bytes(int batch);
// split_tokens: context tokens per CTA, a multiple of 64. pool_pages bounds the page ids.
// rows_per_item 2 (prompt rows only: kv_appended, page_table_stride 0, tensor-core kernel): each CTA
// serves two consecutive query rows, so the cached keys and values are read half as often.
cudaError_t launch_attention(const AttnArgs& a, uint32_t pool_pages, int split_tokens,
                             cudaStream_t stream, bool pdl, int rows_per_item = 1);
cudaError_t launch_kv_gather(const uint16_t* kv, const uint32_t* page_table, uint32_t len,
                             uint16_t* out_k, uint16_t* out_v, cudaStream_t stream);
// Host: fills rope[2][4096][32] with cos/sin(pos * theta^(-2i/64)) computed in double precision.
void rope_table_host(float* table, double theta);
// Device copy of the table for `theta` on the current device, built on first use and kept.
const float* rope_table_device(double theta);
cudaError_t launch_bandwidth_probe(const void* data, size_t bytes, uint32_t* sink, cudaStream_t stream);
// Microseconds per launch of n noop kernels (mode 0 plain, 1 graph, 2 PDL, 3 graph of PDL).
double dispatch_cost(uint32_t n, int mode, float* y, cudaStream_t s);

}  // namespace qne
