// Kernels and launchers of the batched (independent sequences) decode path.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv.cuh"

namespace qne {

enum GemmImpl : int { kGemmTensorCore = 0, kGemmMmaSync = 1 };
// Activation rows one batched GEMM takes: 64 on the tensor-core kernel, 32 on the mma.sync one.
// Also the column stride of the folded-norm partials (GemmArgs::sumsq_out / sumsq_in).
constexpr int kGemmMaxRows = 64;

// Y[b][row] for b < batch: W [rows][k] f16 times the activation planes xh/xl [>= 8*ceil(batch/8)][ldx].
struct GemmArgs {
  const void* w = nullptr;
  // Weight kind: kF16 (w = f16 [rows][k]), or kQ4 / kQ4G64 (w = packed nibbles, ws / wz = scales
  // and zero points in the layouts of Mat; tensor-core kernel, see gemm_int4_direct).
  int wkind = kF16;
  const void* ws = nullptr;
  const void* wz = nullptr;
  int rows = 0;  // physical rows (SwiGLU: gate rows then up rows)
  int k = 0;
  int batch = 1;
  int epi = kStore;  // kStore, kAccumulate (f32 y), kSwiGlu (hi/lo planes yh/yl)
  int row_groups = 1;  // warps of a CTA along rows (1, 2, 4, 8); the rest split k
  const uint16_t* xh = nullptr;
  const uint16_t* xl = nullptr;
  int ldx = 0;
  float* y = nullptr;
  uint16_t* yh = nullptr;
  uint16_t* yl = nullptr;
  int ldy = 0;
  int x_rows = 0;           // rows allocated in xh/xl (0: 8 * ceil(batch / 8))
  int impl = kGemmTensorCore;
  // The previous kernel of the stream writes w (int4 weights dequantized into a scratch): the
  // weight tiles are then loaded only after the dependency wait (tensor-core kernel only).
  bool w_after_wait = false;
  uint32_t* err = nullptr;  // optional: receives kFlagTimeout if a bounded wait gives up
  // RMSNorm folded into the GEMMs on either side of it (tensor-core kernel only). Producer (an
  // accumulating GEMM that updates the residual h): also writes the planes out_xh/out_xl of
  // h * norm_w_out for the next GEMM and, per 16-row block of h and per column b,
  // sumsq_out[block * kGemmMaxRows + b] = sum of h^2. Consumer (the next GEMM, which reads those
  // planes): scales column b of its result by rsqrt(sum_q sumsq_in[q * kGemmMaxRows + b] / norm_k + eps) before
  // the epilogue (for SwiGLU, both halves).
  const float* norm_w_out = nullptr;
  uint16_t* out_xh = nullptr;
  uint16_t* out_xl = nullptr;
  int out_ldx = 0;
  float* sumsq_out = nullptr;
  const float* sumsq_in = nullptr;
  int sumsq_slots = 0;
  int norm_k = 0;
  float eps = 1e-6f;
};
int gemm_row_groups(int out_rows);
// int4 matrix m (kQ4 or kQ4G64, k % 64 == 0) -> out f16[rows][k], each value the per-token
// kernels' (float(q) - zp) * scale rounded to f16; loads before the dependency wait, stores after.
cudaError_t launch_dequant_f16(const Mat& m, uint16_t* out, cudaStream_t stream, bool pdl);
const char* check_gemm(const GemmArgs& a);
// impl kGemmTensorCore: tcgen05 + TMA (gemm_tc.cu); kGemmMmaSync: warp-level mma.sync (gemm.cu).
cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream, bool pdl);
// Whether the tensor-core GEMM takes these int4 weights directly (nibbles widened to f16 in
// shared memory). Otherwise callers decode the matrix into an f16 scratch (launch_dequant_f16).
bool gemm_int4_direct(const GemmArgs& a);
bool gemm_tc_available();
cudaError_t launch_gemm_tc(const GemmArgs& a, cudaStream_t stream, bool pdl);

enum PrepMode : int { kPrepCopy = 0, kPrepNorm = 1, kPrepEmbedNorm = 2, kPrepGdnGate = 3 };
struct PrepArgs {
  int mode = kPrepCopy;
  int k = 0;
  const float* src = nullptr;  // [batch][lds] (copy / norm / gdn gate raw output)
  int lds = 0;
  const float* norm_w = nullptr;
  float eps = 1e-6f;
  const float* zgate = nullptr;  // gdn gate: proj [batch][8224] (z read from column 6144)
  Mat embed;                     // embed: matrix, ctl (token, count), h out [batch][ldh]
  SeqCtl* ctl = nullptr;
  float* h = nullptr;
  int ldh = 0;
  uint16_t* xh = nullptr;
  uint16_t* xl = nullptr;
  int ldx = 0;
  // Optional (chunked prefill): after a GDN scan of conv_n tokens, commit its last three conv
  // inputs conv_tail[3][6144] to the ring conv_ring[4][6144] at slots (count + conv_n - 3 + j) % 4.
  const float* conv_tail = nullptr;
  float* conv_ring = nullptr;
  const SeqCtl* conv_ctl = nullptr;
  int conv_n = 0;
  // Optional (norm and embedding modes): RMSNorm folded into the next GEMM (GemmArgs::sumsq_in):
  // the planes hold x * norm_w, and sumsq_out[q * kGemmMaxRows + b] receives the row's sum of squares for
  // q = 0 and zero for 0 < q < sumsq_slots.
  float* sumsq_out = nullptr;
  int sumsq_slots = 0;
};
cudaError_t launch_prep(const PrepArgs& a, int batch, cudaStream_t stream, bool pdl);

size_t argmax_batched_scratch_bytes(int batch);
cudaError_t launch_argmax_batched(const float* logits, uint32_t n, size_t ld, int batch, SeqCtl* ctl,
                                  uint32_t* picks, void* scratch, int update, cudaStream_t stream, bool pdl);
cudaError_t launch_fill_kv(uint16_t* kv, const uint32_t* table, uint32_t len, uint64_t seed, uint32_t pool_pages,
                           cudaStream_t stream);
cudaError_t launch_fill_f32(float* p, size_t n, uint64_t seed, float scale, cudaStream_t stream);
cudaError_t launch_hilo_to_f32(const uint16_t* hi, const uint16_t* lo, float* out, size_t n, cudaStream_t stream);

}  // namespace qne
