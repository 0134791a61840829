// Batched prompt processing: the n <= 64 tokens of a chunk go through every layer together
// (Model::prefill_chunk, kernels/src/model.rs:349-372; its per-chunk dispatch list is built at
// kernels/src/model.rs:222-259 from the kernels of kernels/src/batch.rs). First the embedding
// prep, then per layer (the RMSNorms are folded into the GEMMs on either side of them):
//   GEMM mixer_in (n rows) |
//   GDN layers: gdn_scan (the recurrence walked token by token, state in registers) |
//     prep (gated RMSNorm)
//   attention layers: kv_append (RMSNorm + RoPE of the n keys; K and V rounded to f16 into the
//     sequence's pages) | attention (one row per token, causal over the cache) | prep (copy)
//   | GEMM mixer_out (+= h) | GEMM gate_up (SwiGLU) | GEMM down (+= h);
// then chunk_finish advances the sequence's control words by n and leaves the last row's hidden
// state where the B = 1 LM head reads it. The weights stream once per chunk instead of once per
// token, so a chunk costs about what one batched decode step of as many sequences costs.
//
// Numerics follow the per-token kernels: the GDN scan and the key normalization repeat the
// decode kernels' arithmetic per token; the GEMMs accumulate in f32 from f16 weights and hi/lo
// f16 activations (the batched decode GEMM). int4 decoder matrices feed the int4 tcgen05 GEMM,
// which widens the nibbles to f16 in shared memory (one rounding of each dequantized weight, the
// value the per-token kernels use); shapes it does not take are decoded to f16 by one more launch
// before the GEMM.
#include <algorithm>
#include <string>

#include "../../include/qne.h"
#include "attn_dev.cuh"
#include "batch.cuh"
#include "gdn.cuh"
#include "model.hpp"
#include "prefill.hpp"

namespace qne {
namespace {

using namespace dev;

// ------------------------------------------------------------------------------------------
// Gated DeltaNet over the chunk (batch::gdn, kernels/src/batch.rs:168-255; per-token math
// kernels/src/shaders.rs:445-520). One CTA of 512 threads per (16-column slice, head). Only
// the state recurrence is sequential, so the kernel runs in two phases:
//  1. everything that does not depend on the state, for all n tokens at once (every input of the
//     chunk is requested up front, so the token loops wait on no memory): causal conv + SiLU of
//     the head's q channels (threads 0..127), k channels (128..255) and this slice's v channels
//     (256..271), windows in registers seeded from the conv ring; decay g and write strength
//     beta (272..303); then the L2 normalization of q (times 1/sqrt(128)) and k, and k . q;
//  2. warp w owns value column w of the 128 x 16 state slice (4 rows per lane, in registers for
//     the whole chunk) and walks the tokens with no block barrier: S^T k and S^T q by warp
//     shuffles, the rank-1 update, the output.
// The conv ring holds input j at slot j % 4. All 8 CTAs of a head read the head's q/k ring
// channels, so none of them may overwrite a slot: each writes its channels' last three inputs to
// `tail` instead, and the gated-norm prep kernel that follows commits them to the ring.
// ------------------------------------------------------------------------------------------
struct ScanArgs {
  const float* proj;    // [n][8224] mixer_in rows of the chunk
  float* conv;          // [4][6144] conv input ring of the sequence
  const float* conv_w;  // [6144][4]
  float* state;         // [16][128][128] recurrent state
  const float* params;  // dt_bias[16], A[16], norm weight[128]
  const SeqCtl* ctl;    // ctl->count: tokens processed before the chunk
  int n;
  float* out;           // [n][2048] raw output (before the gated RMSNorm)
  float* tail;          // [3][6144]: the chunk's last three conv inputs, oldest first
};

constexpr int kScanRows = 64;  // tokens per chunk
constexpr int kScanThreads = 512;

struct ScanShared {
  __align__(16) float qk[kScanRows][2 * kGdnDim];  // per token: q channels 0..127, k channels 128..255
  float red[kScanRows][8];                          // per token: per-warp sums of squares
  float vv[kScanRows][kSlice];                      // per token: conv + SiLU of this slice's v channels
  float g[kScanRows], beta[kScanRows], kq[kScanRows];
};
static_assert(kScanRows == PrefillRunner::kRows, "the scan holds one chunk's tokens");
static_assert(kScanRows <= kGemmMaxRows, "a chunk's rows go through one batched GEMM");

__global__ void __launch_bounds__(kScanThreads, 1) gdn_scan_kernel(const __grid_constant__ ScanArgs a) {
  extern __shared__ __align__(16) uint8_t scan_smem[];  // one ScanShared (about 71 KB: dynamic)
  ScanShared& sh = *reinterpret_cast<ScanShared*>(scan_smem);
  const int h = blockIdx.y, t0 = blockIdx.x * kSlice;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = a.n;
  // phase-1 roles: a q/k channel (tid < 256), a v channel (256 .. 271)
  const int iq = tid & (kGdnDim - 1);
  const bool is_qk = tid < 2 * kGdnDim, is_v = tid >= 2 * kGdnDim && tid < 2 * kGdnDim + kSlice;
  const int ch = is_qk ? (tid < kGdnDim ? 0 : 2048) + h * kGdnDim + iq : 4096 + h * kGdnDim + t0 + (tid & 15);
  pdl_launch();
  pdl_wait();
  const uint32_t cnt0 = a.ctl->count;
  const int r0 = (int)((cnt0 - 3u) & 3u), r1 = (int)((cnt0 - 2u) & 3u), r2 = (int)((cnt0 - 1u) & 3u);
  const bool conv_thread = is_qk || is_v;
  float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
  float x0 = 0.f, x1 = 0.f, x2 = 0.f;
  float xs[kScanRows];
  if (conv_thread) {
    w = *reinterpret_cast<const float4*>(a.conv_w + (size_t)ch * 4);
    x0 = a.conv[r0 * kConvChannels + ch];
    x1 = a.conv[r1 * kConvChannels + ch];
    x2 = a.conv[r2 * kConvChannels + ch];
#pragma unroll
    for (int i = 0; i < kScanRows; ++i) xs[i] = i < n ? a.proj[(size_t)i * kGdnProj + ch] : 0.f;
  }
  // phase-2 role: value column `warp`, state rows 4 lane .. 4 lane + 3
  float* S = a.state + (size_t)h * kGdnDim * kGdnDim + (size_t)(lane * 4) * kGdnDim + t0 + warp;
  float sv[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) sv[r] = S[(size_t)r * kGdnDim];

  // ---- phase 1 ----
  const int gt = tid - (2 * kGdnDim + kSlice);
  if (gt >= 0 && gt < n) {
    const float* pr = a.proj + (size_t)gt * kGdnProj;
    sh.g[gt] = expf(a.params[16 + h] * logf(1.0f + expf(pr[8192 + h] + a.params[h])));
    sh.beta[gt] = 1.0f / (1.0f + expf(-pr[8208 + h]));
  }
  if (conv_thread) {
#pragma unroll
    for (int i = 0; i < kScanRows; ++i) {
      if (i < n) {
        const float y = x0 * w.x + x1 * w.y + x2 * w.z + xs[i] * w.w;
        x0 = x1;
        x1 = x2;
        x2 = xs[i];
        const float val = silu(y);
        if (is_qk) {
          sh.qk[i][tid] = val;
          const float ss = warp_sum(val * val);
          if (lane == 0) sh.red[i][warp] = ss;
        } else {
          sh.vv[i][tid & 15] = val;
        }
      }
    }
  }
  __syncthreads();
  for (int e = tid; e < n * 2 * kGdnDim; e += kScanThreads) {
    const int i = e >> 8, c = e & 255;
    const float* r = sh.red[i];
    sh.qk[i][c] *= c < kGdnDim ? rsqrtf(r[0] + r[1] + r[2] + r[3] + 1e-6f) * 0.08838834764f
                               : rsqrtf(r[4] + r[5] + r[6] + r[7] + 1e-6f);
  }
  __syncthreads();
  for (int i = warp; i < n; i += kScanThreads / 32) {
    float p = 0.f;
#pragma unroll
    for (int c = lane; c < kGdnDim; c += 32) p = fmaf(sh.qk[i][kGdnDim + c], sh.qk[i][c], p);
    p = warp_sum(p);
    if (lane == 0) sh.kq[i] = p;
  }
  __syncthreads();

  // ---- phase 2: the recurrence, one value column per warp, no block barrier ----
#pragma unroll 1
  for (int i = 0; i < n; ++i) {
    const float4 q4 = *reinterpret_cast<const float4*>(&sh.qk[i][lane * 4]);
    const float4 k4 = *reinterpret_cast<const float4*>(&sh.qk[i][kGdnDim + lane * 4]);
    float sk = sv[0] * k4.x, sq = sv[0] * q4.x;
    sk = fmaf(sv[1], k4.y, sk);
    sq = fmaf(sv[1], q4.y, sq);
    sk = fmaf(sv[2], k4.z, sk);
    sq = fmaf(sv[2], q4.z, sq);
    sk = fmaf(sv[3], k4.w, sk);
    sq = fmaf(sv[3], q4.w, sq);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sk += __shfl_xor_sync(0xffffffffu, sk, o);
      sq += __shfl_xor_sync(0xffffffffu, sq, o);
    }
    const float g = sh.g[i];
    const float dv = sh.beta[i] * (sh.vv[i][warp] - g * sk);
    sv[0] = g * sv[0] + dv * k4.x;
    sv[1] = g * sv[1] + dv * k4.y;
    sv[2] = g * sv[2] + dv * k4.z;
    sv[3] = g * sv[3] + dv * k4.w;
    if (lane == 0) a.out[(size_t)i * kMixerOut + h * kGdnDim + t0 + warp] = g * sq + dv * sh.kq[i];
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) S[(size_t)r * kGdnDim] = sv[r];
  // this slice's share of the head's q and k channels, and its own v channels
  if ((is_qk && iq >= t0 && iq < t0 + kSlice) || is_v) {
    a.tail[ch] = x0;
    a.tail[kConvChannels + ch] = x1;
    a.tail[2 * kConvChannels + ch] = x2;
  }
}

// ------------------------------------------------------------------------------------------
// Keys and values of the chunk into the cache (batch::kv_prep, kernels/src/batch.rs:290-314):
// one CTA per (token, KV head); RMSNorm with k_norm, rotate-half RoPE on dims 0..63 at the
// token's position, both rounded to f16 into the sequence's page. The arithmetic is the
// attention decode kernel's append, so a chunk writes the same cache rows as per-token steps.
// ------------------------------------------------------------------------------------------
struct AppendArgs {
  const float* proj;          // [n][5120]
  const float* norms;         // q_norm[256], k_norm[256]
  const float* rope;          // [2][4096][32]
  uint16_t* kv;               // page pool
  const uint32_t* page_table; // [256] pages of the sequence
  uint32_t pool_pages;
  const SeqCtl* rows;         // rows[i].pos: position of chunk token i
};

__global__ void __launch_bounds__(256) kv_append_kernel(const __grid_constant__ AppendArgs a) {
  __shared__ float red[8];
  __shared__ float ks[kHeadDim];
  const int i = blockIdx.x, kvh = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  pdl_launch();
  pdl_wait();
  uint32_t pos = a.rows[i].pos;
  if (pos >= (uint32_t)kMaxContext) pos = kMaxContext - 1;  // the host rejects such chunks
  const float* pr = a.proj + (size_t)i * kAttnProj;
  const float xk = pr[4096 + kvh * kHeadDim + t];
  const float ssk = warp_sum(xk * xk);
  if (lane == 0) red[warp] = ssk;
  __syncthreads();
  float sum = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) sum += red[w];
  const float kn = xk * rsqrtf(sum / (float)kHeadDim + 1e-6f) * a.norms[kHeadDim + t];
  ks[t] = kn;
  __syncthreads();
  float kr = kn;
  if (t < 2 * kRopeHalf) {
    const int j = t & (kRopeHalf - 1);
    const float c = a.rope[(size_t)pos * kRopeHalf + j];
    const float sn = a.rope[(size_t)kMaxContext * kRopeHalf + (size_t)pos * kRopeHalf + j];
    kr = (t < kRopeHalf) ? ks[t] * c - ks[t + kRopeHalf] * sn : ks[t] * c + ks[t - kRopeHalf] * sn;
  }
  const uint32_t page = a.page_table[pos / kPageTokens];
  if (page < a.pool_pages) {
    uint16_t* kdst = const_cast<uint16_t*>(kv_row(a.kv, page, 0, kvh, pos % kPageTokens));
    uint16_t* vdst = const_cast<uint16_t*>(kv_row(a.kv, page, 1, kvh, pos % kPageTokens));
    kdst[t] = __half_as_ushort(__float2half_rn(kr));
    vdst[t] = __half_as_ushort(__float2half_rn(pr[4608 + kvh * kHeadDim + t]));
  }
}

// Advances the sequence past the chunk and hands the last row's hidden state to the B = 1 LM
// head: control words (last token, its position, count + n), h_out = h_rows[n - 1].
__global__ void __launch_bounds__(256) chunk_finish_kernel(SeqCtl* ctl, const SeqCtl* rows, int n,
                                                           const float* h_rows, int hidden, float* h_out) {
  pdl_launch();
  pdl_wait();
  const float* src = h_rows + (size_t)(n - 1) * hidden;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) h_out[i] = src[i];
  if (threadIdx.x == 0) {
    ctl->token = rows[n - 1].token;
    ctl->pos = rows[n - 1].pos;
    ctl->count += (uint32_t)n;
  }
}

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, cudaStream_t stream, bool pdl, cudaLaunchAttribute* attr) {
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

}  // namespace

bool PrefillRunner::supported(const Model& m) {
  for (const LayerWeights& L : m.layers)
    for (const Mat* w : {&L.in, &L.out, &L.gate_up, &L.down})
      if ((w->kind != kF16 && w->kind != kQ4 && w->kind != kQ4G64) || w->k % 64) return false;
  return !m.layers.empty();
}

PrefillRunner::PrefillRunner(Model* model, Runner* single) : m(model), r(single) {
  const Config& c = m->cfg;
  ldx0 = c.hidden > kMixerOut ? c.hidden : kMixerOut;
  h = static_cast<float*>(m->alloc((size_t)kRows * c.hidden * 4));
  proj = static_cast<float*>(m->alloc((size_t)kRows * kGdnProj * 4));
  raw = static_cast<float*>(m->alloc((size_t)kRows * kMixerOut * 4));
  x0h = static_cast<uint16_t*>(m->alloc((size_t)kRows * ldx0 * 2));
  x0l = static_cast<uint16_t*>(m->alloc((size_t)kRows * ldx0 * 2));
  x1h = static_cast<uint16_t*>(m->alloc((size_t)kRows * c.inter * 2));
  x1l = static_cast<uint16_t*>(m->alloc((size_t)kRows * c.inter * 2));
  for (auto* p : {x0h, x0l}) cuda_check(cudaMemset(p, 0, (size_t)kRows * ldx0 * 2), "memset");
  for (auto* p : {x1h, x1l}) cuda_check(cudaMemset(p, 0, (size_t)kRows * c.inter * 2), "memset");
  xnh = static_cast<uint16_t*>(m->alloc((size_t)kRows * c.hidden * 2));
  xnl = static_cast<uint16_t*>(m->alloc((size_t)kRows * c.hidden * 2));
  for (auto* p : {xnh, xnl}) cuda_check(cudaMemset(p, 0, (size_t)kRows * c.hidden * 2), "memset");
  sumsq = static_cast<float*>(m->alloc((size_t)(c.hidden / 16) * kGemmMaxRows * 4));
  cuda_check(cudaMemset(sumsq, 0, (size_t)(c.hidden / 16) * kGemmMaxRows * 4), "memset");
  rows = static_cast<SeqCtl*>(m->alloc((size_t)kRows * sizeof(SeqCtl)));
  cuda_check(cudaMemset(rows, 0, (size_t)kRows * sizeof(SeqCtl)), "memset");
  conv_tail = static_cast<float*>(m->alloc((size_t)3 * kConvChannels * 4));
  attn_scratch = m->alloc(attention_scratch_bytes(kRows));
  cuda_check(cudaMemset(attn_scratch, 0, attention_scratch_bytes(kRows)), "memset");
  cuda_check(cudaMallocHost(&pinned, (size_t)kMaxContext * sizeof(SeqCtl)), "cudaMallocHost");
  size_t deq_elems = 0;  // the largest int4 decoder matrix, decoded to f16 before its GEMM
  for (const LayerWeights& L : m->layers)
    for (const Mat* w : {&L.in, &L.out, &L.gate_up, &L.down})
      if (w->kind != kF16) deq_elems = std::max(deq_elems, (size_t)w->rows * w->k);
  if (deq_elems) wdeq = static_cast<uint16_t*>(m->alloc(deq_elems * 2));
  cuda_check(cudaFuncSetAttribute(gdn_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sizeof(ScanShared)),
             "gdn scan shared memory");
}

PrefillRunner::~PrefillRunner() {
  for (auto& g : graphs)
    if (g.second) cudaGraphExecDestroy(g.second);
  if (pinned) cudaFreeHost(pinned);
}

void PrefillRunner::record(int n, cudaStream_t s) {
  const Model& M = *m;
  const Config& c = M.cfg;
  size_t cnt = 0;
  auto prep = [&](PrepArgs p) {
    p.xh = x0h;
    p.xl = x0l;
    p.ldx = ldx0;
    cuda_check(launch_prep(p, n, s, true), "prefill prep");
    ++cnt;
  };
  // RMSNorm folded into the GEMMs: the GEMM that updates h writes the planes of h * (next norm
  // weight) and partial sums of h^2; the GEMM that reads those planes applies 1 / rms.
  const int slots = c.hidden / 16;
  auto gemm = [&](const Mat& w, const uint16_t* xh, const uint16_t* xl, int ldx, int epi, float* y, uint16_t* yh,
                  uint16_t* yl, int ldy, const float* norm_out, bool norm_in) {
    GemmArgs g;
    g.w = w.w;
    g.rows = w.rows;
    g.k = w.k;
    g.batch = n;
    g.epi = epi;
    if (w.kind != kF16) {
      // int4: widened to f16 inside the GEMM, or (the many-wave LM head) decoded into the f16
      // scratch first
      g.wkind = w.kind;
      g.ws = w.s;
      g.wz = w.z;
      if (!gemm_int4_direct(g)) {
        cuda_check(launch_dequant_f16(w, wdeq, s, true), "prefill dequant launch");
        ++cnt;
        g.wkind = kF16;
        g.w = wdeq;
        g.w_after_wait = true;
      }
    }
    g.row_groups = gemm_row_groups(epi == kSwiGlu ? w.rows / 2 : w.rows);
    g.xh = xh;
    g.xl = xl;
    g.ldx = ldx;
    g.y = y;
    g.yh = yh;
    g.yl = yl;
    g.ldy = ldy;
    if (norm_out) {
      g.norm_w_out = norm_out;
      g.out_xh = xnh;
      g.out_xl = xnl;
      g.out_ldx = c.hidden;
      g.sumsq_out = sumsq;
    }
    if (norm_in) {
      g.sumsq_in = sumsq;
      g.sumsq_slots = slots;
      g.norm_k = c.hidden;
    }
    if (const char* why = check_gemm(g)) throw QneError(kEInval, why);
    cuda_check(launch_gemm(g, s, true), "prefill gemm");
    ++cnt;
  };
  cudaLaunchAttribute attr[1];
  {
    PrepArgs p;  // embedding rows (reads rows[b].token) -> h, planes of h * input_norm[0], sums
    p.mode = kPrepEmbedNorm;
    p.k = c.hidden;
    p.norm_w = M.layers[0].input_norm;
    p.embed = M.embed;
    p.ctl = rows;
    p.h = h;
    p.ldh = c.hidden;
    p.sumsq_out = sumsq;
    p.sumsq_slots = slots;
    p.xh = xnh;
    p.xl = xnl;
    p.ldx = c.hidden;
    cuda_check(launch_prep(p, n, s, true), "prefill prep");
    ++cnt;
  }
  for (int i = 0; i < c.layers; ++i) {
    const LayerWeights& L = M.layers[i];
    gemm(L.in, xnh, xnl, c.hidden, kStore, proj, nullptr, nullptr, L.in.rows, nullptr, true);
    PrepArgs q;
    q.k = kMixerOut;
    q.src = raw;
    q.lds = kMixerOut;
    if (L.attention) {
      const AppendArgs ap{proj, L.attn_norms, M.rope, r->st.kv[i], r->st.page_table, r->st.pool_pages, rows};
      cudaLaunchConfig_t cfg = make_cfg(dim3(n, kKvHeads), dim3(256), s, true, attr);
      count_launch();
      cuda_check(cudaLaunchKernelEx(&cfg, kv_append_kernel, ap), "kv append launch");
      ++cnt;
      AttnArgs at;
      at.proj = proj;
      at.norms = L.attn_norms;
      at.rope = M.rope;
      at.kv = r->st.kv[i];
      at.page_table = r->st.page_table;
      at.page_table_stride = 0;
      at.kv_appended = 1;
      at.pos = &rows->pos;
      at.pos_stride = 4;
      at.flags = &r->st.ctl->flags;
      at.flags_stride = 0;
      at.out = raw;
      at.out_xh = x0h;  // the out-projection's activation planes, written by the merge itself
      at.out_xl = x0l;
      at.out_ldx = ldx0;
      at.batch = n;
      at.scratch = attn_scratch;
      at.scratch_rows = kRows;  // one layout for every chunk size, so tickets stay where they were reset
      cuda_check(launch_attention(at, r->st.pool_pages, n >= 8 ? 512 : 64, s, true, n >= 2 ? 2 : 1),
                 "prefill attention launch");
      ++cnt;
    } else {
      const ScanArgs sa{proj, r->st.conv[i], L.conv_w, r->st.rec[i], L.gdn_params, r->st.ctl, n, raw, conv_tail};
      cudaLaunchConfig_t cfg = make_cfg(dim3(kSlices, kGdnHeads), dim3(kScanThreads), s, true, attr);
      cfg.dynamicSmemBytes = sizeof(ScanShared);
      count_launch();
      cuda_check(cudaLaunchKernelEx(&cfg, gdn_scan_kernel, sa), "gdn scan launch");
      ++cnt;
      q.mode = kPrepGdnGate;
      q.zgate = proj;
      q.norm_w = L.gdn_params + 32;
      q.conv_tail = conv_tail;  // the prep also commits the scan's conv inputs to the ring
      q.conv_ring = r->st.conv[i];
      q.conv_ctl = r->st.ctl;
      q.conv_n = n;
    }
    if (!L.attention) prep(q);
    gemm(L.out, x0h, x0l, ldx0, kAccumulate, h, nullptr, nullptr, c.hidden, L.post_norm, false);
    gemm(L.gate_up, xnh, xnl, c.hidden, kSwiGlu, nullptr, x1h, x1l, c.inter, nullptr, true);
    // the next layer's input norm (after the last layer the B = 1 LM head normalizes h itself)
    const float* next_norm = i + 1 < c.layers ? M.layers[i + 1].input_norm : nullptr;
    gemm(L.down, x1h, x1l, c.inter, kAccumulate, h, nullptr, nullptr, c.hidden, next_norm, false);
  }
  cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(256), s, true, attr);
  count_launch();
  cuda_check(cudaLaunchKernelEx(&cfg, chunk_finish_kernel, r->st.ctl, (const SeqCtl*)rows, n, (const float*)h,
                                c.hidden, r->h),
             "chunk finish launch");
  ++cnt;
  launches[n] = cnt;
}

cudaGraphExec_t PrefillRunner::graph_for(int n) {
  auto it = graphs.find(n);
  if (it != graphs.end()) return it->second;
  cudaStream_t cs;
  cuda_check(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "cudaStreamCreate");
  cuda_check(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "begin capture");
  try {
    record(n, cs);
  } catch (...) {
    cudaGraph_t g = nullptr;
    cudaStreamEndCapture(cs, &g);
    if (g) cudaGraphDestroy(g);
    cudaStreamDestroy(cs);
    throw;
  }
  cudaGraph_t g = nullptr;
  const cudaError_t ec = cudaStreamEndCapture(cs, &g);
  cudaStreamDestroy(cs);
  cuda_check(ec, "end capture");
  cudaGraphExec_t exec = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
  cudaGraphDestroy(g);
  cuda_check(e, "graph instantiate");
  graphs[n] = exec;
  return exec;
}

size_t PrefillRunner::launches_per_chunk(int n) const {
  auto it = launches.find(n);
  return it == launches.end() ? 0 : it->second;
}

void PrefillRunner::run(const uint32_t* ids, uint32_t n, uint32_t start, bool finish, cudaStream_t s) {
  for (uint32_t i = 0; i < n; ++i) pinned[i] = SeqCtl{ids[i], start + i, 0u, 0u};
  for (uint32_t c0 = 0; c0 < n; c0 += kRows) {
    const int cn = (int)std::min<uint32_t>(kRows, n - c0);
    cudaGraphExec_t g = graph_for(cn);
    cuda_check(cudaMemcpyAsync(rows, pinned + c0, (size_t)cn * sizeof(SeqCtl), cudaMemcpyHostToDevice, s),
               "prefill rows");
    cuda_check(cudaGraphLaunch(g, s), "prefill graph");
    for (size_t i = 0; i < launches[cn]; ++i) count_launch();
  }
  if (finish) {
    // The LM head of the B = 1 path on the last row: logits, then (greedy pick, start + n).
    const GemvArgs hd = r->head_args(Runner::kGreedy);
    if (const char* why = check_gemv(hd)) throw QneError(kEInval, why);
    cuda_check(launch_gemv(hd, s, false), "prefill head");
  }
}

}  // namespace qne
