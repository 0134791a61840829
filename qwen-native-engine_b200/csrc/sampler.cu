// Token sampling on the device over the model's logits (Sampler::try_sample / choose,
// src/sampling.rs:40-134): greedy, or temperature + top-k + top-p, with a presence penalty on
// already generated tokens (not under a grammar mask), an optional grammar mask, and the agent's
// tool-call bias added to one logit first (agent/src/session.rs:400-406). Only the chosen token
// and a status word return to the host (8 bytes instead of the 993 KB of f32 logits).
//
// Two kernels:
//  * sample_candidates_kernel, one CTA per 2048-token slice of the vocabulary: biased and
//    penalized logits of the allowed tokens as order-preserving 32-bit keys (0 = not allowed);
//    the NaN / +inf and "any finite" checks of try_sample; then either the slice's greedy pick
//    or its top-k candidates, found by a byte-wise radix select over the keys in shared memory;
//  * sample_final_kernel, one CTA: the global greedy pick, or the top-k of all candidates (the
//    same radix select), sorted by (logit descending, index ascending), then the reference's
//    sequential f32 arithmetic: weights exp((l - top) / T), their sum, the shortest prefix
//    holding top_p of it, and the draw r = u * kept walked down the prefix.
// The uniform u comes from the host, which runs the reference's xorshift64 generator, so the
// device holds no generator state; the presence-penalty set is a device bitmap.
//
// Ties: the reference selects and sorts with unstable algorithms, so the order of equal logits
// is unspecified there; here equal logits rank by lower token index (greedy included, as the
// reference's strict `>` scan does).
#include <math.h>

#include <cstring>
#include <string>
#include <vector>

#include "../../include/qne.h"
#include "model.hpp"

extern "C" qne_status qne_internal_fail(int code, const char* msg);

namespace qne {
namespace {

constexpr int kSliceTokens = 2048;  // vocabulary tokens per candidate CTA
constexpr int kMaxSlices = 128;     // vocabularies up to 262144 tokens
constexpr int kMaxTopK = 256;
constexpr int kCandThreads = 256;
constexpr int kFinalThreads = 1024;
constexpr uint32_t kFlagNonFinite = 1u, kFlagFinite = 2u;

struct SampleArgs {
  const float* logits;
  int vocab;
  const uint32_t* mask;  // bitset, or null
  int mask_tokens;
  const uint32_t* seen;  // presence-penalty bitmap
  float penalty;         // 0 under a mask
  int bias_token;        // -1: none
  float bias;
  int k;                 // top_k clamped to 1..256
  int greedy;
  float temperature, top_p, u;
  uint32_t* cand_key;    // [slices][256]
  uint32_t* cand_idx;
  uint32_t* cand_count;  // [slices]
  float* gval;           // [slices] greedy partials
  uint32_t* gidx;
  uint32_t* flags;       // kFlagNonFinite | kFlagFinite, reset by the final kernel
  uint32_t* result;      // token, status
  uint32_t* seen_out;    // bitmap updated with the pick when the penalty is on (else null)
};

// Order-preserving map of a float to 32 bits; allowed keys are >= 0x007FFFFF (-inf), 0 = none.
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Block-wide radix select: among the items with valid[i], finds the value T of the want-th
// largest key (1-based) and how many items equal to T belong to the top `want` (returned in
// `ties`). All threads of the block must call it; hist and bc are shared scratch.
template <int N, int THREADS>
__device__ uint32_t select_kth_largest(const uint32_t (&key)[N], const bool (&valid)[N], uint32_t want,
                                       uint32_t* hist, uint32_t* bc, uint32_t& ties) {
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t prefix = 0, pmask = 0;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += THREADS) hist[i] = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (valid[j] && (key[j] & pmask) == prefix) atomicAdd(&hist[(key[j] >> shift) & 255u], 1u);
    __syncthreads();
    if (tid < 32) {
      // lane l scans digits 255 - 8l .. 248 - 8l (descending); suffix counts by a warp scan
      uint32_t c[8], s = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = hist[255 - 8 * lane - i];
        s += c[i];
      }
      uint32_t incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      uint32_t before = incl - s;  // items with a larger digit than this lane's range
      if (before < want && want <= incl) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (before + c[i] >= want) {
            bc[0] = 255u - 8u * lane - i;
            bc[1] = want - before;
            break;
          }
          before += c[i];
        }
      }
    }
    __syncthreads();
    prefix |= bc[0] << shift;
    pmask |= 255u << shift;
    want = bc[1];
    __syncthreads();
  }
  ties = want;
  return prefix;
}

template <int THREADS>
__device__ uint32_t block_count(uint32_t v, uint32_t* red) {
  v = __reduce_add_sync(0xffffffffu, v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t s = 0;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) s += red[w];
  __syncthreads();
  return s;
}

// Keeps the top `k` of the items (ties at the threshold by lower index): returns per item whether
// it is kept. n_valid = number of valid items in the block. When every item equal to the k-th
// largest key belongs to the top k (no tie crosses the threshold: the usual case), the second
// selection that orders the tied items by index is skipped.
template <int N, int THREADS>
__device__ void keep_top_k(const uint32_t (&key)[N], const uint32_t (&idx)[N], const bool (&valid)[N], uint32_t k,
                           uint32_t n_valid, bool (&keep)[N], uint32_t* hist, uint32_t* bc, uint32_t* red) {
  if (n_valid <= k) {
#pragma unroll
    for (int j = 0; j < N; ++j) keep[j] = valid[j];
    return;
  }
  uint32_t ties = 0;
  const uint32_t T = select_kth_largest<N, THREADS>(key, valid, k, hist, bc, ties);
  uint32_t ne = 0;
#pragma unroll
  for (int j = 0; j < N; ++j) ne += (valid[j] && key[j] == T) ? 1u : 0u;
  if (block_count<THREADS>(ne, red) == ties) {
#pragma unroll
    for (int j = 0; j < N; ++j) keep[j] = valid[j] && key[j] >= T;
    return;
  }
  // among the items equal to T, the `ties` lowest indices: the ties-th largest of ~index
  uint32_t nidx[N];
  bool tie[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    tie[j] = valid[j] && key[j] == T;
    nidx[j] = ~idx[j];
  }
  uint32_t dummy = 0;
  const uint32_t TI = select_kth_largest<N, THREADS>(nidx, tie, ties, hist, bc, dummy);
#pragma unroll
  for (int j = 0; j < N; ++j) keep[j] = valid[j] && (key[j] > T || (key[j] == T && nidx[j] >= TI));
}

__global__ void __launch_bounds__(kCandThreads) sample_candidates_kernel(const SampleArgs a) {
  constexpr int N = kSliceTokens / kCandThreads;  // 8
  __shared__ uint32_t hist[256], bc[2], red[kCandThreads / 32], cnt;
  __shared__ float bv[kCandThreads / 32];
  __shared__ uint32_t bi[kCandThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = blockIdx.x * kSliceTokens;
  uint32_t key[N], idx[N];
  bool valid[N];
  uint32_t fl = 0;
  float best = -INFINITY;
  uint32_t best_i = 0xFFFFFFFFu;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const int i = c0 + j * kCandThreads + tid;
    idx[j] = (uint32_t)i;
    bool ok = i < a.vocab;
    if (ok && a.mask) ok = i < a.mask_tokens && ((a.mask[i >> 5] >> (i & 31)) & 1u);
    float raw = ok ? a.logits[i] : 0.f;
    if (i == a.bias_token) raw += a.bias;
    if (ok) {
      if (isnan(raw) || raw == INFINITY) fl |= kFlagNonFinite;
      if (isfinite(raw)) fl |= kFlagFinite;
    }
    float l = raw;
    if (ok && a.penalty != 0.f && ((a.seen[i >> 5] >> (i & 31)) & 1u)) l = raw - a.penalty;
    valid[j] = ok;
    key[j] = ok ? fkey(l) : 0u;
    if (ok && l > best) {  // ascending index per thread: the first maximum wins
      best = l;
      best_i = (uint32_t)i;
    }
  }
  fl = __reduce_or_sync(0xffffffffu, fl);
  if (lane == 0 && fl) atomicOr(a.flags, fl);
  if (a.greedy) {
    // block (max, lowest index)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (oi != 0xFFFFFFFFu && (best_i == 0xFFFFFFFFu || ov > best || (ov == best && oi < best_i))) {
        best = ov;
        best_i = oi;
      }
    }
    if (lane == 0) {
      bv[warp] = best;
      bi[warp] = best_i;
    }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < kCandThreads / 32; ++w)
        if (bi[w] != 0xFFFFFFFFu && (best_i == 0xFFFFFFFFu || bv[w] > best || (bv[w] == best && bi[w] < best_i))) {
          best = bv[w];
          best_i = bi[w];
        }
      a.gval[blockIdx.x] = best;
      a.gidx[blockIdx.x] = best_i;
    }
    return;
  }
  uint32_t nv = 0;
#pragma unroll
  for (int j = 0; j < N; ++j) nv += valid[j] ? 1u : 0u;
  const uint32_t n_valid = block_count<kCandThreads>(nv, red);
  bool keep[N];
  keep_top_k<N, kCandThreads>(key, idx, valid, (uint32_t)a.k, n_valid, keep, hist, bc, red);
  if (tid == 0) cnt = 0;
  __syncthreads();
  uint32_t* ck = a.cand_key + (size_t)blockIdx.x * kMaxTopK;
  uint32_t* ci = a.cand_idx + (size_t)blockIdx.x * kMaxTopK;
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (keep[j]) {
      const uint32_t p = atomicAdd(&cnt, 1u);
      ck[p] = key[j];
      ci[p] = idx[j];
    }
  __syncthreads();
  if (tid == 0) a.cand_count[blockIdx.x] = cnt;
}

// N: candidate slots per thread; the slices' candidates are read compacted (slice s's kept items
// at offsets off[s] .. off[s + 1] of one list), so N * kFinalThreads only has to cover their count.
template <int N>
__global__ void __launch_bounds__(kFinalThreads) sample_final_kernel(const SampleArgs a, int slices) {
  __shared__ uint32_t hist[256], bc[2], red[kFinalThreads / 32], cnt;
  __shared__ uint32_t sk[kMaxTopK], si[kMaxTopK], ok[kMaxTopK], oi[kMaxTopK];
  __shared__ uint32_t off[kMaxSlices + 1];
  __shared__ float ew[kMaxTopK];
  const int tid = threadIdx.x;
  const uint32_t fl = *a.flags;
  const uint32_t status = (fl & kFlagNonFinite) ? 1u : ((fl & kFlagFinite) ? 0u : 2u);
  uint32_t token = 0;
  if (a.greedy) {
    if (tid == 0) {
      float best = -INFINITY;
      uint32_t best_i = 0xFFFFFFFFu;
      for (int s = 0; s < slices; ++s) {
        const float v = a.gval[s];
        const uint32_t i = a.gidx[s];
        if (i != 0xFFFFFFFFu && (best_i == 0xFFFFFFFFu || v > best || (v == best && i < best_i))) {
          best = v;
          best_i = i;
        }
      }
      token = best_i == 0xFFFFFFFFu ? 0u : best_i;
    }
  } else {
    // exclusive prefix of the slices' candidate counts (warp 0: 4 slices per lane)
    static_assert(kMaxSlices == 32 * 4, "one warp scans the slice counts");
    if (tid < 32) {
      uint32_t c[4], sum = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int sl = tid * 4 + i;
        c[i] = sl < slices ? a.cand_count[sl] : 0u;
        sum += c[i];
      }
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += v;
      }
      uint32_t run = incl - sum;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        off[tid * 4 + i] = run;
        run += c[i];
      }
      if (tid == 31) off[kMaxSlices] = incl;
    }
    __syncthreads();
    const uint32_t total = off[kMaxSlices];
    uint32_t key[N], idx[N];
    bool valid[N];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const uint32_t e = (uint32_t)(j * kFinalThreads + tid);
      valid[j] = e < total;
      key[j] = 0u;
      idx[j] = 0u;
      if (valid[j]) {
        int lo = 0, hi = slices - 1;  // the slice holding candidate e: last s with off[s] <= e
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (off[mid] <= e) lo = mid;
          else hi = mid - 1;
        }
        const size_t q = (size_t)lo * kMaxTopK + (e - off[lo]);
        key[j] = a.cand_key[q];
        idx[j] = a.cand_idx[q];
      }
    }
    uint32_t nv = 0;
#pragma unroll
    for (int j = 0; j < N; ++j) nv += valid[j] ? 1u : 0u;
    const uint32_t n_valid = block_count<kFinalThreads>(nv, red);
    const uint32_t k = min((uint32_t)a.k, n_valid);
    bool keep[N];
    keep_top_k<N, kFinalThreads>(key, idx, valid, k, n_valid, keep, hist, bc, red);
    if (tid == 0) cnt = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (keep[j]) {
        const uint32_t p = atomicAdd(&cnt, 1u);
        sk[p] = key[j];
        si[p] = idx[j];
      }
    __syncthreads();
    // sort by (logit descending, index ascending): rank of each kept item
    const uint32_t n = cnt;
    if ((uint32_t)tid < n) {
      uint32_t r = 0;
      for (uint32_t j = 0; j < n; ++j) r += (sk[j] > sk[tid] || (sk[j] == sk[tid] && si[j] < si[tid])) ? 1u : 0u;
      ok[r] = sk[tid];
      oi[r] = si[tid];
    }
    __syncthreads();
    // the weights exp((l - top) / T) in parallel (each value as the reference computes it)
    if ((uint32_t)tid < n) ew[tid] = expf((key_f(ok[tid]) - key_f(ok[0])) / a.temperature);
    __syncthreads();
    if (tid == 0 && n > 0 && status == 0) {
      // The reference's arithmetic, in its order (src/sampling.rs:105-133).
      float wsum = 0.f;
      for (uint32_t j = 0; j < n; ++j) wsum += ew[j];
      float kept = 0.f;
      uint32_t m = 0;
      for (uint32_t j = 0; j < n; ++j) {
        kept += ew[j];
        ++m;
        if (kept >= a.top_p * wsum) break;
      }
      float r = a.u * kept;
      token = oi[m - 1];
      for (uint32_t j = 0; j < m; ++j) {
        r -= ew[j];
        if (r <= 0.f) {
          token = oi[j];
          break;
        }
      }
    }
  }
  if (tid == 0) {
    if (status != 0) token = 0;
    a.result[0] = token;
    a.result[1] = status;
    *a.flags = 0u;
    if (status == 0 && a.seen_out) atomicOr(a.seen_out + (token >> 5), 1u << (token & 31));
  }
}

}  // namespace

// ------------------------------------------------------------------------------------------
// Host side: the sampler of one generation (Sampler, src/sampling.rs:30-58).
// ------------------------------------------------------------------------------------------
struct Sampler {
  Model* m = nullptr;
  qne_sampling opts{};
  uint64_t state = 0;
  int vocab = 0, slices = 0;
  uint32_t *seen = nullptr, *mask = nullptr, *cand_key = nullptr, *cand_idx = nullptr, *cand_count = nullptr;
  float* gval = nullptr;
  uint32_t *gidx = nullptr, *flags = nullptr, *result = nullptr;
  uint32_t* pinned = nullptr;  // token, status
  std::vector<void*> owned;    // device buffers of this sampler
  void* alloc(size_t bytes) {
    void* p = nullptr;
    cuda_check(cudaMalloc(&p, bytes), "cudaMalloc");
    owned.push_back(p);
    return p;
  }
  ~Sampler() {
    for (void* p : owned) cudaFree(p);
    if (pinned) cudaFreeHost(pinned);
  }
  // The reference's xorshift64 draw (src/sampling.rs:45-53).
  float next_f32() {
    uint64_t x = state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    state = x;
    return (float)(x >> 40) / (float)(1ull << 24);
  }
  void sample(const float* logits, const uint32_t* host_mask, uint32_t mask_tokens, int bias_token, float bias,
              uint32_t* token_out) {
    cudaStream_t s = m->stream();
    const bool use_mask = host_mask != nullptr;
    if (use_mask) {
      const size_t words = ((size_t)std::min<uint32_t>(mask_tokens, (uint32_t)vocab) + 31) / 32;
      if (words) cuda_check(cudaMemcpyAsync(mask, host_mask, words * 4, cudaMemcpyHostToDevice, s), "sampling mask");
    }
    const uint64_t saved = state;
    SampleArgs a{};
    a.logits = logits;
    a.vocab = vocab;
    a.mask = use_mask ? mask : nullptr;
    a.mask_tokens = use_mask ? (int)std::min<uint32_t>(mask_tokens, (uint32_t)vocab) : 0;
    a.seen = seen;
    a.penalty = use_mask ? 0.f : opts.presence_penalty;
    a.bias_token = (bias != 0.f && bias_token >= 0 && bias_token < vocab) ? bias_token : -1;
    a.bias = bias;
    a.k = (int)std::min<uint32_t>(std::max<uint32_t>(opts.top_k, 1u), (uint32_t)kMaxTopK);
    a.greedy = opts.temperature <= 0.f ? 1 : 0;
    a.temperature = opts.temperature;
    a.top_p = opts.top_p;
    a.u = a.greedy ? 0.f : next_f32();
    a.cand_key = cand_key;
    a.cand_idx = cand_idx;
    a.cand_count = cand_count;
    a.gval = gval;
    a.gidx = gidx;
    a.flags = flags;
    a.result = result;
    a.seen_out = opts.presence_penalty != 0.f ? seen : nullptr;
    count_launch();
    sample_candidates_kernel<<<slices, kCandThreads, 0, s>>>(a);
    cuda_check(cudaGetLastError(), "sampling launch");
    count_launch();
    // candidate slots: every slice keeps at most k; 4 per thread cover up to 4096 of them
    if ((size_t)slices * (size_t)a.k <= 4u * kFinalThreads) sample_final_kernel<4><<<1, kFinalThreads, 0, s>>>(a, slices);
    else sample_final_kernel<kMaxSlices * kMaxTopK / kFinalThreads><<<1, kFinalThreads, 0, s>>>(a, slices);
    cuda_check(cudaGetLastError(), "sampling launch");
    cuda_check(cudaMemcpyAsync(pinned, result, 8, cudaMemcpyDeviceToHost, s), "sampling result");
    m->sync(600000);
    if (pinned[1] != 0) {
      state = saved;  // a failed draw does not advance the generator
      throw QneError(kEInval, pinned[1] == 1 ? "non-finite model logits"
                                             : "no finite token is allowed by the sampling mask");
    }
    *token_out = pinned[0];
  }
};

}  // namespace qne

using namespace qne;

namespace {
qne_status sfail(int code, const std::string& msg) { return qne_internal_fail(code, msg.c_str()); }
template <typename F>
qne_status sguard(F&& f) {
  try {
    f();
    qne_internal_fail(0, "");
    return QNE_OK;
  } catch (const QneError& e) {
    return sfail(e.code, e.what());
  } catch (const std::bad_alloc&) {
    return sfail(QNE_ENOMEM, "host allocation failed");
  } catch (const std::exception& e) {
    return sfail(QNE_EINVAL, e.what());
  }
}
}  // namespace

extern "C" {

qne_status qne_sampler_create(qne_model* model, const qne_sampling* opts, qne_sampler** out) {
  if (!out) return sfail(QNE_EINVAL, "null output handle");
  *out = nullptr;
  if (!model || !opts) return sfail(QNE_EINVAL, "null model or options");
  return sguard([&] {
    Model* M = reinterpret_cast<Model*>(model);
    if (!(opts->top_p == opts->top_p) || !(opts->temperature == opts->temperature))
      throw QneError(kEInval, "NaN sampling option");
    if (opts->temperature > 0.f && opts->top_k > (uint32_t)kMaxTopK)
      throw QneError(kEInval, "top_k above 256 is not supported on the device");
    if (M->cfg.vocab > kMaxSlices * kSliceTokens) throw QneError(kEInval, "vocabulary above 262144 tokens");
    DeviceGuard g(M->device);
    auto* S = new Sampler();
    try {
      S->m = M;
      S->opts = *opts;
      S->state = opts->seed * 0x9E3779B97F4A7C15ull | 1ull;  // xorshift has a fixed point at zero
      S->vocab = M->cfg.vocab;
      S->slices = (S->vocab + kSliceTokens - 1) / kSliceTokens;
      const size_t words = ((size_t)S->vocab + 31) / 32;
      S->seen = static_cast<uint32_t*>(S->alloc(words * 4));
      S->mask = static_cast<uint32_t*>(S->alloc(words * 4));
      S->cand_key = static_cast<uint32_t*>(S->alloc((size_t)kMaxSlices * kMaxTopK * 4));
      S->cand_idx = static_cast<uint32_t*>(S->alloc((size_t)kMaxSlices * kMaxTopK * 4));
      S->cand_count = static_cast<uint32_t*>(S->alloc((size_t)kMaxSlices * 4));
      S->gval = static_cast<float*>(S->alloc((size_t)kMaxSlices * 4));
      S->gidx = static_cast<uint32_t*>(S->alloc((size_t)kMaxSlices * 4));
      S->flags = static_cast<uint32_t*>(S->alloc(16));
      S->result = static_cast<uint32_t*>(S->alloc(16));
      for (void* p : {(void*)S->seen, (void*)S->mask}) cuda_check(cudaMemset(p, 0, words * 4), "sampler");
      cuda_check(cudaMemset(S->flags, 0, 16), "sampler");
      cuda_check(cudaMallocHost(&S->pinned, 16), "cudaMallocHost");
    } catch (...) {
      delete S;
      throw;
    }
    *out = reinterpret_cast<qne_sampler*>(S);
  });
}

void qne_sampler_free(qne_sampler* s) {
  if (!s) return;
  Sampler* S = reinterpret_cast<Sampler*>(s);
  const int dev = S->m->device;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != dev) cudaSetDevice(dev);
  delete S;
  if (prev >= 0 && prev != dev) cudaSetDevice(prev);
}

qne_status qne_sampler_sample(qne_sampler* s, const uint32_t* mask, uint32_t mask_tokens, int32_t bias_token,
                              float bias, uint32_t* token_out) {
  if (!s || !token_out) return sfail(QNE_EINVAL, "null sampler or output");
  return sguard([&] {
    Sampler* S = reinterpret_cast<Sampler*>(s);
    DeviceGuard g(S->m->device);
    S->sample(S->m->logits_device(), mask, mask_tokens, bias_token, bias, token_out);
  });
}

qne_status qne_sampler_sample_device(qne_sampler* s, const float* logits, const uint32_t* mask, uint32_t mask_tokens,
                                     int32_t bias_token, float bias, uint32_t* token_out) {
  if (!s || !logits || !token_out) return sfail(QNE_EINVAL, "null sampler, logits or output");
  return sguard([&] {
    Sampler* S = reinterpret_cast<Sampler*>(s);
    DeviceGuard g(S->m->device);
    S->sample(logits, mask, mask_tokens, bias_token, bias, token_out);
  });
}

qne_status qne_step_sample(qne_model* model, qne_sampler* s, uint32_t token, uint32_t pos, const uint32_t* mask,
                           uint32_t mask_tokens, int32_t bias_token, float bias, uint32_t* token_out) {
  if (!model || !s || !token_out) return sfail(QNE_EINVAL, "null model, sampler or output");
  return sguard([&] {
    Model* M = reinterpret_cast<Model*>(model);
    Sampler* S = reinterpret_cast<Sampler*>(s);
    if (S->m != M) throw QneError(kEInval, "the sampler belongs to another model");
    DeviceGuard g(M->device);
    M->step_async(token, pos);
    S->sample(M->logits_device(), mask, mask_tokens, bias_token, bias, token_out);
  });
}

}  // extern "C"
