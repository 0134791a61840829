// Fused layer kernels: one decoder layer of kernels/src/model.rs:220-269 (in-projection, GDN or
// attention mixer, out-projection + residual, gate/up + SwiGLU, down + residual; the last layer
// also the final norm, LM head and greedy pick) as ONE launch of a co-resident grid, for a single
// sequence with f16 weights. A token takes one launch per layer instead of five or six kernels.
//
// Every CTA stays resident for the whole layer; a grid-wide barrier separates phases whose
// inputs the previous phase produces. Before arriving at a barrier each CTA already loads what
// the next phase needs and nobody in this launch writes: the first units of its GEMV rows (into
// its cp.async ring), its GDN state slice, or the keys and values of its attention split. The
// barrier's latency therefore overlaps the next phase's DRAM traffic. Consecutive layer launches
// overlap through programmatic dependent launch: the next layer's in-projection weights stream
// before it waits. (Bulk L2 prefetch of later phases' weights was measured and slows the step:
// it competes with the current phase for DRAM rather than filling the gaps between phases.)
//
// The layer is straight-line code on purpose: the phases of a runtime loop over layers keep
// each other's loop-invariant state live and exceed the 128 registers that two CTAs per SM
// allow.
//
// Grid barriers (GridBarrier below) wait with a time limit and, on timeout, set kFlagTimeout in
// the sequence's control word and carry on, so a fault can never hang the GPU. The grid is the
// occupancy bound, so all CTAs are co-resident (see launch_layer_t).

#include "attn_dev.cuh"
#include "gdn_dev.cuh"
#include "gemv_dev.cuh"
#include "persist.cuh"

namespace qne {
namespace {

using namespace dev;


__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_release64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Optional phase trace: thread 0 of every CTA stamps %globaltimer into trace[cta * 32 + slot]
// (slot 0 kernel start, 1 end of the wait on the previous kernel, 2 + p end of phase p, 8-15
// barrier arrivals, 16-23 barrier releases).
struct Trace {
  unsigned long long* t;
  int nb;
  __device__ __forceinline__ void mark(int slot) const {
    if (t && threadIdx.x == 0) t[blockIdx.x * 32 + slot] = global_ns();
  }
};

// Grid-wide barrier on an arrival counter that every launch finds at zero: barrier n of the
// launch completes when the counter reaches n * gridDim.x. Thread 0 of each CTA arrives with a
// release reduction (publishing the CTA's writes, ordered before it by the CTA barrier) and polls
// with acquire loads, so an arrival costs no round trip and there is no second write by a last
// arrival. At exit every CTA counts itself out; the last one clears both counters for the next
// launch, which touches them only after its dependency wait on this launch. Waits are bounded in
// time; once any CTA has given up (kFlagTimeout in *err) the others stop waiting too, so a broken
// barrier costs one limit, not one per phase. The host clears the counters when it sees the flag.
struct GridBarrier {
  unsigned long long* count;  // [0] arrivals, [1] exits
  unsigned long long target;  // thread 0 only
  uint64_t limit_ns;          // time limit of one wait
  uint32_t extra;             // arrivals waited for beyond the grid (0; 1 = never completes, test only)

  __device__ __forceinline__ void wait(uint32_t* err, Trace& tr) {
    __syncthreads();
    if (threadIdx.x == 0) {
      tr.mark(8 + tr.nb);
      target += gridDim.x + extra;
      red_add_release64(count, 1ull);
      const uint64_t t0 = global_ns();
      uint32_t rounds = 0;
      while (ld_acquire64(count) < target) {
        if ((++rounds & 63u) == 0u) {
          if (ld_acquire(err) & kFlagTimeout) break;
          if (global_ns() - t0 > limit_ns) {
            atomicOr(err, kFlagTimeout);
            break;
          }
        }
      }
      tr.mark(16 + tr.nb);
      ++tr.nb;
    }
    __syncthreads();
  }

  __device__ __forceinline__ void exit() {
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(count + 1, 1ull) == gridDim.x - 1) {
      count[0] = 0ull;
      count[1] = 0ull;
      __threadfence();
    }
  }
};

// One GEMV phase: the warp's first units of weights into its ring, then the wait for the input
// (the previous kernel for the in-projection, else the grid barrier), then the prologue and the
// stream.
__device__ __forceinline__ void gemv_phase(const GemvArgs& g, float* xs, uint8_t* ring,
                                           GemvShared& sh, GridBarrier& bar, uint32_t* err, Trace& tr,
                                           bool first) {
  RingPipe pipe;
  pipe.init(g, blockIdx.x, gridDim.x, ring);
  pipe.prefetch();
  if (first) {
    pdl_wait();
    tr.mark(1);
  } else {
    bar.wait(err, tr);
  }
  pipe.run(g, xs, sh);
}

// The mixer phases have 128 work items and the grid at least 128 CTAs (persist_ctas), so each
// CTA runs at most one item and the item's loads stay in registers across the barrier.
__device__ __forceinline__ void attention_phase(const KernelArgs& ka, GridBarrier& bar,
                                                uint32_t* err, AttnShared& ash, Trace& tr) {
  const bool mine = (int)blockIdx.x < kMaxSplits * kKvHeads;
  AttnItem it;
  __syncthreads();  // the item stages K/V into the region other warps' GEMV rings just used
  if (mine) it.prefetch(ka, ash, blockIdx.x);
  bar.wait(err, tr);
  if (mine) it.run(ka, ash);
}

__device__ __forceinline__ void gdn_phase(const GdnArgs& ga, GridBarrier& bar, uint32_t* err,
                                          GdnShared& dsh, Trace& tr) {
  const bool mine = (int)blockIdx.x < kGdnItemsPerSeq;
  GdnItem it;
  if (mine) it.prefetch(ga, blockIdx.x);
  bar.wait(err, tr);
  if (mine) it.run(ga, dsh);
}

// Dynamic shared memory of a fused layer kernel: the GEMV input planes (max_k floats), then one
// region used in turn by the GEMV cp.async rings and by the GDN or attention work item (phases
// never overlap within a CTA: a mixer item runs after the in-projection's ring has drained and
// the next GEMV fills the ring only after the item is done).
constexpr size_t kUnionBytes = sizeof(AttnShared) > (size_t)RingPipe::kRingBytes
                                   ? (sizeof(AttnShared) > sizeof(GdnShared) ? sizeof(AttnShared) : sizeof(GdnShared))
                                   : ((size_t)RingPipe::kRingBytes > sizeof(GdnShared) ? (size_t)RingPipe::kRingBytes
                                                                                        : sizeof(GdnShared));

template <bool ATTN, bool HEAD>
__global__ void __launch_bounds__(256, 2) layer_kernel(const __grid_constant__ LayerLaunch a) {
  extern __shared__ __align__(16) uint8_t smem[];
  float* xs = reinterpret_cast<float*>(smem);
  uint8_t* ring = smem + a.xs_bytes;
  AttnShared& ash = *reinterpret_cast<AttnShared*>(ring);
  GdnShared& dsh = *reinterpret_cast<GdnShared*>(ring);
  __shared__ GemvShared gsh;
  GridBarrier bar{a.barrier, 0ull, a.wait_limit_ns, a.wait_extra};
  uint32_t* err = a.err;
  Trace tr{a.trace, 0};
  tr.mark(0);
  pdl_launch();
  // One loop over the phases with a single GEMV call site: the GEMV code exists once in the
  // kernel, so its instructions stay cached from one phase to the next.
  const int phases = HEAD ? kPhases : kPhHead;
#pragma unroll 1
  for (int ph = kPhIn; ph < phases; ++ph) {
    if (ph == kPhMixer) {
      if (ATTN) attention_phase(a.attn, bar, err, ash, tr);
      else gdn_phase(a.gdn, bar, err, dsh, tr);
    } else {
      gemv_phase(a.g[ph], xs, ring, gsh, bar, err, tr, ph == kPhIn);
    }
    tr.mark(2 + ph);
  }
  if (HEAD) argmax_finish(a.g[kPhHead], blockIdx.x, gridDim.x, gsh);
  bar.exit();
}

template <bool ATTN, bool HEAD>
cudaError_t launch_layer_t(const LayerLaunch& args, int ctas, size_t smem, cudaStream_t stream, bool pdl) {
  cudaError_t e = cudaFuncSetAttribute(layer_kernel<ATTN, HEAD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // A plain launch with programmatic dependent launch, not a cooperative one: the next layer's
  // CTAs then start (and fill their rings) while this one drains, which a cooperative launch does
  // not allow. All CTAs are still co-resident: the grid is the occupancy bound (persist_ctas),
  // the next launch can only take SM slots once every CTA of this one has started (each calls
  // launch_dependents first), and every barrier wait is bounded in time.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  return cudaLaunchKernelEx(&cfg, layer_kernel<ATTN, HEAD>, args);
}

}  // namespace

size_t persist_xs_bytes(int max_k) { return ((size_t)max_k * sizeof(float) + 127) & ~(size_t)127; }
size_t persist_smem_bytes(int max_k) { return persist_xs_bytes(max_k) + kUnionBytes; }

int persist_ctas(int max_k) {
  int dev = 0, sms = 0, n = 1 << 30;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = persist_smem_bytes(max_k);
  const void* kernels[4] = {(const void*)layer_kernel<false, false>, (const void*)layer_kernel<false, true>,
                            (const void*)layer_kernel<true, false>, (const void*)layer_kernel<true, true>};
  for (const void* k : kernels) {
    int per_sm = 0;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, 256, smem) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    if (per_sm > 2) per_sm = 2;
    n = per_sm * sms < n ? per_sm * sms : n;
  }
  if (n > kMaxGrid) n = kMaxGrid;
  return n < kMaxSplits * kKvHeads || n < kGdnItemsPerSeq ? 0 : n;
}

cudaError_t launch_layer(const LayerLaunch& args, bool attention, bool head, int ctas, int max_k,
                         cudaStream_t stream, bool pdl) {
  const size_t smem = persist_smem_bytes(max_k);
  if (attention) return head ? launch_layer_t<true, true>(args, ctas, smem, stream, pdl)
                             : launch_layer_t<true, false>(args, ctas, smem, stream, pdl);
  return head ? launch_layer_t<false, true>(args, ctas, smem, stream, pdl)
              : launch_layer_t<false, false>(args, ctas, smem, stream, pdl);
}

}  // namespace qne
