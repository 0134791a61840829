// Streaming-read probe (bandwidth, kernels/src/shaders.rs:703-717), the dispatch-cost probe
// (noop + dispatch_cost, kernels/src/shaders.rs:720-729 and kernels/src/lib.rs:718-724) and the
// per-device RoPE table cache used by the attention operator entry point.
#include <map>
#include <mutex>
#include <vector>

#include "gdn.cuh"
#include "gemv.cuh"
#include "model.hpp"

namespace qne {
namespace {

__global__ void __launch_bounds__(256) bandwidth_kernel(const uint4* data, size_t n, uint32_t* sink) {
  uint4 acc = make_uint4(0, 0, 0, 0);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n; i += 4 * stride) {
    const uint4 a = ld_stream(data + i), b = ld_stream(data + i + stride);
    const uint4 c = ld_stream(data + i + 2 * stride), d = ld_stream(data + i + 3 * stride);
    acc.x ^= a.x ^ b.x ^ c.x ^ d.x;
    acc.y ^= a.y ^ b.y ^ c.y ^ d.y;
    acc.z ^= a.z ^ b.z ^ c.z ^ d.z;
    acc.w ^= a.w ^ b.w ^ c.w ^ d.w;
  }
  for (; i < n; i += stride) {
    const uint4 a = ld_stream(data + i);
    acc.x ^= a.x;
    acc.y ^= a.y;
    acc.z ^= a.z;
    acc.w ^= a.w;
  }
  const uint32_t v = acc.x ^ acc.y ^ acc.z ^ acc.w;
  atomicXor(sink, v);
}

// noop, kernels/src/shaders.rs:720-729: thread 0 of one 64-thread block adds 1 to y[0]. The PDL
// form releases its successor first and waits for its predecessor before the update, as every
// kernel of the decode graphs does.
template <bool PDL>
__global__ void __launch_bounds__(64) noop_kernel(float* y) {
  if (PDL) {
    pdl_launch();
    pdl_wait();
  }
  if (threadIdx.x == 0) y[0] = y[0] + 1.0f;
}

cudaError_t launch_noop(float* y, bool pdl, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(64);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  return pdl ? cudaLaunchKernelEx(&cfg, noop_kernel<true>, y) : cudaLaunchKernelEx(&cfg, noop_kernel<false>, y);
}

}  // namespace

// dispatch_cost (kernels/src/lib.rs:718-724): n back-to-back noop launches on `s`, timed with CUDA
// events, as plain launches (mode 0), one CUDA graph of the n launches (1), launches with
// programmatic dependent launch (2) or a graph of those (3, how the decode step runs). Returns
// microseconds per launch.
double dispatch_cost(uint32_t n, int mode, float* y, cudaStream_t s) {
  const bool pdl = mode == 2 || mode == 3, graph = mode == 1 || mode == 3;
  cudaGraphExec_t exec = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaStream_t cs = nullptr;
  auto cleanup = [&]() {
    if (exec) cudaGraphExecDestroy(exec);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (cs) cudaStreamDestroy(cs);
  };
  try {
    cuda_check(cudaEventCreate(&e0), "cudaEventCreate");
    cuda_check(cudaEventCreate(&e1), "cudaEventCreate");
    if (graph) {
      cuda_check(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "cudaStreamCreate");
      cuda_check(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "begin capture");
      cudaError_t le = cudaSuccess;
      for (uint32_t i = 0; i < n && le == cudaSuccess; ++i) le = launch_noop(y, pdl, cs);
      cudaGraph_t g = nullptr;
      const cudaError_t ce = cudaStreamEndCapture(cs, &g);
      cuda_check(le, "noop launch");
      cuda_check(ce, "end capture");
      const cudaError_t ie = cudaGraphInstantiate(&exec, g, 0);
      cudaGraphDestroy(g);
      cuda_check(ie, "graph instantiate");
      cuda_check(cudaGraphLaunch(exec, s), "graph launch");  // warm-up
    } else {
      for (int i = 0; i < 10; ++i) cuda_check(launch_noop(y, pdl, s), "noop launch");
    }
    cuda_check(cudaStreamSynchronize(s), "dispatch_cost");
    cuda_check(cudaEventRecord(e0, s), "cudaEventRecord");
    if (graph) cuda_check(cudaGraphLaunch(exec, s), "graph launch");
    else
      for (uint32_t i = 0; i < n; ++i) cuda_check(launch_noop(y, pdl, s), "noop launch");
    cuda_check(cudaEventRecord(e1, s), "cudaEventRecord");
    cuda_check(cudaEventSynchronize(e1), "dispatch_cost");
    float ms = 0.f;
    cuda_check(cudaEventElapsedTime(&ms, e0, e1), "cudaEventElapsedTime");
    cleanup();
    return (double)ms * 1000.0 / n;
  } catch (...) {
    cleanup();
    throw;
  }
}

cudaError_t launch_bandwidth_probe(const void* data, size_t bytes, uint32_t* sink, cudaStream_t stream) {
  count_launch();
  bandwidth_kernel<<<kNumSms * 8, 256, 0, stream>>>(static_cast<const uint4*>(data), bytes / 16, sink);
  return cudaGetLastError();
}

const float* rope_table_device(double theta) {
  static std::mutex mu;
  static std::map<std::pair<int, double>, float*> tables;
  int dev = 0;
  cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(dev, theta);
  auto it = tables.find(key);
  if (it != tables.end()) return it->second;
  std::vector<float> host((size_t)2 * kMaxContext * kRopeHalf);
  rope_table_host(host.data(), theta);
  float* d = nullptr;
  cuda_check(cudaMalloc(&d, host.size() * 4), "cudaMalloc rope");
  cuda_check(cudaMemcpy(d, host.data(), host.size() * 4, cudaMemcpyHostToDevice), "upload rope");
  tables[key] = d;
  return d;
}

}  // namespace qne
