// Streaming-read probe (bandwidth, kernels/src/shaders.rs:703-717) and the per-device RoPE
// table cache used by the attention operator entry point.
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

}  // namespace

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
