// qne_gemm_noalloc: the batched tensor-core GEMM of qne_gemm with its working buffers in a fixed
// static device array, so that a call allocates no device memory at all.
//
// Why: qne_gemm stages x (and, for SwiGLU, the gate/up intermediate) in a per-device workspace
// that it grows with cudaMalloc (and frees with cudaFree) whenever a larger call arrives. Some
// callers cannot have that: a serving process that sized its memory plan up front (every byte
// not held by weights already belongs to its KV pool, so a late cudaMalloc fails or steals from
// the pool), and a latency-critical decode loop, where cudaFree synchronizes the device and a
// first-time cudaMalloc can take milliseconds. This entry point launches the same kernels as
// qne_gemm, in the same order, on buffers carved from kScratchBytes of static device memory.
//
// Set-up: the first call on each device (with that device current) resolves the array's device
// address with cudaGetSymbolAddress and caches it; later calls on that device reuse it. Make one
// call per device before any stream capture, so that capture never sees the set-up.
//
// Limits and contracts:
// - batch 1..64 (kGemmMaxRows), as qne_gemm.
// - A call needs 2 * Bp * k * 2 bytes for the x hi/lo planes (Bp = batch rounded up to 8), plus
//   2 * Bp * out_rows * 2 bytes with the SwiGLU epilogue; calls needing more than kScratchBytes
//   are rejected with QNE_EINVAL before anything is launched.
// - Nothing in the array has to start at zero: the planes' padding rows (batch .. Bp-1) only
//   feed output rows that are never stored, and every byte a stored output depends on is written
//   by the same call before it is read. (The array is zero at module load all the same.)
// - There is ONE array per device: calls that overlap in time on one device (different streams,
//   or different host threads without ordering) race on it and corrupt each other's results.
//   Serialize them on one stream.
#include <mutex>
#include <string>

#include "../../include/qne.h"
#include "batch.cuh"
#include "model.hpp"

using namespace qne;

extern "C" qne_status qne_internal_fail(int code, const char* msg);

namespace {

constexpr size_t kScratchBytes = 2u << 20;  // 2 MiB
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_gemm_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_gemm_scratch on the current device (set-up on the first call per device).
uint8_t* scratch_on_current_device() {
  int dev = -1;
  cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) throw QneError(kEInval, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gemm_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      throw QneError(kECuda, std::string("cudaGetSymbolAddress of the static GEMM scratch: ") +
                                 cudaGetErrorString(e));
    }
    g_scratch_ptr[dev] = p;
  }
  return static_cast<uint8_t*>(g_scratch_ptr[dev]);
}

}  // namespace

extern "C" {

qne_status qne_gemm_noalloc(const qne_matrix* m, const float* x, int batch, float* y, int epilogue, void* stream) {
  try {
    if (!m || !x || !y) throw QneError(kEInval, "null argument");
    if (m->kind != QNE_KIND_F16) throw QneError(kEInval, "batched GEMM supports f16 weights");
    if (epilogue < 0 || epilogue > 2) throw QneError(kEInval, "unknown epilogue");
    if (batch < 1 || batch > kGemmMaxRows) throw QneError(kEInval, "batch must be 1..64");
    if (m->k % 32 || m->k <= 0 || m->rows <= 0) throw QneError(kEInval, "batched GEMM needs k % 32 == 0");
    if (epilogue == QNE_EPI_SWIGLU && m->rows % 2) throw QneError(kEInval, "SwiGLU needs an even row count");
    const int Bp = (batch + 7) / 8 * 8;
    const int out_rows = epilogue == QNE_EPI_SWIGLU ? m->rows / 2 : m->rows;
    const size_t plane = (size_t)Bp * m->k * 2;
    const size_t need = 2 * plane + (epilogue == QNE_EPI_SWIGLU ? 2 * (size_t)Bp * out_rows * 2 : 0);
    if (need > kScratchBytes)
      throw QneError(kEInval, "qne_gemm_noalloc needs " + std::to_string(need) + " bytes of scratch for batch " +
                                  std::to_string(batch) + ", k " + std::to_string(m->k) + ", " +
                                  std::to_string(out_rows) + " output rows; its static array holds " +
                                  std::to_string(kScratchBytes) + " (use qne_gemm)");
    uint8_t* base = scratch_on_current_device();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint16_t* xh = reinterpret_cast<uint16_t*>(base);
    uint16_t* xl = xh + plane / 2;
    PrepArgs p;
    p.mode = kPrepCopy;
    p.k = m->k;
    p.src = x;
    p.lds = m->k;
    p.xh = xh;
    p.xl = xl;
    p.ldx = m->k;
    cuda_check(launch_prep(p, batch, s, false), "gemm prep");
    GemmArgs g;
    g.w = m->w;
    g.rows = m->rows;
    g.k = m->k;
    g.batch = batch;
    g.epi = epilogue;
    g.row_groups = gemm_row_groups(out_rows);
    g.xh = xh;
    g.xl = xl;
    g.ldx = m->k;
    g.ldy = out_rows;
    uint16_t* yh = xl + plane / 2;
    uint16_t* yl = yh + (size_t)Bp * out_rows;
    if (epilogue == QNE_EPI_SWIGLU) {
      g.yh = yh;
      g.yl = yl;
    } else {
      g.y = y;
    }
    if (const char* why = check_gemm(g)) throw QneError(kEInval, why);
    cuda_check(launch_gemm(g, s, false), "gemm");
    if (epilogue == QNE_EPI_SWIGLU)
      cuda_check(launch_hilo_to_f32(yh, yl, y, (size_t)batch * out_rows, s), "gemm swiglu output");
    qne_internal_fail(0, "");
    return QNE_OK;
  } catch (const QneError& e) {
    return qne_internal_fail(e.code, e.what());
  } catch (const std::exception& e) {
    return qne_internal_fail(QNE_EINVAL, e.what());
  }
}

}  // extern "C"
