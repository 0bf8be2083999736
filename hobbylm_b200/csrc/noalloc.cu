// hg_op_q8_matvec_noalloc: the Q8 matvec entry point for callers that cannot allocate device memory.
//
// hg_op_q8_matvec quantizes its f32 activation rows into a scratch buffer it allocates on the
// stream. This variant keeps that scratch in a file-scope device array instead, so it makes no
// allocation call at all. The array is HG_NOALLOC_SCRATCH_BYTES bytes, lives on every device that
// loads the library until the process exits, and is shared by every call: concurrent or
// overlapping calls on one device race on it. Every byte a call reads is written by the same call
// first (the quantized rows and their scales), so nothing needs clearing between calls.
#include <climits>
#include <mutex>
#include <string>

#include "hg_host.h"
#include "hg_launch.h"

namespace hg {

static __device__ __align__(256) unsigned char g_noalloc_scratch[HG_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;

// Host code only has a host-side stand-in for g_noalloc_scratch; the device address is looked up
// once per device, with that device current, and cached. The cache assumes the device's primary
// context (the one the runtime API uses) for the life of the process: after cudaDeviceReset the
// cached address would be stale.
void* noalloc_scratch(int dev) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) throw Error(HG_ERR_INVALID, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) throw Error(HG_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    addr[dev] = p;
  }
  return addr[dev];
}

size_t up256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace
}  // namespace hg

using namespace hg;

extern "C" int hg_op_q8_matvec_noalloc(const int8_t* qs, const float* scales, int64_t rows, int64_t cols,
                                       const float* x, float* y, int ntok, void* stream) {
  try {
    if (!qs || !scales || !x || !y || rows <= 0 || cols <= 0 || cols % 32 != 0 || ntok <= 0)
      throw Error(HG_ERR_INVALID, "bad argument");
    // the kernels index rows and columns with int: bound both before the scratch size is formed
    // (with cols <= INT_MAX and ntok <= INT_MAX the products below cannot wrap in size_t)
    if (rows > INT_MAX || cols > INT_MAX) throw Error(HG_ERR_INVALID, "rows and cols must be at most INT_MAX");
    const size_t need = up256((size_t)ntok * (size_t)cols) + (size_t)ntok * host_q8_ss(cols) * 4;
    if (need > HG_NOALLOC_SCRATCH_BYTES)
      throw Error(HG_ERR_INVALID, "hg_op_q8_matvec_noalloc: ntok * cols needs " + std::to_string(need) +
                                      " scratch bytes, more than the fixed " +
                                      std::to_string((size_t)HG_NOALLOC_SCRATCH_BYTES));
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) throw Error(HG_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    char* base = static_cast<char*>(noalloc_scratch(dev));
    int8_t* aq = reinterpret_cast<int8_t*>(base);
    float* as = reinterpret_cast<float*>(base + up256((size_t)ntok * (size_t)cols));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    launch_quant_rows(x, ntok, (int)cols, aq, as, st);
    Q8M W;
    W.qs = qs;
    W.sc = scales;
    W.rows = (int)rows;
    W.cols = (int)cols;
    W.ss = host_q8_ss(cols);
    W.qs_mstride = rows * cols;
    W.sc_mstride = rows * W.ss;
    Dims D{};
    DecodeBufs B{};
    B.T = ntok;
    launch_mv_store(D, B, W, aq, as, y, (int)rows, st);
    e = cudaGetLastError();
    if (e != cudaSuccess) throw Error(HG_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
    return HG_OK;
  } catch (const Error& ex) {
    set_last_error(ex.what());
    return ex.code;
  } catch (const std::exception& ex) {
    set_last_error(ex.what());
    return HG_ERR_INVALID;
  }
}
