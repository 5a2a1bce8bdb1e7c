// noalloc.cu — a BitLinear forward that allocates nothing.
//
// obn_bitlinear_forward needs a device workspace from its caller. Some callers
// cannot provide one: hosts whose device memory is reserved up front by another
// allocator (nothing is left for a foreign library to cudaMalloc, and they have no
// way to lend it a buffer), and latency-critical threads that must never call
// cudaMalloc/cudaFree, which can block and synchronise the whole device. This
// file gives them obn_bitlinear_forward_noalloc, whose scratch (int8
// activations, per-token scales and code sums) lives in one fixed device array
// below instead.
//
// The array is kNoAllocBytes (1 MiB + 32 KiB) on every device that loads the
// library, for the life of the process. It is shared by every call on a device
// and keeps the previous call's contents; nothing in it has to start at zero,
// because the quantize kernel writes every byte the matmul later reads. Calls
// that overlap on the GPU (two streams, or two threads) race on it.
#include <cstdio>
#include <mutex>

#include "../../include/obn.h"

namespace obn {
int report_error(int code, const char* message);
}  // namespace obn

namespace {

constexpr size_t kNoAllocActBytes = size_t(1) << 20;  // n * in_dim int8 activations
constexpr int kNoAllocMaxTokens = 4096;                // scales + code sums, 4 B each
constexpr size_t kNoAllocBytes = kNoAllocActBytes + 2 * sizeof(float) * kNoAllocMaxTokens;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// In host code g_noalloc_scratch names a host-side stand-in, not device memory:
// each device's address is looked up once, with that device current.
constexpr int kMaxDevices = 64;
struct DeviceScratch {
  std::once_flag once;
  void* ptr = nullptr;
  cudaError_t err = cudaSuccess;
};
DeviceScratch g_scratch[kMaxDevices];

}  // namespace

extern "C" int obn_bitlinear_forward_noalloc(const obn_bitlinear* layer, const float* x, int n,
                                             float* y, void* stream) {
  if (!layer) return obn::report_error(OBN_ERR_INVALID_ARGUMENT, "layer is NULL");
  if (n <= 0) return obn::report_error(OBN_ERR_INVALID_ARGUMENT, "n must be positive");
  const size_t act = static_cast<size_t>(n) * obn_bitlinear_in_dim(layer);
  if (act > kNoAllocActBytes || n > kNoAllocMaxTokens) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "obn_bitlinear_forward_noalloc: n=%d x in_dim=%d needs %zu activation bytes; the "
             "fixed scratch holds at most %zu bytes and %d tokens",
             n, obn_bitlinear_in_dim(layer), act, kNoAllocActBytes, kNoAllocMaxTokens);
    return obn::report_error(OBN_ERR_UNSUPPORTED, msg);
  }
  if (obn_bitlinear_workspace_bytes(layer, n) > kNoAllocBytes) {
    char msg[192];
    snprintf(msg, sizeof(msg),
             "obn_bitlinear_forward_noalloc: n=%d needs %zu scratch bytes; the fixed scratch "
             "holds %zu",
             n, obn_bitlinear_workspace_bytes(layer, n), kNoAllocBytes);
    return obn::report_error(OBN_ERR_UNSUPPORTED, msg);
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return obn::report_error(OBN_ERR_NO_DEVICE, "obn_bitlinear_forward_noalloc: no usable device");
  DeviceScratch& d = g_scratch[dev];
  std::call_once(d.once, [&d] { d.err = cudaGetSymbolAddress(&d.ptr, g_noalloc_scratch); });
  if (d.err != cudaSuccess || !d.ptr) {
    char msg[256];
    snprintf(msg, sizeof(msg), "obn_bitlinear_forward_noalloc: cudaGetSymbolAddress failed (%s)",
             cudaGetErrorString(d.err));
    return obn::report_error(OBN_ERR_CUDA, msg);
  }
  return obn_bitlinear_forward(layer, x, n, y, d.ptr, kNoAllocBytes, stream);
}
