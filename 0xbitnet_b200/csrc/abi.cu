// abi.cu — the extern "C" surface declared in include/obn.h.
//
// Host-side BitLinear: validation, the one-time repack of I2_S weights into the
// T16 device layout (layout.cuh), workspace partitioning and kernel dispatch.
// Error handling follows the reference's C ABI: a status return plus a
// thread-local message (packages/rust/crates/oxbitnet-ffi/src/lib.rs:31-46).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/obn.h"
#include "gemm.h"
#include "kernels.h"
#include "layout.cuh"
#include "lmhead.h"
#include "attention.h"

struct obn_bitlinear {
  int device = 0;
  int in_dim = 0;   // K
  int out_dim = 0;  // output features of the forward
  int rows = 0;     // weight rows the matmul computes (2 * out_dim when gated)
  int gated = 0;    // merged gate|up FFN projection: forward = act(gate) * up
  int act = 0;      // gated activation: 0 = ReLU^2, 1 = SiLU
  int m_pad = 0;
  float eps = 1e-5f;
  uint8_t* w = nullptr;     // T16 layout, m_pad * K / 4 bytes
  float* s_w = nullptr;     // [m_pad]
  float* norm = nullptr;    // [K] or null
};

namespace {

thread_local std::string g_error;
thread_local bool g_has_error = false;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  g_has_error = true;
  return code;
}

void clear_error() { g_has_error = false; }

int cuda_fail(cudaError_t e, const char* what) {
  return fail(OBN_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

int check_device(int dev) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    return fail(OBN_ERR_NO_DEVICE, "no CUDA device available (%s)",
                e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
  if (dev < 0 || dev >= count) return fail(OBN_ERR_INVALID_ARGUMENT, "device %d out of range", dev);
  int major = 0;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  if (major != 10)
    return fail(OBN_ERR_NO_DEVICE, "device %d is sm_%d x; libobn is built for sm_100a only", dev,
                major);
  return OBN_OK;
}

int check_dims(int in_dim, int out_dim) {
  if (in_dim <= 0 || out_dim <= 0)
    return fail(OBN_ERR_INVALID_ARGUMENT, "in_dim and out_dim must be positive (got %d, %d)",
                in_dim, out_dim);
  if (in_dim % obn::kBlockK != 0)
    return fail(OBN_ERR_UNSUPPORTED,
                "in_dim %d is not a multiple of 128 (the I2_S block interleave needs whole blocks)",
                in_dim);
  return OBN_OK;
}

obn::WeightView view(const obn_bitlinear* L) {
  return obn::WeightView{L->w, L->s_w, L->in_dim, L->rows, L->m_pad};
}

void free_layer(obn_bitlinear* L) {
  if (!L) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(L->device);
  cudaFree(L->w);
  cudaFree(L->s_w);
  cudaFree(L->norm);
  cudaSetDevice(prev);
  delete L;
}

// Allocates the layer on the current device and fills its scale table
// (scales_dev: device [out_dim] or null with host_scale used for every row).
int alloc_layer(int in_dim, int out_dim, float eps, obn_bitlinear** out) {
  auto* L = new obn_bitlinear;
  cudaGetDevice(&L->device);
  L->in_dim = in_dim;
  L->out_dim = out_dim;
  L->rows = out_dim;
  L->m_pad = obn::round_up(out_dim, obn::kTileRows);
  L->eps = eps;
  const size_t wbytes = static_cast<size_t>(L->m_pad) * in_dim / 4;
  cudaError_t e = cudaMalloc(&L->w, wbytes);
  if (e == cudaSuccess) e = cudaMalloc(&L->s_w, sizeof(float) * L->m_pad);
  if (e != cudaSuccess) {
    free_layer(L);
    cudaGetLastError();
    return fail(OBN_ERR_OUT_OF_MEMORY, "cudaMalloc of %zu weight bytes failed", wbytes);
  }
  *out = L;
  return OBN_OK;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int check_layer(const obn_bitlinear* L) {
  if (!L) return fail(OBN_ERR_INVALID_ARGUMENT, "layer is NULL");
  return OBN_OK;
}

// A gated layer whose n-token forward runs the dp4a GEMV (not the single-token
// kernel, not the tensor-core GEMM): only then are the interleaved gate|up rows
// stored in the workspace before k_act_mul forms act(gate) * up.
bool gated_gemv_path(const obn_bitlinear* L, int n) {
  if (!L->gated) return false;
  if (n == 1 && L->in_dim <= obn::kGemvMaxK) return false;
  return !obn::mma_gemv_supported(view(L), n) && !obn::gemm_supported(view(L), n);
}

// The matmul after the quantize pass for n tokens: the warp-MMA decode kernel
// (2..32 tokens), the tcgen05 GEMM, or the dp4a GEMV.
cudaError_t run_matmul(const obn_bitlinear* L, const int8_t* q, const float* sc,
                       const int32_t* qs, int n, float* y, int32_t* acc, int order,
                       cudaStream_t s, bool* unsupported) {
  *unsupported = false;
  if (obn::mma_gemv_supported(view(L), n))
    return obn::launch_mma_gemv(view(L), q, sc, qs, n, y, acc, order, s);
  if (obn::gemm_supported(view(L), n))
    return obn::launch_gemm(view(L), q, sc, qs, n, y, acc, order, s);
  if (L->in_dim <= obn::kGemvMaxK && !(order & obn::kOutGated))
    return obn::launch_gemv(view(L), q, sc, qs, n, y, acc, order, s);
  *unsupported = true;
  return cudaSuccess;
}

}  // namespace

namespace obn {
// Lets other translation units of the library report through the same
// thread-local error slot as the entry points in this file.
int report_error(int code, const char* message) { return fail(code, "%s", message); }
}  // namespace obn

extern "C" {

int obn_version(void) { return 100; }

const char* obn_error_message(void) { return g_has_error ? g_error.c_str() : nullptr; }

int obn_bitlinear_load_i2s(const uint8_t* i2s_tensor, size_t nbytes, int in_dim, int out_dim,
                           const float* norm_weight, float eps, int device,
                           obn_bitlinear** out_layer) {
  clear_error();
  if (!i2s_tensor || !out_layer) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  *out_layer = nullptr;
  if (int rc = check_dims(in_dim, out_dim)) return rc;
  const size_t packed = static_cast<size_t>(out_dim) * in_dim / 4;
  if (nbytes < packed + 32)  // loader.rs:109-110: ceil(n/4) + 32 bytes
    return fail(OBN_ERR_INVALID_ARGUMENT,
                "I2_S tensor of %dx%d needs %zu bytes (packed + 32-byte scale), got %zu", out_dim,
                in_dim, packed + 32, nbytes);
  if (int rc = check_device(device)) return rc;
  DeviceGuard g(device);
  float scale;  // loader.rs:129-131: first f32 of the trailing 32 bytes
  std::memcpy(&scale, i2s_tensor + packed, sizeof(float));

  obn_bitlinear* L = nullptr;
  if (int rc = alloc_layer(in_dim, out_dim, eps, &L)) return rc;
  uint8_t* staging = nullptr;
  cudaError_t e = cudaMalloc(&staging, packed);
  if (e != cudaSuccess) {
    free_layer(L);
    cudaGetLastError();
    return fail(OBN_ERR_OUT_OF_MEMORY, "cudaMalloc of %zu staging bytes failed", packed);
  }
  std::vector<float> table(L->m_pad, 0.0f);
  for (int m = 0; m < out_dim; ++m) table[m] = scale;  // loader.rs:132-136 replication
  e = cudaMemcpy(staging, i2s_tensor, packed, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = obn::launch_repack_i2s(staging, L->w, out_dim, in_dim, L->m_pad, 0);
  if (e == cudaSuccess)
    e = cudaMemcpy(L->s_w, table.data(), sizeof(float) * L->m_pad, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && norm_weight) {
    e = cudaMalloc(&L->norm, sizeof(float) * in_dim);
    if (e == cudaSuccess)
      e = cudaMemcpy(L->norm, norm_weight, sizeof(float) * in_dim, cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(staging);
  if (e != cudaSuccess) {
    free_layer(L);
    return cuda_fail(e, "loading I2_S tensor");
  }
  *out_layer = L;
  return OBN_OK;
}

int obn_bitlinear_load_i2s_concat(int count, const uint8_t* const* tensors, const size_t* nbytes,
                                  const int* out_dims, int in_dim, const float* norm_weight,
                                  float eps, int device, obn_bitlinear** out_layer) {
  clear_error();
  if (!tensors || !nbytes || !out_dims || !out_layer)
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  *out_layer = nullptr;
  if (count <= 0 || count > 64) return fail(OBN_ERR_INVALID_ARGUMENT, "count %d out of range", count);
  const size_t row_bytes = static_cast<size_t>(in_dim) / 4;
  long long total = 0;
  for (int t = 0; t < count; ++t) {
    if (!tensors[t]) return fail(OBN_ERR_INVALID_ARGUMENT, "tensor %d is NULL", t);
    if (out_dims[t] <= 0) return fail(OBN_ERR_INVALID_ARGUMENT, "out_dims[%d] = %d", t, out_dims[t]);
    const size_t packed = static_cast<size_t>(out_dims[t]) * row_bytes;
    if (nbytes[t] < packed + 32)  // loader.rs:109-110: ceil(n/4) + 32 bytes
      return fail(OBN_ERR_INVALID_ARGUMENT,
                  "I2_S tensor %d of %dx%d needs %zu bytes (packed + 32-byte scale), got %zu", t,
                  out_dims[t], in_dim, packed + 32, nbytes[t]);
    total += out_dims[t];
  }
  if (total > (1 << 29)) return fail(OBN_ERR_INVALID_ARGUMENT, "%lld rows too many", total);
  const int out_dim = static_cast<int>(total);
  if (int rc = check_dims(in_dim, out_dim)) return rc;
  if (int rc = check_device(device)) return rc;
  DeviceGuard g(device);
  obn_bitlinear* L = nullptr;
  if (int rc = alloc_layer(in_dim, out_dim, eps, &L)) return rc;
  uint8_t* staging = nullptr;
  cudaError_t e = cudaMalloc(&staging, static_cast<size_t>(out_dim) * row_bytes);
  if (e != cudaSuccess) {
    free_layer(L);
    cudaGetLastError();
    return fail(OBN_ERR_OUT_OF_MEMORY, "cudaMalloc of staging bytes failed");
  }
  std::vector<float> table(L->m_pad, 0.0f);
  size_t row0 = 0;
  for (int t = 0; t < count && e == cudaSuccess; ++t) {
    const size_t packed = static_cast<size_t>(out_dims[t]) * row_bytes;
    float scale;  // loader.rs:129-131: first f32 of the trailing 32 bytes
    std::memcpy(&scale, tensors[t] + packed, sizeof(float));
    for (int m = 0; m < out_dims[t]; ++m) table[row0 + m] = scale;
    e = cudaMemcpy(staging + row0 * row_bytes, tensors[t], packed, cudaMemcpyHostToDevice);
    row0 += out_dims[t];
  }
  if (e == cudaSuccess) e = obn::launch_repack_i2s(staging, L->w, out_dim, in_dim, L->m_pad, 0);
  if (e == cudaSuccess)
    e = cudaMemcpy(L->s_w, table.data(), sizeof(float) * L->m_pad, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && norm_weight) {
    e = cudaMalloc(&L->norm, sizeof(float) * in_dim);
    if (e == cudaSuccess)
      e = cudaMemcpy(L->norm, norm_weight, sizeof(float) * in_dim, cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(staging);
  if (e != cudaSuccess) {
    free_layer(L);
    return cuda_fail(e, "loading concatenated I2_S tensors");
  }
  *out_layer = L;
  return OBN_OK;
}

int obn_bitlinear_set_activation(obn_bitlinear* layer, int act) {
  clear_error();
  if (int rc = check_layer(layer)) return rc;
  if (!layer->gated) return fail(OBN_ERR_INVALID_ARGUMENT, "only a gated layer has an activation");
  if (act != 0 && act != 1) return fail(OBN_ERR_INVALID_ARGUMENT, "activation %d is not 0 or 1", act);
  layer->act = act;
  return OBN_OK;
}

int obn_activation(const float* x, size_t count, int act, float* y, void* stream) {
  clear_error();
  if ((!x || !y) && count) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (act != 0 && act != 1) return fail(OBN_ERR_INVALID_ARGUMENT, "activation %d is not 0 or 1", act);
  cudaError_t e = obn::launch_act(x, count, act, y, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "activation launch");
  return OBN_OK;
}

int obn_bitlinear_load_i2s_gated(const uint8_t* gate_i2s, size_t gate_bytes,
                                 const uint8_t* up_i2s, size_t up_bytes, int in_dim, int out_dim,
                                 const float* norm_weight, float eps, int device,
                                 obn_bitlinear** out_layer) {
  clear_error();
  if (!gate_i2s || !up_i2s || !out_layer)
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  *out_layer = nullptr;
  if (int rc = check_dims(in_dim, out_dim)) return rc;
  if (out_dim > (1 << 29)) return fail(OBN_ERR_INVALID_ARGUMENT, "out_dim %d too large", out_dim);
  const size_t row_bytes = static_cast<size_t>(in_dim) / 4;
  const size_t packed = static_cast<size_t>(out_dim) * row_bytes;
  if (gate_bytes < packed + 32 || up_bytes < packed + 32)
    return fail(OBN_ERR_INVALID_ARGUMENT,
                "each I2_S tensor of %dx%d needs %zu bytes (packed + 32-byte scale), got %zu and "
                "%zu",
                out_dim, in_dim, packed + 32, gate_bytes, up_bytes);
  if (int rc = check_device(device)) return rc;
  DeviceGuard g(device);
  float gscale, uscale;  // loader.rs:129-131
  std::memcpy(&gscale, gate_i2s + packed, sizeof(float));
  std::memcpy(&uscale, up_i2s + packed, sizeof(float));
  const int rows = 2 * out_dim;
  obn_bitlinear* L = nullptr;
  if (int rc = alloc_layer(in_dim, rows, eps, &L)) return rc;
  L->out_dim = out_dim;
  L->gated = 1;
  // Row 2i = gate row i, row 2i + 1 = up row i: a gate row and its up row always
  // share a tile, a subtile and a split-K owner range.
  std::vector<uint8_t> merged(2 * packed);
  for (int i = 0; i < out_dim; ++i) {
    std::memcpy(&merged[(2 * static_cast<size_t>(i)) * row_bytes], gate_i2s + i * row_bytes,
                row_bytes);
    std::memcpy(&merged[(2 * static_cast<size_t>(i) + 1) * row_bytes], up_i2s + i * row_bytes,
                row_bytes);
  }
  std::vector<float> table(L->m_pad, 0.0f);
  for (int i = 0; i < out_dim; ++i) {
    table[2 * i] = gscale;
    table[2 * i + 1] = uscale;
  }
  uint8_t* staging = nullptr;
  cudaError_t e = cudaMalloc(&staging, merged.size());
  if (e != cudaSuccess) {
    free_layer(L);
    cudaGetLastError();
    return fail(OBN_ERR_OUT_OF_MEMORY, "cudaMalloc of %zu staging bytes failed", merged.size());
  }
  e = cudaMemcpy(staging, merged.data(), merged.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = obn::launch_repack_i2s(staging, L->w, rows, in_dim, L->m_pad, 0);
  if (e == cudaSuccess)
    e = cudaMemcpy(L->s_w, table.data(), sizeof(float) * L->m_pad, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && norm_weight) {
    e = cudaMalloc(&L->norm, sizeof(float) * in_dim);
    if (e == cudaSuccess)
      e = cudaMemcpy(L->norm, norm_weight, sizeof(float) * in_dim, cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(staging);
  if (e != cudaSuccess) {
    free_layer(L);
    return cuda_fail(e, "loading gated I2_S tensors");
  }
  *out_layer = L;
  return OBN_OK;
}

int obn_bitlinear_create(const void* packed_dev, const float* scales_dev, const float* norm_dev,
                         float eps, int in_dim, int out_dim, void* stream,
                         obn_bitlinear** out_layer) {
  clear_error();
  if (!packed_dev || !scales_dev || !out_layer)
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  *out_layer = nullptr;
  if (int rc = check_dims(in_dim, out_dim)) return rc;
  if (!aligned(packed_dev, 16))
    return fail(OBN_ERR_INVALID_ARGUMENT, "packed weights must be 16-byte aligned");
  int dev = 0;
  cudaGetDevice(&dev);
  if (int rc = check_device(dev)) return rc;
  auto s = static_cast<cudaStream_t>(stream);
  obn_bitlinear* L = nullptr;
  if (int rc = alloc_layer(in_dim, out_dim, eps, &L)) return rc;
  cudaError_t e = obn::launch_repack_i2s(static_cast<const uint8_t*>(packed_dev), L->w, out_dim,
                                         in_dim, L->m_pad, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(L->s_w, 0, sizeof(float) * L->m_pad, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(L->s_w, scales_dev, sizeof(float) * out_dim, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess && norm_dev) {
    e = cudaMalloc(&L->norm, sizeof(float) * in_dim);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(L->norm, norm_dev, sizeof(float) * in_dim, cudaMemcpyDeviceToDevice, s);
  }
  if (e != cudaSuccess) {
    free_layer(L);
    return cuda_fail(e, "creating BitLinear");
  }
  *out_layer = L;
  return OBN_OK;
}

int obn_bitlinear_create_gated(const void* gate_packed_dev, const float* gate_scales_dev,
                               const void* up_packed_dev, const float* up_scales_dev,
                               const float* norm_dev, float eps, int in_dim, int out_dim,
                               void* stream, obn_bitlinear** out_layer) {
  clear_error();
  if (!gate_packed_dev || !gate_scales_dev || !up_packed_dev || !up_scales_dev || !out_layer)
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  *out_layer = nullptr;
  if (int rc = check_dims(in_dim, out_dim)) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  if (int rc = check_device(dev)) return rc;
  auto s = static_cast<cudaStream_t>(stream);
  const size_t rb = static_cast<size_t>(in_dim) / 4;
  obn_bitlinear* L = nullptr;
  if (int rc = alloc_layer(in_dim, 2 * out_dim, eps, &L)) return rc;
  L->out_dim = out_dim;
  L->gated = 1;
  uint8_t* staging = nullptr;
  cudaError_t e = cudaMalloc(&staging, 2 * rb * out_dim);
  if (e != cudaSuccess) {
    free_layer(L);
    cudaGetLastError();
    return fail(OBN_ERR_OUT_OF_MEMORY, "cudaMalloc of staging bytes failed");
  }
  // rows 2i <- gate row i, 2i + 1 <- up row i; the same for the scale table
  e = cudaMemcpy2DAsync(staging, 2 * rb, gate_packed_dev, rb, rb, out_dim,
                        cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpy2DAsync(staging + rb, 2 * rb, up_packed_dev, rb, rb, out_dim,
                          cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess)
    e = obn::launch_repack_i2s(staging, L->w, 2 * out_dim, in_dim, L->m_pad, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(L->s_w, 0, sizeof(float) * L->m_pad, s);
  if (e == cudaSuccess)
    e = cudaMemcpy2DAsync(L->s_w, 2 * sizeof(float), gate_scales_dev, sizeof(float),
                          sizeof(float), out_dim, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpy2DAsync(L->s_w + 1, 2 * sizeof(float), up_scales_dev, sizeof(float),
                          sizeof(float), out_dim, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess && norm_dev) {
    e = cudaMalloc(&L->norm, sizeof(float) * in_dim);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(L->norm, norm_dev, sizeof(float) * in_dim, cudaMemcpyDeviceToDevice, s);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // the staging rows are read by then
  cudaFree(staging);
  if (e != cudaSuccess) {
    free_layer(L);
    return cuda_fail(e, "creating gated BitLinear");
  }
  *out_layer = L;
  return OBN_OK;
}

void obn_bitlinear_free(obn_bitlinear* layer) { free_layer(layer); }

int obn_bitlinear_in_dim(const obn_bitlinear* layer) { return layer ? layer->in_dim : 0; }
int obn_bitlinear_out_dim(const obn_bitlinear* layer) { return layer ? layer->out_dim : 0; }
int obn_bitlinear_rows(const obn_bitlinear* layer) { return layer ? layer->rows : 0; }

size_t obn_bitlinear_workspace_bytes(const obn_bitlinear* layer, int n) {
  if (!layer || n <= 0) return 0;
  // interleaved gate|up outputs before the activation: only the dp4a GEMV path of
  // a gated layer stores them (the single-token kernel and the tensor-core GEMM
  // epilogues write act(gate) * up straight to y)
  const size_t pre = gated_gemv_path(layer, n)
                         ? align256(sizeof(float) * n * static_cast<size_t>(layer->rows))
                         : 0;
  return align256(static_cast<size_t>(n) * layer->in_dim) + 2 * align256(sizeof(float) * n) + pre;
}

int obn_ternary_matmul(const obn_bitlinear* layer, const int8_t* q, const float* scales,
                       const int32_t* qsum, int n, float* y, void* stream) {
  clear_error();
  if (int rc = check_layer(layer)) return rc;
  if (!q || !scales || !qsum || !y) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (n <= 0) return fail(OBN_ERR_INVALID_ARGUMENT, "n must be positive (got %d)", n);
  if (!aligned(q, 16)) return fail(OBN_ERR_INVALID_ARGUMENT, "q must be 16-byte aligned");
  const int order = n == 1 ? obn::kOrderGemv : obn::kOrderGemm;
  bool unsupported = false;
  const cudaError_t e = run_matmul(layer, q, scales, qsum, n, y, nullptr, order,
                                   static_cast<cudaStream_t>(stream), &unsupported);
  if (unsupported)
    return fail(OBN_ERR_UNSUPPORTED, "in_dim %d exceeds the kernels' limit", layer->in_dim);
  if (e != cudaSuccess) return cuda_fail(e, "ternary matmul launch");
  return OBN_OK;
}

int obn_ternary_acc(const obn_bitlinear* layer, const int8_t* q, const int32_t* qsum, int n,
                    int32_t* acc, void* stream) {
  clear_error();
  if (int rc = check_layer(layer)) return rc;
  if (!q || !qsum || !acc) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (n <= 0) return fail(OBN_ERR_INVALID_ARGUMENT, "n must be positive (got %d)", n);
  if (!aligned(q, 16)) return fail(OBN_ERR_INVALID_ARGUMENT, "q must be 16-byte aligned");
  bool unsupported = false;
  const cudaError_t e = run_matmul(layer, q, nullptr, qsum, n, nullptr, acc, obn::kOrderGemm,
                                   static_cast<cudaStream_t>(stream), &unsupported);
  if (unsupported)
    return fail(OBN_ERR_UNSUPPORTED, "in_dim %d exceeds the kernels' limit", layer->in_dim);
  if (e != cudaSuccess) return cuda_fail(e, "ternary acc launch");
  return OBN_OK;
}

int obn_rmsnorm_quantize(const float* x, const float* norm_weight, float eps, int n, int d,
                         int8_t* q, float* scales, int32_t* qsum, void* stream) {
  clear_error();
  if (!x || !q || !scales) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (n <= 0 || d <= 0 || d % 4 != 0)
    return fail(OBN_ERR_INVALID_ARGUMENT, "need n > 0 and d > 0 with d %% 4 == 0 (got %d, %d)", n,
                d);
  if (!aligned(x, 16) || !aligned(q, 4) || (norm_weight && !aligned(norm_weight, 16)))
    return fail(OBN_ERR_INVALID_ARGUMENT, "x / norm_weight must be 16-byte and q 4-byte aligned");
  cudaError_t e = obn::launch_rmsnorm_quant(x, norm_weight, eps, n, d, q, scales, qsum,
                                            static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm_quantize launch");
  return OBN_OK;
}

int obn_rmsnorm(const float* x, const float* w, float eps, int n, int d, float* y, void* stream) {
  clear_error();
  if (!x || !w || !y) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (n <= 0 || d <= 0) return fail(OBN_ERR_INVALID_ARGUMENT, "need n > 0 and d > 0");
  cudaError_t e = obn::launch_rmsnorm(x, w, eps, n, d, y, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm launch");
  return OBN_OK;
}

namespace {
int forward_impl(const obn_bitlinear* layer, const float* x, int n, float* y, void* workspace,
                 size_t workspace_bytes, void* stream, int accumulate);
}  // namespace

int obn_bitlinear_forward(const obn_bitlinear* layer, const float* x, int n, float* y,
                          void* workspace, size_t workspace_bytes, void* stream) {
  return forward_impl(layer, x, n, y, workspace, workspace_bytes, stream, 0);
}

int obn_bitlinear_forward_residual(const obn_bitlinear* layer, const float* x, int n, float* y,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (layer && layer->gated)
    return fail(OBN_ERR_UNSUPPORTED, "the residual forward does not take a gated FFN layer");
  if (x && y && x == y)
    return fail(OBN_ERR_INVALID_ARGUMENT, "the residual forward needs y distinct from x");
  return forward_impl(layer, x, n, y, workspace, workspace_bytes, stream, obn::kOutAccumulate);
}

}  // extern "C"

namespace {
int forward_impl(const obn_bitlinear* layer, const float* x, int n, float* y, void* workspace,
                 size_t workspace_bytes, void* stream, int accumulate) {
  clear_error();
  if (int rc = check_layer(layer)) return rc;
  if (!x || !y || !workspace) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (n <= 0) return fail(OBN_ERR_INVALID_ARGUMENT, "n must be positive (got %d)", n);
  const size_t need = obn_bitlinear_workspace_bytes(layer, n);
  if (workspace_bytes < need)
    return fail(OBN_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is smaller than the %zu needed",
                workspace_bytes, need);
  if (!aligned(workspace, 256) || !aligned(x, 16))
    return fail(OBN_ERR_INVALID_ARGUMENT, "workspace must be 256-byte and x 16-byte aligned");
  auto* base = static_cast<uint8_t*>(workspace);
  auto* q = reinterpret_cast<int8_t*>(base);
  auto* sc = reinterpret_cast<float*>(base + align256(static_cast<size_t>(n) * layer->in_dim));
  auto* qs = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(sc) + align256(sizeof(float) * n));
  // Gated layers on the dp4a GEMV path (2-3 tokens): the matmul writes the
  // interleaved [n, 2*out_dim] gate|up outputs here and act(gate) * up goes to y.
  // The single-token kernel and the tensor-core GEMMs write act(gate) * up to y
  // from their epilogues.
  float* ym = gated_gemv_path(layer, n) ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(qs) +
                                                                  align256(sizeof(float) * n))
                                       : y;
  auto s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (n == 1 && layer->in_dim <= obn::kGemvMaxK) {  // whole BitLinear in one kernel
    // (a gated layer's activation included: the kernel writes y directly)
    e = obn::launch_bitlinear_n1(view(layer), layer->norm, layer->eps, x,
                                 layer->gated ? y : ym, s, accumulate,
                                 layer->gated ? layer->act : -1);
    if (e != cudaSuccess) return cuda_fail(e, "bitlinear (n=1) launch");
    return OBN_OK;
  } else if (obn::bitlinear_mma_supported(view(layer), n)) {  // few tokens, many rows: one kernel
    e = obn::launch_bitlinear_mma(view(layer), layer->norm, layer->eps, x, n, y, accumulate,
                                  layer->gated ? layer->act : -1, s);
    if (e != cudaSuccess) return cuda_fail(e, "bitlinear (fused few-token) launch");
    return OBN_OK;
  } else {
    e = obn::launch_rmsnorm_quant(x, layer->norm, layer->eps, n, layer->in_dim, q, sc, qs, s);
    if (e != cudaSuccess) return cuda_fail(e, "rmsnorm_quantize launch");
    const int order =
        (n == 1 ? obn::kOrderGemv : obn::kOrderGemm) | accumulate;  // bitlinear.rs:90-94
    bool unsupported = false;
    if (layer->gated && !gated_gemv_path(layer, n)) {
      // the warp-MMA and GEMM epilogues form act(gate) * up themselves
      e = run_matmul(layer, q, sc, qs, n, y, nullptr,
                     order | obn::kOutGated | (layer->act ? obn::kOutSilu : 0), s, &unsupported);
      if (e != cudaSuccess) return cuda_fail(e, "ternary matmul launch");
      return OBN_OK;
    }
    e = run_matmul(layer, q, sc, qs, n, ym, nullptr, order, s, &unsupported);
    if (unsupported)
      return fail(OBN_ERR_UNSUPPORTED, "in_dim %d exceeds the kernels' limit", layer->in_dim);
    if (e != cudaSuccess) return cuda_fail(e, "ternary matmul launch");
  }
  if (layer->gated) {  // ffn.rs:70-79: activation.wgsl then elementwise.wgsl (multiply)
    e = obn::launch_act_mul(ym, n, layer->out_dim, layer->act, y, s);
    if (e != cudaSuccess) return cuda_fail(e, "act(gate) * up launch");
  }
  return OBN_OK;
}
}  // namespace

extern "C" {

int obn_bitlinear_forward_tp(const obn_bitlinear* layer, const float* x, int n, float* y_mc,
                             float* const* y_ranks, int world, int out_total, int col0,
                             void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (int rc = check_layer(layer)) return rc;
  if (!x || !workspace || (!y_mc && !y_ranks))
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (world < 1 || world > obn::kMaxGatherRanks)
    return fail(OBN_ERR_INVALID_ARGUMENT, "world must be in 1..%d (got %d)", obn::kMaxGatherRanks,
                world);
  if (col0 < 0 || out_total <= 0 || static_cast<long long>(col0) + layer->out_dim > out_total)
    return fail(OBN_ERR_INVALID_ARGUMENT,
                "columns [%d, %d) do not fit an output of %d columns", col0,
                col0 + layer->out_dim, out_total);
  if (layer->gated)
    return fail(OBN_ERR_UNSUPPORTED, "the gathered forward does not take a gated FFN layer");
  if (n < obn::kGemmMinTokens || !obn::gemm_supported(view(layer), n))
    return fail(OBN_ERR_UNSUPPORTED, "the gathered forward needs n >= %d tokens (got %d)",
                obn::kGemmMinTokens, n);
  const size_t need = obn_bitlinear_workspace_bytes(layer, n);
  if (workspace_bytes < need)
    return fail(OBN_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is smaller than the %zu needed",
                workspace_bytes, need);
  if (!aligned(workspace, 256) || !aligned(x, 16))
    return fail(OBN_ERR_INVALID_ARGUMENT, "workspace must be 256-byte and x 16-byte aligned");
  obn::GatherOut go;
  go.mc = y_mc;
  go.world = world;
  go.ldy = out_total;
  go.col0 = col0;
  if (!y_mc)
    for (int r = 0; r < world; ++r) {
      if (!y_ranks[r]) return fail(OBN_ERR_INVALID_ARGUMENT, "y_ranks[%d] is null", r);
      if (!aligned(y_ranks[r], 4))
        return fail(OBN_ERR_INVALID_ARGUMENT, "y_ranks[%d] is not 4-byte aligned", r);
      go.ranks[r] = y_ranks[r];
    }
  else if (!aligned(y_mc, 4))
    return fail(OBN_ERR_INVALID_ARGUMENT, "y_mc is not 4-byte aligned");
  go.vec4 = out_total % 4 == 0 && col0 % 4 == 0 && layer->out_dim % 4 == 0;
  if (y_mc) go.vec4 = go.vec4 && aligned(y_mc, 16);
  else
    for (int r = 0; r < world; ++r) go.vec4 = go.vec4 && aligned(y_ranks[r], 16);
  auto* base = static_cast<uint8_t*>(workspace);
  auto* q = reinterpret_cast<int8_t*>(base);
  auto* sc = reinterpret_cast<float*>(base + align256(static_cast<size_t>(n) * layer->in_dim));
  auto* qs = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(sc) + align256(sizeof(float) * n));
  auto s = static_cast<cudaStream_t>(stream);
  cudaError_t e = obn::launch_rmsnorm_quant(x, layer->norm, layer->eps, n, layer->in_dim, q, sc,
                                            qs, s);
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm_quantize launch");
  e = obn::launch_gemm_gather(view(layer), q, sc, qs, n, obn::kOrderGemm, go, s);
  if (e != cudaSuccess) return cuda_fail(e, "gathered ternary GEMM launch");
  return OBN_OK;
}

int obn_lm_head_f16(const void* embed, int vocab, int dim, const float* x,
                    const float* norm_weight, float eps, int n, float* logits, void* stream) {
  clear_error();
  if (!embed || !x || !logits) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (vocab <= 0 || dim <= 0 || n <= 0)
    return fail(OBN_ERR_INVALID_ARGUMENT, "need vocab, dim and n > 0 (got %d, %d, %d)", vocab,
                dim, n);
  if (dim % 8 != 0 || dim > 14336)
    return fail(OBN_ERR_UNSUPPORTED, "dim must be a multiple of 8 and at most 14336 (got %d)",
                dim);
  if (!aligned(embed, 16) || !aligned(x, 16) || (norm_weight && !aligned(norm_weight, 4)) ||
      !aligned(logits, 4))
    return fail(OBN_ERR_INVALID_ARGUMENT, "embed and x must be 16-byte aligned");
  int dev = 0;
  cudaGetDevice(&dev);
  if (int rc = check_device(dev)) return rc;
  cudaError_t e = obn::launch_lm_head_f16(embed, vocab, dim, x, norm_weight, eps, n, logits,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lm head launch");
  return OBN_OK;
}

size_t obn_lm_head_workspace_bytes(int n, int dim) {
  if (n <= 0 || dim <= 0) return 0;
  return obn::lm_head_tc_workspace_bytes(n, dim);
}

int obn_lm_head_f16_batched(const void* embed, int vocab, int dim, const float* x,
                            const float* norm_weight, float eps, int n, float* logits,
                            void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (!embed || !x || !logits || !workspace)
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (vocab <= 0 || dim <= 0 || n <= 0)
    return fail(OBN_ERR_INVALID_ARGUMENT, "need vocab, dim and n > 0 (got %d, %d, %d)", vocab,
                dim, n);
  if (dim % 64 != 0)
    return fail(OBN_ERR_UNSUPPORTED, "dim must be a multiple of 64 (got %d)", dim);
  if (workspace_bytes < obn::lm_head_tc_workspace_bytes(n, dim))
    return fail(OBN_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is smaller than the %zu needed",
                workspace_bytes, obn::lm_head_tc_workspace_bytes(n, dim));
  if (!aligned(embed, 16) || !aligned(workspace, 256) || !aligned(x, 4) || !aligned(logits, 4))
    return fail(OBN_ERR_INVALID_ARGUMENT, "embed 16-byte and workspace 256-byte aligned");
  int dev = 0;
  cudaGetDevice(&dev);
  if (int rc = check_device(dev)) return rc;
  cudaError_t e = obn::launch_lm_head_tc(embed, vocab, dim, x, norm_weight, eps, n, logits,
                                         workspace, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "batched lm head launch");
  return OBN_OK;
}

int obn_rope_kv_append(const float* qkv, int B, int n, int H, int Hkv, int head_dim, int pos,
                       float theta_base, float* q_out, void* k_cache, void* v_cache, int S_max,
                       void* stream) {
  clear_error();
  if (!qkv || !q_out || !k_cache || !v_cache)
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (B <= 0 || n <= 0 || H <= 0 || Hkv <= 0 || pos < 0 || S_max <= 0)
    return fail(OBN_ERR_INVALID_ARGUMENT, "sizes must be positive (pos >= 0)");
  if (head_dim != obn::kAttnHeadDim)
    return fail(OBN_ERR_UNSUPPORTED, "head_dim must be %d (got %d)", obn::kAttnHeadDim, head_dim);
  if (static_cast<long long>(pos) + n > S_max)
    return fail(OBN_ERR_INVALID_ARGUMENT, "positions %d..%d exceed the cache of %d", pos,
                pos + n - 1, S_max);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(qkv, 8) || !aligned(q_out, 8))
    return fail(OBN_ERR_INVALID_ARGUMENT, "caches must be 16-byte, qkv and q_out 8-byte aligned");
  cudaError_t e = obn::launch_rope_kv_append(
      qkv, B, n, H, Hkv, head_dim, pos, theta_base, q_out, static_cast<__half*>(k_cache),
      static_cast<__half*>(v_cache), S_max, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope / kv append launch");
  return OBN_OK;
}

size_t obn_attention_workspace_bytes(int B, int n, int H, int head_dim, int seq_len) {
  if (B <= 0 || n <= 0 || H <= 0 || head_dim <= 0 || seq_len <= 0) return 0;
  return obn::attention_workspace_bytes(B, n, H, head_dim, seq_len);
}

int obn_attention_decode(const float* q, const void* k_cache, const void* v_cache, int B, int n,
                         int H, int Hkv, int head_dim, int S_max, int seq_len, float scale,
                         float* out, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (!q || !k_cache || !v_cache || !out || !workspace)
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (B <= 0 || n <= 0 || H <= 0 || Hkv <= 0 || seq_len <= 0 || n > seq_len || seq_len > S_max)
    return fail(OBN_ERR_INVALID_ARGUMENT, "need 0 < n <= seq_len <= S_max (got %d, %d, %d)", n,
                seq_len, S_max);
  if (head_dim != obn::kAttnHeadDim)
    return fail(OBN_ERR_UNSUPPORTED, "head_dim must be %d (got %d)", obn::kAttnHeadDim, head_dim);
  const int G = H % Hkv == 0 ? H / Hkv : 0;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return fail(OBN_ERR_UNSUPPORTED, "H / Hkv must be 1, 2, 4 or 8 (got %d / %d)", H, Hkv);
  const size_t need = obn::attention_workspace_bytes(B, n, H, head_dim, seq_len);
  if (workspace_bytes < need)
    return fail(OBN_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is smaller than the %zu needed",
                workspace_bytes, need);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(workspace, 256) ||
      !aligned(q, 4) || !aligned(out, 4))
    return fail(OBN_ERR_INVALID_ARGUMENT, "caches must be 16-byte, workspace 256-byte aligned");
  cudaError_t e = obn::launch_attention(q, static_cast<const __half*>(k_cache),
                                        static_cast<const __half*>(v_cache), B, n, H, Hkv,
                                        head_dim, S_max, seq_len, scale, out, workspace,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return OBN_OK;
}

int obn_rope_kv_append_at(const float* qkv, int B, int n, int H, int Hkv, int head_dim,
                          const int* pos_dev, float theta_base, float* q_out, void* k_cache,
                          void* v_cache, int S_max, void* stream) {
  clear_error();
  if (!qkv || !q_out || !k_cache || !v_cache || !pos_dev)
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (B <= 0 || n <= 0 || H <= 0 || Hkv <= 0 || S_max <= 0 || n > S_max)
    return fail(OBN_ERR_INVALID_ARGUMENT, "sizes must be positive, n <= S_max");
  if (head_dim != obn::kAttnHeadDim)
    return fail(OBN_ERR_UNSUPPORTED, "head_dim must be %d (got %d)", obn::kAttnHeadDim, head_dim);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(qkv, 8) || !aligned(q_out, 8) ||
      !aligned(pos_dev, 4))
    return fail(OBN_ERR_INVALID_ARGUMENT, "caches must be 16-byte, qkv and q_out 8-byte aligned");
  cudaError_t e = obn::launch_rope_kv_append(
      qkv, B, n, H, Hkv, head_dim, 0, theta_base, q_out, static_cast<__half*>(k_cache),
      static_cast<__half*>(v_cache), S_max, static_cast<cudaStream_t>(stream), pos_dev);
  if (e != cudaSuccess) return cuda_fail(e, "rope / kv append launch");
  return OBN_OK;
}

int obn_attention_decode_at(const float* q, const void* k_cache, const void* v_cache, int B,
                            int n, int H, int Hkv, int head_dim, int S_max, const int* pos_dev,
                            float scale, float* out, void* workspace, size_t workspace_bytes,
                            void* stream) {
  clear_error();
  if (!q || !k_cache || !v_cache || !out || !workspace || !pos_dev)
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (B <= 0 || n <= 0 || H <= 0 || Hkv <= 0 || n > S_max)
    return fail(OBN_ERR_INVALID_ARGUMENT, "sizes must be positive, n <= S_max");
  if (head_dim != obn::kAttnHeadDim)
    return fail(OBN_ERR_UNSUPPORTED, "head_dim must be %d (got %d)", obn::kAttnHeadDim, head_dim);
  const int G = H % Hkv == 0 ? H / Hkv : 0;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return fail(OBN_ERR_UNSUPPORTED, "H / Hkv must be 1, 2, 4 or 8 (got %d / %d)", H, Hkv);
  const size_t need = obn::attention_workspace_bytes(B, n, H, head_dim, S_max);
  if (workspace_bytes < need)
    return fail(OBN_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is smaller than the %zu needed",
                workspace_bytes, need);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(workspace, 256) ||
      !aligned(q, 4) || !aligned(out, 4) || !aligned(pos_dev, 4))
    return fail(OBN_ERR_INVALID_ARGUMENT, "caches must be 16-byte, workspace 256-byte aligned");
  cudaError_t e = obn::launch_attention(q, static_cast<const __half*>(k_cache),
                                        static_cast<const __half*>(v_cache), B, n, H, Hkv,
                                        head_dim, S_max, S_max, scale, out, workspace,
                                        static_cast<cudaStream_t>(stream), pos_dev);
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return OBN_OK;
}

namespace {
int attention_rope_common(const float* qkv, void* k_cache, void* v_cache, int B, int H, int Hkv,
                          int head_dim, int S_max, int pos, const int* pos_dev, float theta_base,
                          float scale, float* out, void* workspace, size_t workspace_bytes,
                          void* stream) {
  if (!qkv || !k_cache || !v_cache || !out || !workspace)
    return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (B <= 0 || H <= 0 || Hkv <= 0 || S_max <= 0 || (!pos_dev && (pos < 0 || pos >= S_max)))
    return fail(OBN_ERR_INVALID_ARGUMENT, "need B, H, Hkv > 0 and 0 <= pos < S_max");
  if (head_dim != obn::kAttnHeadDim)
    return fail(OBN_ERR_UNSUPPORTED, "head_dim must be %d (got %d)", obn::kAttnHeadDim, head_dim);
  const int G = H % Hkv == 0 ? H / Hkv : 0;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return fail(OBN_ERR_UNSUPPORTED, "H / Hkv must be 1, 2, 4 or 8 (got %d / %d)", H, Hkv);
  const size_t need =
      obn::attention_workspace_bytes(B, 1, H, head_dim, pos_dev ? S_max : pos + 1);
  if (workspace_bytes < need)
    return fail(OBN_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is smaller than the %zu needed",
                workspace_bytes, need);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(workspace, 256) ||
      !aligned(qkv, 8) || !aligned(out, 4) || (pos_dev && !aligned(pos_dev, 4)))
    return fail(OBN_ERR_INVALID_ARGUMENT, "caches must be 16-byte, workspace 256-byte aligned");
  cudaError_t e = obn::launch_attention_rope(
      qkv, static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), B, H, Hkv, head_dim,
      S_max, pos, theta_base, scale, out, workspace, static_cast<cudaStream_t>(stream), pos_dev);
  if (e != cudaSuccess) return cuda_fail(e, "fused rope + attention launch");
  return OBN_OK;
}
}  // namespace

int obn_attention_decode_rope(const float* qkv, void* k_cache, void* v_cache, int B, int H,
                              int Hkv, int head_dim, int S_max, int pos, float theta_base,
                              float scale, float* out, void* workspace, size_t workspace_bytes,
                              void* stream) {
  clear_error();
  return attention_rope_common(qkv, k_cache, v_cache, B, H, Hkv, head_dim, S_max, pos, nullptr,
                               theta_base, scale, out, workspace, workspace_bytes, stream);
}

int obn_attention_decode_rope_at(const float* qkv, void* k_cache, void* v_cache, int B, int H,
                                 int Hkv, int head_dim, int S_max, const int* pos_dev,
                                 float theta_base, float scale, float* out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  clear_error();
  if (!pos_dev) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  return attention_rope_common(qkv, k_cache, v_cache, B, H, Hkv, head_dim, S_max, 0, pos_dev,
                               theta_base, scale, out, workspace, workspace_bytes, stream);
}

int obn_add(const float* a, const float* b, size_t count, float* y, void* stream) {
  clear_error();
  if (!a || !b || !y) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  cudaError_t e = obn::launch_add(a, b, count, y, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "add launch");
  return OBN_OK;
}

int obn_embed_f16(const void* table, int vocab, int dim, const int32_t* ids, int n, float* y,
                  void* stream) {
  clear_error();
  if (!table || !ids || !y) return fail(OBN_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (vocab <= 0 || dim <= 0 || n <= 0)
    return fail(OBN_ERR_INVALID_ARGUMENT, "vocab, dim and n must be positive");
  cudaError_t e =
      obn::launch_embed_f16(table, vocab, dim, ids, n, y, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "embedding launch");
  return OBN_OK;
}

int obn_bitlinear_export_i2s(const obn_bitlinear* layer, uint8_t* dst_dev, void* stream) {
  clear_error();
  if (int rc = check_layer(layer)) return rc;
  if (!dst_dev || !aligned(dst_dev, 16))
    return fail(OBN_ERR_INVALID_ARGUMENT, "destination must be non-null and 16-byte aligned");
  cudaError_t e = obn::launch_export_i2s(layer->w, dst_dev, layer->rows, layer->in_dim,
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "export launch");
  return OBN_OK;
}

int obn_check_device_errors(void) {
  clear_error();
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  uint32_t word = 0;
  e = obn::read_and_clear_dev_error(&word);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  if (word != 0)
    return fail(OBN_ERR_DEVICE_TIMEOUT, "%s (device error code %u)",
                word == 1u ? "a bounded device-side wait gave up"
                                                 : "a kernel was launched outside its geometry",
                word);
  return OBN_OK;
}

}  // extern "C"
