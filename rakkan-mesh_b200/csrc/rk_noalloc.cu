// rk_noalloc.cu — a matrix-vector product that allocates nothing.
//
// rk_matrix_mulvec needs device memory of its own: at rk_device_open the
// library cudaMallocs a staging area for the input vector, its Q8_0 form
// and the output. Some callers cannot let a library allocate like that: a
// node whose whole GPU memory is handed to one pool (the model's weights,
// KV caches and every scratch buffer reserved up front so that a stage can
// be admitted or refused by its size, as rakkan-mesh plans stages by
// memory), a sandboxed worker whose device memory is metered, or a caller
// that keeps cudaMalloc and its implicit device synchronisation off the
// per-token path. Such a caller already owns device buffers for the input
// and the output; what the product needs besides those is the quantized
// copy of the input (Q8_0 values, one scale and one sum per 32-block). This
// entry point keeps that scratch in a fixed array compiled into the
// library, so the call itself allocates nothing.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/rakkan_cuda.h"
#include "rk_matvec.cuh"

namespace {

// The quantized input: RK_NOALLOC_MAX_COLS int8 values, then one float
// scale and one int sum per 32-block. Every GPU that loads the library
// holds these 40 KiB until the process exits.
constexpr int kMaxCols = RK_NOALLOC_MAX_COLS;
constexpr size_t kQxBytes = kMaxCols;
constexpr size_t kXsBytes = sizeof(float) * (kMaxCols / 32);
constexpr size_t kXsumBytes = sizeof(int) * (kMaxCols / 32);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kQxBytes + kXsBytes + kXsumBytes];

// The array's device address on each device, looked up once per device
// (host code must not use the symbol itself as a device pointer).
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {};

}  // namespace

// Library internals the entry point reuses (rk_capi.cu).
namespace rk {
int internal_fail(int code, const char *msg);
int internal_matrix_view(const rk_matrix *m, int *device, int *rows, int *cols, int *fmt, const void **w,
                         const float **scales, void **stream, int **err_word, int *sms);
void internal_device_lock(const rk_matrix *m);
void internal_device_unlock(const rk_matrix *m);
int internal_check_dev_err(const rk_matrix *m);
}  // namespace rk

namespace {
// Holds the matrix's device mutex for the whole call: the call shares the
// device's stream (when given none) and its error word with every other
// entry point on that device.
struct DeviceLock {
  const rk_matrix *m;
  explicit DeviceLock(const rk_matrix *mm) : m(mm) { rk::internal_device_lock(m); }
  ~DeviceLock() { rk::internal_device_unlock(m); }
};
}  // namespace

// Looks up the scratch array's address on the current device (once).
static int scratch_address(int device, void **out) {
  if (device < 0 || device >= kMaxDevices) return rk::internal_fail(RK_ERR_ARGS, "noalloc: device index out of range");
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_scratch_addr[device]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      char msg[256];
      snprintf(msg, sizeof msg, "noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return rk::internal_fail(RK_ERR_CUDA, msg);
    }
    g_scratch_addr[device] = p;
  }
  *out = g_scratch_addr[device];
  return RK_OK;
}

extern "C" int rk_matrix_mulvec_noalloc(rk_matrix *m, const float *x_dev, float *out_dev, void *stream) {
  if (!m || !x_dev || !out_dev) return rk::internal_fail(RK_ERR_ARGS, "noalloc: null argument");
  int device, rows, cols, fmt, sms;
  const void *w;
  const float *scales;
  void *dev_stream;
  int *err_word;
  int rc = rk::internal_matrix_view(m, &device, &rows, &cols, &fmt, &w, &scales, &dev_stream, &err_word, &sms);
  if (rc) return rc;
  if (fmt != RK_FMT_Q8_0 && fmt != RK_FMT_Q4_0)
    return rk::internal_fail(RK_ERR_ARGS, "noalloc: only Q8_0 and Q4_0 matrices have a quantized-input scratch");
  if (cols > kMaxCols) {
    char msg[160];
    snprintf(msg, sizeof msg, "noalloc: %d columns exceed the fixed scratch of %d (RK_NOALLOC_MAX_COLS)", cols, kMaxCols);
    return rk::internal_fail(RK_ERR_TOO_BIG, msg);
  }
  DeviceLock lock(m);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return rk::internal_fail(RK_ERR_CUDA, "noalloc: cudaSetDevice failed");
  void *base = nullptr;
  if ((rc = scratch_address(device, &base))) return rc;
  unsigned char *b = static_cast<unsigned char *>(base);
  int8_t *qx = reinterpret_cast<int8_t *>(b);
  float *xs = reinterpret_cast<float *>(b + kQxBytes);
  int *xsum = reinterpret_cast<int *>(b + kQxBytes + kXsBytes);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : static_cast<cudaStream_t>(dev_stream);
  // The quantizer rewrites qx, xs and xsum for all `cols` before the matvec
  // reads them, so nothing in the array has to start at zero.
  e = rk::launch_quantize_act(x_dev, cols, nullptr, 0.0f, 0.0f, nullptr, qx, xs, xsum, st);
  if (e == cudaSuccess) {
    rk::MvArgs a{};
    a.fmt = fmt;
    a.cols = cols;
    a.epi = rk::EPI_STORE;
    a.qx = qx;
    a.xs = xs;
    a.xsum = xsum;
    a.x = x_dev;
    a.err = err_word;
    a.part[0].w = static_cast<const uint8_t *>(w);
    a.part[0].s = scales;
    a.part[0].out = out_dev;
    a.part[0].rows = rows;
    a.nparts = 1;
    e = rk::launch_matvec(a, sms, st);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof msg, "noalloc: %s", cudaGetErrorString(e));
    return rk::internal_fail(RK_ERR_CUDA, msg);
  }
  // The device error word, classified as every other entry point does
  // (an expired bounded wait, or an index a kernel refused).
  return rk::internal_check_dev_err(m);
}
