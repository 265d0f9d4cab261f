// rk_capi.cu — the C ABI of librakkan_cuda.so (include/rakkan_cuda.h).
//
// Host-side mirror of rakkan-mesh's internal/gpu API (Device, Matrix,
// Vectors, Arena, Batch: internal/gpu/device.go, batch.go), of the parts of
// internal/llm that drive it (Layer.toDevice, NewStage, Stage.ForwardMany,
// Head.Logits, Embed: internal/llm/model.go, gpustage.go) and of
// rakkan_tensor_v1's matmul (internal/sandbox/tensor.go:286-339).
//
// The library owns device memory and one CUDA stream per device. Every
// entry point is synchronous at the boundary and returns a status; errors
// latch per batch like gpu.Batch (batch.go:136-147). There is no host
// fallback: a failing CUDA call is an error.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <initializer_list>
#include <chrono>
#include <condition_variable>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/rakkan_cuda.h"
#include "rk_common.cuh"
#include "rk_gen.cuh"
#include "rk_layer.cuh"
#include "rk_matvec.cuh"
#include "rk_tensor.cuh"

using namespace rk;

// ---------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------
static thread_local std::string g_err = "";

static int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

static int cuda_fail(cudaError_t e, const char *what) {
  return fail(e == cudaErrorMemoryAllocation ? RK_ERR_NOMEM : RK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(call)                                         \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);  \
  } while (0)

extern "C" const char *rk_last_error(void) { return g_err.c_str(); }
extern "C" const char *rk_version(void) { return "rakkan-cuda 0.1 (sm_100a)"; }

// ---------------------------------------------------------------------------
// Devices
// ---------------------------------------------------------------------------
// A lock that, like Go's sync.Mutex, may be released by another call than
// the one that took it (a Batch holds its device from Begin to Submit).
struct DevLock {
  std::mutex m;
  std::condition_variable cv;
  bool held = false;
  void lock() {
    std::unique_lock<std::mutex> g(m);
    cv.wait(g, [&] { return !held; });
    held = true;
  }
  void unlock() {
    {
      std::lock_guard<std::mutex> g(m);
      held = false;
    }
    cv.notify_one();
  }
};

struct rk_device {
  int ordinal = 0;
  int sms = 148;
  cudaStream_t st = nullptr;
  DevLock mu;
  int64_t used = 0;
  int *err_dev = nullptr;  // device-side error word (kernels' bounded waits)
  // The MulVecs arena (device.go:769-793): input, its Q8_0 form, outputs.
  float *mv_x = nullptr, *mv_out = nullptr, *mv_xs = nullptr;
  int8_t *mv_qx = nullptr;
  int *mv_xsum = nullptr;
  float *pin_in = nullptr, *pin_out = nullptr;
  void *flush = nullptr;
  size_t flush_bytes = 0;
};

struct Guard {
  rk_device *d;
  explicit Guard(rk_device *dd) : d(dd) { d->mu.lock(); }
  ~Guard() { d->mu.unlock(); }
};

static int set_device(rk_device *d) {
  CK(cudaSetDevice(d->ordinal));
  return RK_OK;
}

// Reads and clears the device error word after a synchronisation.
static int check_dev_err(rk_device *d) {
  int e = 0;
  CK(cudaMemcpy(&e, d->err_dev, sizeof e, cudaMemcpyDeviceToHost));
  if (e != 0) {
    CK(cudaMemset(d->err_dev, 0, sizeof(int)));
    if (e == DEV_ERR_RANGE) return fail(RK_ERR_ARGS, "a kernel refused an out-of-range index (device error %d)", e);
    return fail(RK_ERR_TIMEOUT, "a kernel's bounded wait expired (device error %d)", e);
  }
  return RK_OK;
}

static int sync_dev(rk_device *d) {
  CK(cudaStreamSynchronize(d->st));
  return check_dev_err(d);
}

extern "C" int rk_device_count(int *n) {
  if (!n) return fail(RK_ERR_ARGS, "null argument");
  int c = 0;
  cudaError_t e = cudaGetDeviceCount(&c);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) c = 0;
  else if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  *n = c;
  return RK_OK;
}

extern "C" int rk_device_get_info(int index, rk_device_info *info) {
  if (!info) return fail(RK_ERR_ARGS, "null argument");
  cudaDeviceProp p;
  CK(cudaGetDeviceProperties(&p, index));
  memset(info, 0, sizeof *info);
  info->index = index;
  snprintf(info->name, sizeof info->name, "%s", p.name);
  info->memory = (int64_t)p.totalGlobalMem;
  info->sm_count = p.multiProcessorCount;
  info->cc_major = p.major;
  info->cc_minor = p.minor;
  info->exact = (p.major == 10 && p.minor == 0) ? 1 : 0;
  return RK_OK;
}

extern "C" int rk_device_best(int *index) {
  int n = 0;
  int rc = rk_device_count(&n);
  if (rc) return rc;
  int best = -1;
  int64_t mem = -1;
  for (int i = 0; i < n; i++) {
    rk_device_info info;
    if (rk_device_get_info(i, &info) == RK_OK && info.exact && info.memory > mem) {
      best = i;
      mem = info.memory;
    }
  }
  if (best < 0) return fail(RK_ERR_ARGS, "no sm_100 device");
  *index = best;
  return RK_OK;
}

extern "C" int rk_device_open(int index, rk_device **out) {
  if (!out) return fail(RK_ERR_ARGS, "null argument");
  rk_device_info info;
  int rc = rk_device_get_info(index, &info);
  if (rc) return rc;
  if (!info.exact) return fail(RK_ERR_ARGS, "device %d (%s) is not sm_100: the kernels are built for sm_100a", index, info.name);
  auto *d = new rk_device();
  d->ordinal = index;
  d->sms = info.sm_count;
  auto cleanup = [&](int code) {
    rk_device_close(d);
    return code;
  };
  if (cudaSetDevice(index) != cudaSuccess) return cleanup(fail(RK_ERR_CUDA, "cudaSetDevice(%d)", index));
  cudaError_t e = init_matvec_attributes();
  if (e == cudaSuccess) e = init_layer_attributes();
  if (e == cudaSuccess) e = init_tensor_attributes();
  if (e == cudaSuccess) e = init_mvmany_attributes();
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&d->err_dev, 2 * sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(d->err_dev, 0, 2 * sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&d->mv_x, sizeof(float) * RK_MAX_COLS);
  if (e == cudaSuccess) e = cudaMalloc(&d->mv_qx, RK_MAX_COLS);
  if (e == cudaSuccess) e = cudaMalloc(&d->mv_xs, sizeof(float) * (RK_MAX_COLS / 32));
  if (e == cudaSuccess) e = cudaMalloc(&d->mv_xsum, sizeof(int) * (RK_MAX_COLS / 32));
  if (e == cudaSuccess) e = cudaMalloc(&d->mv_out, sizeof(float) * RK_MAX_ROWS);
  if (e == cudaSuccess) e = cudaMallocHost(&d->pin_in, sizeof(float) * RK_MAX_COLS);
  if (e == cudaSuccess) e = cudaMallocHost(&d->pin_out, sizeof(float) * RK_MAX_ROWS);
  if (e != cudaSuccess) return cleanup(cuda_fail(e, "device open"));
  *out = d;
  return RK_OK;
}

extern "C" void rk_device_close(rk_device *d) {
  if (!d) return;
  cudaSetDevice(d->ordinal);
  if (d->st) cudaStreamSynchronize(d->st);
  cudaFree(d->err_dev);
  cudaFree(d->mv_x);
  cudaFree(d->mv_qx);
  cudaFree(d->mv_xs);
  cudaFree(d->mv_xsum);
  cudaFree(d->mv_out);
  cudaFree(d->flush);
  cudaFreeHost(d->pin_in);
  cudaFreeHost(d->pin_out);
  if (d->st) cudaStreamDestroy(d->st);
  delete d;
}

extern "C" int64_t rk_device_used(rk_device *d) { return d ? d->used : 0; }

// Runs each kind of bounded device wait where nothing completes it, with a
// limit of limit_ns: the chained product kernel waiting for tagged input
// words that no producer writes (what a rank sees when a peer stops
// mid-step), and an mbarrier waiting for copy bytes that never come. Each
// must give up, set the device's error word and end its kernel; the call
// then reports that as any expired wait is reported (RK_ERR_TIMEOUT, the
// word cleared), and the device stays usable.
extern "C" int rk_device_wait_selftest(rk_device *d, int64_t limit_ns) {
  if (!d || limit_ns <= 0 || limit_ns > 10000000000LL) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  // A product of sms rows × 32 columns of zero Q8_0 weights whose input is
  // 32 tagged words that stay at tag 0, while the wait expects epoch 1's.
  const int rows = d->sms, cols = 32;
  const size_t wbytes = (size_t)rows * cols, sbytes = 4 * (size_t)rows, lbytes = 8 * (size_t)cols;
  const size_t off_s = (wbytes + 255) & ~size_t(255), off_ll = off_s + ((sbytes + 255) & ~size_t(255));
  const size_t off_epoch = off_ll + lbytes, off_out = off_epoch + 16, total = off_out + 4 * (size_t)rows;
  char *buf = nullptr;
  CK(cudaMalloc(&buf, total));
  cudaError_t e = cudaMemsetAsync(buf, 0, total, d->st);
  const unsigned one = 1;
  if (e == cudaSuccess) e = cudaMemcpyAsync(buf + off_epoch, &one, 4, cudaMemcpyHostToDevice, d->st);
  ChainArgs ca{};
  MvArgs &a = ca.step[0];
  a.fmt = FMT_Q8_0;
  a.cols = cols;
  a.epi = EPI_STORE;
  a.err = d->err_dev;
  a.part[0].w = (const uint8_t *)buf;
  a.part[0].s = (const float *)(buf + off_s);
  a.part[0].out = (float *)(buf + off_out);
  a.part[0].rows = rows;
  a.nparts = 1;
  a.pro = PRO_QUANT;
  a.wait.ll = (const unsigned long long *)(buf + off_ll);
  a.wait.epoch = (const unsigned *)(buf + off_epoch);
  a.wait.slot = 0;
  a.wait.nslots = 1;
  ca.nsteps = 1;
  ca.wait_ns = (unsigned long long)limit_ns;
  if (e == cudaSuccess) e = launch_matvec_chain(ca, d->sms, d->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  int gather_word = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&gather_word, d->err_dev, sizeof gather_word, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemset(d->err_dev, 0, sizeof(int));
  if (e == cudaSuccess) e = launch_mbar_wait_selftest(d->err_dev, (unsigned long long)limit_ns, d->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  int mbar_word = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&mbar_word, d->err_dev, sizeof mbar_word, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemset(d->err_dev, 0, sizeof(int));
  cudaFree(buf);
  if (e != cudaSuccess) return cuda_fail(e, "wait self-test");
  if (gather_word != DEV_ERR_TIMEOUT || mbar_word != DEV_ERR_TIMEOUT)
    return fail(RK_ERR_STATE, "wait self-test: a wait did not report its expiry (gather word %d, mbarrier word %d)",
                gather_word, mbar_word);
  return fail(RK_ERR_TIMEOUT, "wait self-test: both bounded waits expired and reported (as designed)");
}

// ---------------------------------------------------------------------------
// Groups: one NCCL communicator per process (one process per GPU), for the
// row-sharded stage and head. NCCL is loaded when the first group is made,
// so the library itself does not depend on it; a process that already has
// NCCL loaded (e.g. through torch) shares that copy.
// ---------------------------------------------------------------------------
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

static const NcclApi &nccl() {
  static NcclApi api = [] {
    NcclApi a;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return a;
    a.get_unique_id = (decltype(a.get_unique_id))dlsym(h, "ncclGetUniqueId");
    a.comm_init_rank = (decltype(a.comm_init_rank))dlsym(h, "ncclCommInitRank");
    a.comm_destroy = (decltype(a.comm_destroy))dlsym(h, "ncclCommDestroy");
    a.all_gather = (decltype(a.all_gather))dlsym(h, "ncclAllGather");
    a.send = (decltype(a.send))dlsym(h, "ncclSend");
    a.recv = (decltype(a.recv))dlsym(h, "ncclRecv");
    a.broadcast = (decltype(a.broadcast))dlsym(h, "ncclBroadcast");
    a.error_string = (decltype(a.error_string))dlsym(h, "ncclGetErrorString");
    a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.all_gather && a.send && a.recv &&
           a.broadcast && a.error_string;
    return a;
  }();
  return api;
}

static int nccl_fail(ncclResult_t r, const char *what) {
  return fail(RK_ERR_CUDA, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "nccl");
}

struct rk_group {
  rk_device *d = nullptr;
  ncclComm_t comm = nullptr;
  int rank = 0, n = 1;
};

extern "C" int rk_group_id(unsigned char id[RK_GROUP_ID_BYTES]) {
  if (!id) return fail(RK_ERR_ARGS, "null argument");
  if (!nccl().ok) return fail(RK_ERR_STATE, "NCCL (libnccl.so.2) is not available");
  static_assert(sizeof(ncclUniqueId) == RK_GROUP_ID_BYTES, "group id size");
  ncclUniqueId u;
  ncclResult_t r = nccl().get_unique_id(&u);
  if (r != ncclSuccess) return nccl_fail(r, "group id");
  memcpy(id, &u, sizeof u);
  return RK_OK;
}

extern "C" int rk_group_new(rk_device *d, int nranks, int rank, const unsigned char id[RK_GROUP_ID_BYTES],
                            rk_group **out) {
  if (!d || !id || !out || nranks < 1 || rank < 0 || rank >= nranks) return fail(RK_ERR_ARGS, "bad argument");
  if (!nccl().ok) return fail(RK_ERR_STATE, "NCCL (libnccl.so.2) is not available");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  auto *gr = new rk_group();
  gr->d = d;
  gr->rank = rank;
  gr->n = nranks;
  ncclUniqueId u;
  memcpy(&u, id, sizeof u);
  ncclResult_t r = nccl().comm_init_rank(&gr->comm, nranks, u, rank);
  if (r != ncclSuccess) {
    delete gr;
    return nccl_fail(r, "group init");
  }
  *out = gr;
  return RK_OK;
}

extern "C" void rk_group_free(rk_group *g) {
  if (!g) return;
  cudaSetDevice(g->d->ordinal);
  cudaStreamSynchronize(g->d->st);
  if (g->comm) nccl().comm_destroy(g->comm);
  delete g;
}

extern "C" int rk_group_size(const rk_group *g, int *rank, int *nranks) {
  if (!g) return fail(RK_ERR_ARGS, "null group");
  if (rank) *rank = g->rank;
  if (nranks) *nranks = g->n;
  return RK_OK;
}

// In place: rank r's count floats at buf + r·count go to every rank's buf.
static int group_gather(rk_group *g, float *buf, size_t count, cudaStream_t st) {
  ncclResult_t r = nccl().all_gather(buf + (size_t)g->rank * count, buf, count, ncclFloat32, g->comm, st);
  if (r != ncclSuccess) return nccl_fail(r, "all-gather");
  return RK_OK;
}

extern "C" int rk_group_all_gather(rk_group *g, float *buf_dev, int64_t count) {
  if (!g || !buf_dev || count < 0) return fail(RK_ERR_ARGS, "bad argument");
  rk_device *d = g->d;
  Guard gd(d);
  int rc = set_device(d);
  if (rc) return rc;
  if ((rc = group_gather(g, buf_dev, (size_t)count, d->st))) return rc;
  return sync_dev(d);
}

// ---------------------------------------------------------------------------
// Matrices
// ---------------------------------------------------------------------------
struct rk_matrix {
  rk_device *d = nullptr;
  int rows = 0, cols = 0, fmt = 0;
  uint8_t *w = nullptr;
  float *s = nullptr;
  size_t wbytes = 0, sbytes = 0;
  int64_t bytes = 0;
};

static size_t row_bytes(int fmt, int cols) {
  switch (fmt) {
    case RK_FMT_F32: return 4 * (size_t)cols;
    case RK_FMT_BF16: return 2 * (size_t)cols;
    case RK_FMT_Q8_0: return (size_t)cols;
    default: return (size_t)cols / 2;
  }
}

static bool quantized_fmt(int fmt) { return fmt == RK_FMT_Q8_0 || fmt == RK_FMT_Q4_0; }

// Allocates a matrix. Weights and scales get 256 bytes of zeroed padding:
// the streaming kernels copy 16-byte-aligned supersets of scale runs.
static int matrix_alloc(rk_device *d, int rows, int cols, int fmt, rk_matrix **out) {
  if (fmt < RK_FMT_F32 || fmt > RK_FMT_Q4_0) return fail(RK_ERR_ARGS, "unknown matrix format %d", fmt);
  if (rows <= 0 || cols <= 0 || cols > RK_MAX_COLS || rows > (1 << 24))
    return fail(RK_ERR_ARGS, "gpu: matrix %d×%d out of range", rows, cols);
  if (quantized_fmt(fmt) && cols % 32 != 0) return fail(RK_ERR_ARGS, "gpu: quantized matrix of the wrong shape");
  if (fmt == RK_FMT_BF16 && cols % 2 != 0) return fail(RK_ERR_ARGS, "gpu: bfloat16 rows need an even width");
  auto *m = new rk_matrix();
  m->d = d;
  m->rows = rows;
  m->cols = cols;
  m->fmt = fmt;
  m->wbytes = row_bytes(fmt, cols) * (size_t)rows;
  size_t walloc = ((m->wbytes + 255) & ~size_t(255)) + 256;
  cudaError_t e = cudaMalloc(&m->w, walloc);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->w, 0, walloc, d->st);
  size_t salloc = 0;
  if (e == cudaSuccess && quantized_fmt(fmt)) {
    m->sbytes = sizeof(float) * (size_t)rows * (cols / 32);
    salloc = ((m->sbytes + 255) & ~size_t(255)) + 256;
    e = cudaMalloc(&m->s, salloc);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->s, 0, salloc, d->st);
  }
  if (e != cudaSuccess) {
    cudaFree(m->w);
    cudaFree(m->s);
    delete m;
    return cuda_fail(e, "matrix allocation");
  }
  m->bytes = (int64_t)walloc + (int64_t)salloc;
  d->used += m->bytes;
  *out = m;
  return RK_OK;
}

static void matrix_release(rk_matrix *m) {
  if (!m) return;
  cudaSetDevice(m->d->ordinal);
  cudaStreamSynchronize(m->d->st);
  cudaFree(m->w);
  cudaFree(m->s);
  m->d->used -= m->bytes;
  delete m;
}

extern "C" int rk_matrix_upload(rk_device *d, int rows, int cols, int fmt, const void *w, const float *scales,
                                rk_matrix **out) {
  if (!d || !w || !out) return fail(RK_ERR_ARGS, "null argument");
  if (quantized_fmt(fmt) && !scales) return fail(RK_ERR_ARGS, "gpu: quantized matrix without scales");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  rk_matrix *m = nullptr;
  if ((rc = matrix_alloc(d, rows, cols, fmt, &m))) return rc;
  cudaError_t e = cudaMemcpyAsync(m->w, w, m->wbytes, cudaMemcpyHostToDevice, d->st);
  if (e == cudaSuccess && m->s) e = cudaMemcpyAsync(m->s, scales, m->sbytes, cudaMemcpyHostToDevice, d->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  if (e != cudaSuccess) {
    matrix_release(m);
    return cuda_fail(e, "matrix upload");
  }
  *out = m;
  return RK_OK;
}

extern "C" void rk_matrix_free(rk_matrix *m) {
  if (!m) return;
  rk_device *d = m->d;
  Guard g(d);
  matrix_release(m);
}

extern "C" int64_t rk_matrix_bytes(const rk_matrix *m) { return m ? m->bytes : 0; }
extern "C" int rk_same_device(const rk_matrix *a, const rk_matrix *b) { return a && b && a->d == b->d; }

// Per-launch timing of the matvec kernels during rk_model_profile: events
// around each launch on the launching stream, and the launch's algorithmic
// bytes (weights + scales: matBytes, model.go:269-279).
struct ProfLaunch {
  cudaEvent_t e0, e1;
  double bytes;
};
static thread_local std::vector<ProfLaunch> *g_prof = nullptr;

static double algorithmic_bytes(const MvArgs &a) {
  double b = 0;
  const int nsub = a.epi == EPI_SILU ? 2 : a.nparts;
  for (int p = 0; p < nsub; p++) {
    const double n = (double)a.part[p].rows * a.cols;
    switch (a.fmt) {
      case FMT_F32: b += 4 * n; break;
      case FMT_BF16: b += 2 * n; break;
      case FMT_Q8_0: b += n + n / 32 * 4; break;
      default: b += n / 2 + n / 32 * 4;
    }
  }
  return b;
}

static cudaError_t launch_mv(rk_device *d, const MvArgs &a, cudaStream_t st) {
  if (!g_prof) return launch_matvec(a, d->sms, st);
  ProfLaunch pl{};
  pl.bytes = algorithmic_bytes(a);
  cudaError_t e = cudaEventCreate(&pl.e0);
  if (e == cudaSuccess) e = cudaEventCreate(&pl.e1);
  if (e == cudaSuccess) e = cudaEventRecord(pl.e0, st);
  if (e == cudaSuccess) e = launch_matvec(a, d->sms, st);
  if (e == cudaSuccess) e = cudaEventRecord(pl.e1, st);
  g_prof->push_back(pl);
  return e;
}

static cudaError_t launch_chain(rk_device *d, const ChainArgs &ca, cudaStream_t st) {
  if (!g_prof) return launch_matvec_chain(ca, d->sms, st);
  ProfLaunch pl{};
  for (int k = 0; k < ca.nsteps; k++) pl.bytes += algorithmic_bytes(ca.step[k]);
  cudaError_t e = cudaEventCreate(&pl.e0);
  if (e == cudaSuccess) e = cudaEventCreate(&pl.e1);
  if (e == cudaSuccess) e = cudaEventRecord(pl.e0, st);
  if (e == cudaSuccess) e = launch_matvec_chain(ca, d->sms, st);
  if (e == cudaSuccess) e = cudaEventRecord(pl.e1, st);
  g_prof->push_back(pl);
  return e;
}

static MvPart part_of(const rk_matrix *m, float *out) {
  MvPart p;
  p.w = m->w;
  p.s = m->s;
  p.out = out;
  p.rows = m->rows;
  return p;
}

// How a quantized product gets its Q8_0 input: given in qx/xs/xsum, or
// quantized by every CTA from x_dev (after rmsNorm with norm_w).
struct Pro {
  int pro = PRO_GIVEN;
  const float *norm_w = nullptr;
  float recipN = 0.0f, eps = 0.0f;
  GatherPut put{};    // fused gather of the output (row sharding)
  GatherWait wait{};  // the input is a fused gather's
};

// Enqueues products of matrices (same cols) sharing one input, grouping
// runs of the same format into one launch of up to four matrices.
static int enqueue_matvecs(rk_device *d, int n, rk_matrix *const *ms, float *const *outs, const float *x_dev,
                           const int8_t *qx, const float *xs, const int *xsum, int epi, cudaStream_t st = nullptr,
                           Pro pro = Pro()) {
  if (!st) st = d->st;
  int i = 0;
  while (i < n) {
    MvArgs a{};
    a.fmt = ms[i]->fmt;
    a.cols = ms[i]->cols;
    a.epi = epi;
    a.qx = qx;
    a.xs = xs;
    a.xsum = xsum;
    a.x = x_dev;
    a.err = d->err_dev;
    if (quantized_fmt(a.fmt)) {
      a.pro = pro.pro;
      a.norm_w = pro.norm_w;
      a.recipN = pro.recipN;
      a.eps = pro.eps;
      a.put = pro.put;
      a.wait = pro.wait;
    }
    int np = 0;
    while (i < n && np < 4 && ms[i]->fmt == a.fmt) {
      a.part[np++] = part_of(ms[i], outs[i]);
      i++;
    }
    a.nparts = np;
    CK(launch_mv(d, a, st));
  }
  return RK_OK;
}

extern "C" int rk_mulvecs(int n, rk_matrix *const *ms, float *const *outs, const float *x) {
  if (n == 0) return RK_OK;
  if (n < 0 || !ms || !outs || !x) return fail(RK_ERR_ARGS, "null argument");
  rk_device *d = ms[0]->d;
  const int cols = ms[0]->cols;
  int64_t total = 0;
  bool quant = false;
  for (int i = 0; i < n; i++) {
    if (!ms[i] || ms[i]->d != d || ms[i]->cols != cols || !outs[i])
      return fail(RK_ERR_ARGS, "gpu: matrices of mulvecs must share a device and a width");
    total += ms[i]->rows;
    quant |= quantized_fmt(ms[i]->fmt);
  }
  if (total > RK_MAX_ROWS) return fail(RK_ERR_ARGS, "gpu: products too large for one submission");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  memcpy(d->pin_in, x, sizeof(float) * cols);
  CK(cudaMemcpyAsync(d->mv_x, d->pin_in, sizeof(float) * cols, cudaMemcpyHostToDevice, d->st));
  if (quant) CK(launch_quantize_act(d->mv_x, cols, nullptr, 0.0f, 0.0f, nullptr, d->mv_qx, d->mv_xs, d->mv_xsum, d->st));
  std::vector<float *> douts(n);
  int64_t off = 0;
  for (int i = 0; i < n; i++) {
    douts[i] = d->mv_out + off;
    off += ms[i]->rows;
  }
  if ((rc = enqueue_matvecs(d, n, ms, douts.data(), d->mv_x, d->mv_qx, d->mv_xs, d->mv_xsum, EPI_STORE))) return rc;
  CK(cudaMemcpyAsync(d->pin_out, d->mv_out, sizeof(float) * total, cudaMemcpyDeviceToHost, d->st));
  if ((rc = sync_dev(d))) return rc;
  off = 0;
  for (int i = 0; i < n; i++) {
    memcpy(outs[i], d->pin_out + off, sizeof(float) * ms[i]->rows);
    off += ms[i]->rows;
  }
  return RK_OK;
}

extern "C" int rk_matrix_mulvec(rk_matrix *m, float *out, const float *x) {
  if (!m) return fail(RK_ERR_ARGS, "null matrix");
  return rk_mulvecs(1, &m, &out, x);
}

extern "C" int rk_matrix_mulvec_many(rk_matrix *m, int n, float *out, const float *x) {
  if (!m || n < 0 || (n > 0 && (!x || !out))) return fail(RK_ERR_ARGS, "bad argument");
  if (n == 0) return RK_OK;
  if (!mv_many_ok(m->fmt, m->rows, m->cols, m->w, m->s)) {
    // Formats and widths the batched kernel does not take: one product per
    // vector, as ForwardMany's per-token Forward does.
    for (int t = 0; t < n; t++) {
      int rc = rk_matrix_mulvec(m, out + (size_t)t * m->rows, x + (size_t)t * m->cols);
      if (rc) return rc;
    }
    return RK_OK;
  }
  rk_device *d = m->d;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  const size_t cols = (size_t)m->cols, rows = (size_t)m->rows;
  const int xs_pitch = (n + 3) & ~3;  // the batched kernel's block-major input scales
  float *dx = nullptr, *dxs = nullptr, *dout = nullptr;
  int8_t *dqx = nullptr;
  cudaError_t e = cudaMalloc(&dx, 4 * n * cols);
  if (e == cudaSuccess) e = cudaMalloc(&dqx, n * cols);
  if (e == cudaSuccess) e = cudaMalloc(&dxs, 4 * (size_t)xs_pitch * (cols / 32));
  if (e == cudaSuccess) e = cudaMalloc(&dout, 4 * n * rows);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dx, x, 4 * n * cols, cudaMemcpyHostToDevice, d->st);
  if (e == cudaSuccess) e = launch_quantize_many(dx, n, m->cols, nullptr, 0.0f, 0.0f, dqx, dxs, xs_pitch, d->st);
  if (e == cudaSuccess) {
    const MmMat mat{m->w, m->s, m->rows, dout, (long long)rows, EPI_STORE, m->fmt};
    e = launch_mv_many(1, &mat, m->cols, n, dqx, dxs, xs_pitch, d->err_dev, d->sms, d->st);
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, dout, 4 * n * rows, cudaMemcpyDeviceToHost, d->st);
  rc = e == cudaSuccess ? sync_dev(d) : cuda_fail(e, "batched matvec");
  cudaStreamSynchronize(d->st);
  for (void *p : {(void *)dx, (void *)dqx, (void *)dxs, (void *)dout}) cudaFree(p);
  return rc;
}

extern "C" int rk_matrix_download(rk_matrix *m, void *w, float *scales) {
  if (!m || !w) return fail(RK_ERR_ARGS, "null argument");
  Guard g(m->d);
  int rc = set_device(m->d);
  if (rc) return rc;
  CK(cudaMemcpyAsync(w, m->w, m->wbytes, cudaMemcpyDeviceToHost, m->d->st));
  if (scales && m->s) CK(cudaMemcpyAsync(scales, m->s, m->sbytes, cudaMemcpyDeviceToHost, m->d->st));
  CK(cudaStreamSynchronize(m->d->st));
  return RK_OK;
}

// ---------------------------------------------------------------------------
// Vectors
// ---------------------------------------------------------------------------
struct rk_vectors {
  rk_device *d = nullptr;
  float *v = nullptr;
  int64_t n = 0, bytes = 0;
};

static int vectors_alloc(rk_device *d, const float *v, int64_t n, rk_vectors **out) {
  auto *vs = new rk_vectors();
  vs->d = d;
  vs->n = n;
  vs->bytes = ((4 * std::max<int64_t>(n, 1) + 255) & ~int64_t(255));
  cudaError_t e = cudaMalloc(&vs->v, (size_t)vs->bytes);
  if (e == cudaSuccess) e = cudaMemsetAsync(vs->v, 0, (size_t)vs->bytes, d->st);
  if (e == cudaSuccess && n > 0) e = cudaMemcpyAsync(vs->v, v, sizeof(float) * n, cudaMemcpyHostToDevice, d->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  if (e != cudaSuccess) {
    cudaFree(vs->v);
    delete vs;
    return cuda_fail(e, "vectors upload");
  }
  d->used += vs->bytes;
  *out = vs;
  return RK_OK;
}

static void vectors_release(rk_vectors *v) {
  if (!v) return;
  cudaSetDevice(v->d->ordinal);
  cudaStreamSynchronize(v->d->st);
  cudaFree(v->v);
  v->d->used -= v->bytes;
  delete v;
}

extern "C" int rk_vectors_upload(rk_device *d, const float *v, int64_t n, rk_vectors **out) {
  if (!d || !out || n < 0 || (n > 0 && !v)) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  return vectors_alloc(d, v, n, out);
}

extern "C" void rk_vectors_free(rk_vectors *v) {
  if (!v) return;
  rk_device *d = v->d;
  Guard g(d);
  vectors_release(v);
}

// ---------------------------------------------------------------------------
// Arena and Batch (batch.go)
// ---------------------------------------------------------------------------
struct rk_arena {
  rk_device *d = nullptr;
  float *buf = nullptr;
  int64_t words = 0;
  float *staging = nullptr;  // pinned
  int64_t staging_words = 0;
  int64_t qx_off = -1, xs_off = -1;
  int *xsum = nullptr;  // block sums of the quantized input (Q4_0 products)
  int64_t bytes = 0;
};

extern "C" int rk_arena_new(rk_device *d, int64_t words, int64_t staging_words, rk_arena **out) {
  if (!d || !out || words < 0 || staging_words < 0) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  auto *a = new rk_arena();
  a->d = d;
  a->words = words;
  a->staging_words = staging_words;
  size_t bytes = (size_t)4 * std::max<int64_t>(words, 1);
  bytes = ((bytes + 255) & ~size_t(255)) + 256;
  cudaError_t e = cudaMalloc(&a->buf, bytes);
  if (e == cudaSuccess) e = cudaMemsetAsync(a->buf, 0, bytes, d->st);
  if (e == cudaSuccess) e = cudaMallocHost(&a->staging, sizeof(float) * std::max<int64_t>(staging_words, 1));
  if (e == cudaSuccess) e = cudaMalloc(&a->xsum, sizeof(int) * (RK_MAX_COLS / 32));
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  if (e != cudaSuccess) {
    cudaFree(a->buf);
    cudaFreeHost(a->staging);
    cudaFree(a->xsum);
    delete a;
    return cuda_fail(e, "arena allocation");
  }
  a->bytes = (int64_t)bytes;
  d->used += a->bytes;
  *out = a;
  return RK_OK;
}

extern "C" void rk_arena_set_quant_scratch(rk_arena *a, int64_t qx_off, int64_t xs_off) {
  if (!a) return;
  a->qx_off = qx_off;
  a->xs_off = xs_off;
}

extern "C" int64_t rk_arena_bytes(const rk_arena *a) { return a ? a->bytes : 0; }

extern "C" void rk_arena_free(rk_arena *a) {
  if (!a) return;
  rk_device *d = a->d;
  Guard g(d);
  cudaSetDevice(d->ordinal);
  cudaStreamSynchronize(d->st);
  cudaFree(a->buf);
  cudaFreeHost(a->staging);
  cudaFree(a->xsum);
  d->used -= a->bytes;
  delete a;
}

struct PendingRead {
  float *dst;
  int64_t at, n;
};

struct rk_batch {
  rk_arena *a = nullptr;
  std::vector<std::function<int()>> ops;
  std::vector<PendingRead> reads;
  int64_t staged = 0;
  int err = RK_OK;
  std::string msg;
};

static void batch_fail(rk_batch *b, int code, const char *fmt, ...) {
  if (b->err != RK_OK) return;
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  b->err = code;
  b->msg = buf;
}

// Word range [off, off+n) inside the arena?
static bool in_arena(const rk_arena *a, int64_t off, int64_t n) { return off >= 0 && n >= 0 && off + n <= a->words; }

static bool batch_range(rk_batch *b, int64_t off, int64_t n, const char *what) {
  if (b->err != RK_OK) return false;
  if (!in_arena(b->a, off, n)) {
    batch_fail(b, RK_ERR_ARGS, "gpu: %s range [%lld, %lld) outside the arena of %lld words", what, (long long)off,
               (long long)(off + n), (long long)b->a->words);
    return false;
  }
  return true;
}

extern "C" int rk_batch_begin(rk_arena *a, rk_batch **out) {
  if (!a || !out) return fail(RK_ERR_ARGS, "null argument");
  a->d->mu.lock();  // held until rk_batch_submit, as Batch holds Device.mu
  auto *b = new rk_batch();
  b->a = a;
  *out = b;
  return RK_OK;
}

static bool batch_stage(rk_batch *b, int64_t n, int64_t *at) {
  if (b->err != RK_OK) return false;
  if (b->staged + n > b->a->staging_words) {
    batch_fail(b, RK_ERR_ARGS, "gpu: batch moves more than its staging holds");
    return false;
  }
  *at = b->staged;
  b->staged += n;
  return true;
}

extern "C" void rk_batch_write(rk_batch *b, int64_t off, const float *data, int64_t n) {
  if (!b) return;
  int64_t at;
  if (!batch_stage(b, n, &at) || n == 0) return;
  if (!batch_range(b, off, n, "write")) return;
  memcpy(b->a->staging + at, data, sizeof(float) * n);
  rk_arena *a = b->a;
  b->ops.push_back([a, off, at, n]() {
    CK(cudaMemcpyAsync(a->buf + off, a->staging + at, sizeof(float) * n, cudaMemcpyHostToDevice, a->d->st));
    return RK_OK;
  });
}

extern "C" void rk_batch_read(rk_batch *b, int64_t off, float *dst, int64_t n) {
  if (!b) return;
  int64_t at;
  if (!batch_stage(b, n, &at) || n == 0) return;
  if (!batch_range(b, off, n, "read")) return;
  rk_arena *a = b->a;
  b->ops.push_back([a, off, at, n]() {
    CK(cudaMemcpyAsync(a->staging + at, a->buf + off, sizeof(float) * n, cudaMemcpyDeviceToHost, a->d->st));
    return RK_OK;
  });
  b->reads.push_back({dst, at, n});
}

extern "C" void rk_batch_quantize(rk_batch *b, int64_t in_off, int n) {
  if (!b || b->err) return;
  rk_arena *a = b->a;
  if (a->qx_off < 0 || a->xs_off < 0) return batch_fail(b, RK_ERR_ARGS, "gpu: arena has no scratch for quantized inputs");
  if (n % 32 != 0 || n > RK_MAX_COLS) return batch_fail(b, RK_ERR_ARGS, "gpu: quantize of %d floats", n);
  if (!batch_range(b, in_off, n, "quantize input") || !batch_range(b, a->qx_off, n / 4, "quantized input") ||
      !batch_range(b, a->xs_off, n / 32, "input scales"))
    return;
  b->ops.push_back([a, in_off, n]() {
    CK(launch_quantize_act(a->buf + in_off, n, nullptr, 0.0f, 0.0f, nullptr,
                           reinterpret_cast<int8_t *>(a->buf + a->qx_off), a->buf + a->xs_off, a->xsum, a->d->st));
    return RK_OK;
  });
}

extern "C" void rk_batch_matvecs(rk_batch *b, int n, rk_matrix *const *ms, const int64_t *out_offs, int64_t in_off) {
  if (!b || b->err) return;
  rk_arena *a = b->a;
  bool quant = false;
  int qcols = -1;
  for (int i = 0; i < n; i++) {
    if (!ms[i] || ms[i]->d != a->d) return batch_fail(b, RK_ERR_ARGS, "gpu: matrix on another device");
    if (!batch_range(b, out_offs[i], ms[i]->rows, "product output")) return;
    if (quantized_fmt(ms[i]->fmt)) {
      if (qcols >= 0 && qcols != ms[i]->cols) return batch_fail(b, RK_ERR_ARGS, "gpu: quantized products of different widths");
      qcols = ms[i]->cols;
      quant = true;
    } else if (!batch_range(b, in_off, ms[i]->cols, "product input")) {
      return;
    }
  }
  if (quant) rk_batch_quantize(b, in_off, qcols);
  if (b->err) return;
  std::vector<rk_matrix *> mv(ms, ms + n);
  std::vector<int64_t> offs(out_offs, out_offs + n);
  b->ops.push_back([a, mv, offs, in_off]() {
    for (size_t i = 0; i < mv.size(); i++) {
      float *out = a->buf + offs[i];
      int rc = enqueue_matvecs(a->d, 1, &mv[i], &out, a->buf + in_off, reinterpret_cast<int8_t *>(a->buf + a->qx_off),
                               a->buf + a->xs_off, a->xsum, EPI_STORE);
      if (rc) return rc;
    }
    return RK_OK;
  });
}

extern "C" void rk_batch_rmsnorm(rk_batch *b, rk_vectors *vecs, int64_t in_off, int64_t out_off, int64_t w_off, int n,
                                 int segs, int stride, float recip_n, float eps) {
  if (!b || b->err) return;
  if (!vecs || w_off < 0 || w_off + n > vecs->n) return batch_fail(b, RK_ERR_ARGS, "gpu: rmsnorm weights out of range");
  const int64_t span = segs > 0 ? (int64_t)(segs - 1) * stride + n : 0;
  if (!batch_range(b, in_off, span, "rmsnorm input") || !batch_range(b, out_off, span, "rmsnorm output")) return;
  rk_arena *a = b->a;
  b->ops.push_back([=]() {
    CK(launch_rmsnorm(a->buf + in_off, a->buf + out_off, vecs->v + w_off, n, segs, stride, recip_n, eps, a->d->st));
    return RK_OK;
  });
}

extern "C" void rk_batch_addvec(rk_batch *b, rk_vectors *vecs, int64_t out_off, int64_t v_off, int n) {
  if (!b || b->err) return;
  if (!vecs || v_off < 0 || v_off + n > vecs->n) return batch_fail(b, RK_ERR_ARGS, "gpu: vector out of range");
  if (!batch_range(b, out_off, n, "addvec")) return;
  rk_arena *a = b->a;
  b->ops.push_back([=]() {
    CK(launch_addvec(a->buf + out_off, vecs->v + v_off, n, a->d->st));
    return RK_OK;
  });
}

extern "C" void rk_batch_rope(rk_batch *b, int64_t q_off, int64_t k_off, int q_dim, int kv_dim, int head_size,
                              int64_t cos_off, int64_t sin_off) {
  if (!b || b->err) return;
  if (head_size <= 0 || head_size % 2) return batch_fail(b, RK_ERR_ARGS, "gpu: rope head size %d", head_size);
  if (!batch_range(b, q_off, q_dim, "rope q") || !batch_range(b, k_off, std::min(kv_dim, q_dim), "rope k") ||
      !batch_range(b, cos_off, head_size / 2, "rope cos") || !batch_range(b, sin_off, head_size / 2, "rope sin"))
    return;
  rk_arena *a = b->a;
  b->ops.push_back([=]() {
    CK(launch_rope(a->buf + q_off, a->buf + k_off, q_dim, kv_dim, head_size, a->buf + cos_off, a->buf + sin_off, a->d->st));
    return RK_OK;
  });
}

extern "C" void rk_batch_copy(rk_batch *b, int64_t src_off, int64_t dst_off, int n) {
  if (!b || b->err) return;
  if (!batch_range(b, src_off, n, "copy source") || !batch_range(b, dst_off, n, "copy destination")) return;
  rk_arena *a = b->a;
  b->ops.push_back([=]() {
    CK(launch_copy(a->buf + src_off, a->buf + dst_off, n, a->d->st));
    return RK_OK;
  });
}

extern "C" void rk_batch_attention(rk_batch *b, int64_t q_off, int64_t keys_off, int64_t vals_off, int64_t att_off,
                                   int att_stride, int64_t out_off, int positions, int heads, int kv_heads, int head_size,
                                   int kv_dim, float inv_sqrt) {
  if (!b || b->err) return;
  if (positions <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || head_size <= 0 || att_stride < positions ||
      kv_dim < kv_heads * head_size)
    return batch_fail(b, RK_ERR_ARGS, "gpu: attention arguments out of range");
  const int64_t qd = (int64_t)heads * head_size;
  const int64_t cache = (int64_t)(positions - 1) * kv_dim + (int64_t)kv_heads * head_size;
  if (!batch_range(b, q_off, qd, "attention q") || !batch_range(b, keys_off, cache, "attention keys") ||
      !batch_range(b, vals_off, cache, "attention values") ||
      !batch_range(b, att_off, (int64_t)(heads - 1) * att_stride + positions, "attention scores") ||
      !batch_range(b, out_off, qd, "attention output"))
    return;
  rk_arena *a = b->a;
  b->ops.push_back([=]() {
    AttnArgs at{};
    at.q = a->buf + q_off;
    at.keys = a->buf + keys_off;
    at.vals = a->buf + vals_off;
    at.att = a->buf + att_off;
    at.out = a->buf + out_off;
    at.positions = positions;
    at.heads = heads;
    at.kv_heads = kv_heads;
    at.hs = head_size;
    at.kv_dim = kv_dim;
    at.att_stride = att_stride;
    at.inv_sqrt = inv_sqrt;
    at.err = a->d->err_dev;
    CK(launch_attention(at, a->d->st));
    return RK_OK;
  });
}

extern "C" void rk_batch_residual(rk_batch *b, int64_t x_off, int64_t y_off, int n, int canonical) {
  if (!b || b->err) return;
  if (!batch_range(b, x_off, n, "residual x") || !batch_range(b, y_off, n, "residual y")) return;
  rk_arena *a = b->a;
  b->ops.push_back([=]() {
    CK(launch_residual(a->buf + x_off, a->buf + y_off, n, canonical, a->d->st));
    return RK_OK;
  });
}

extern "C" void rk_batch_silumul(rk_batch *b, int64_t a_off, int64_t b_off, int n) {
  if (!b || b->err) return;
  if (!batch_range(b, a_off, n, "silumul a") || !batch_range(b, b_off, n, "silumul b")) return;
  rk_arena *a = b->a;
  b->ops.push_back([=]() {
    CK(launch_silumul(a->buf + a_off, a->buf + b_off, n, a->d->st));
    return RK_OK;
  });
}

extern "C" int rk_batch_submit(rk_batch *b) {
  if (!b) return fail(RK_ERR_ARGS, "null batch");
  rk_arena *a = b->a;
  rk_device *d = a->d;
  int rc = b->err;
  std::string msg = b->msg;
  if (rc == RK_OK) {
    rc = set_device(d);
    for (size_t i = 0; rc == RK_OK && i < b->ops.size(); i++) rc = b->ops[i]();
    if (rc == RK_OK) rc = sync_dev(d);
    if (rc == RK_OK)
      for (const auto &r : b->reads) memcpy(r.dst, a->staging + r.at, sizeof(float) * r.n);
  } else {
    g_err = msg;
  }
  delete b;
  d->mu.unlock();
  return rc;
}

// ---------------------------------------------------------------------------
// Layers and stages (model.go, gpustage.go)
// ---------------------------------------------------------------------------
static int head_size(const rk_config *c) { return c->head_dim > 0 ? c->head_dim : c->dim / c->heads; }
static float cfg_eps(const rk_config *c) {
  return c->norm_eps > 0 ? (float)c->norm_eps : 1e-5f;  // the float32 constant 1e-5 (model.go:90)
}
static bool cfg_quantized(const rk_config *c) {
  return c->dtype == RK_DTYPE_Q8_0 || c->dtype == RK_DTYPE_Q4_0 || c->dtype == RK_DTYPE_Q4_M;
}

extern "C" int rk_config_validate(const rk_config *c) {
  if (!c) return fail(RK_ERR_ARGS, "null config");
  if (c->dim <= 0 || c->hidden <= 0 || c->layers <= 0 || c->heads <= 0 || c->kv_heads <= 0 || c->vocab <= 0 ||
      c->seq_len <= 0 || c->head_dim < 0)
    return fail(RK_ERR_ARGS, "non-positive dimension");
  if ((c->head_dim == 0 && c->dim % c->heads != 0) || c->heads % c->kv_heads != 0 || head_size(c) % 2 != 0)
    return fail(RK_ERR_ARGS, "heads do not divide the model dimension evenly");
  if (c->dim > 1 << 16 || c->hidden > 1 << 18 || c->layers > 1024 || c->vocab > 1 << 20 || c->seq_len > 1 << 20 ||
      head_size(c) > 1024 || c->heads > 1024)
    return fail(RK_ERR_ARGS, "dimensions out of range");
  if (c->dtype < RK_DTYPE_F32 || c->dtype > RK_DTYPE_Q4_M) return fail(RK_ERR_ARGS, "unknown weight type %d", c->dtype);
  if (cfg_quantized(c) && (c->dim % 32 || (c->heads * head_size(c)) % 32 || c->hidden % 32))
    return fail(RK_ERR_ARGS, "quantized models need widths that are multiples of 32");
  if (c->rope_theta < 0 || c->norm_eps < 0 || c->norm_eps > 1) return fail(RK_ERR_ARGS, "rope base or norm epsilon out of range");
  return RK_OK;
}

struct rk_layer {
  rk_device *d = nullptr;
  rk_config c{};
  int nshards = 1, shard = 0;  // row shard `shard` of `nshards` (see layer_dims)
  rk_matrix *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr, *w1 = nullptr, *w2 = nullptr, *w3 = nullptr;
  rk_vectors *vecs = nullptr;
  // Offsets in vecs (vecLayout, model.go:298-314); -1 when absent.
  int64_t o_rms_att = 0, o_rms_ffn = 0, o_bq = -1, o_bk = -1, o_bv = -1, o_qn = -1, o_kn = -1;
};

static void layer_release(rk_layer *l) {
  if (!l) return;
  for (rk_matrix *m : {l->wq, l->wk, l->wv, l->wo, l->w1, l->w2, l->w3}) matrix_release(m);
  vectors_release(l->vecs);
  delete l;
}

static int layer_vectors(rk_device *d, const rk_config *c, const rk_host_layer *h, rk_layer *l) {
  const int hs = head_size(c), qd = c->heads * hs, kvd = c->kv_heads * hs;
  std::vector<float> all;
  auto put = [&](const float *v, int n) -> int64_t {
    int64_t at = (int64_t)all.size();
    all.insert(all.end(), v, v + n);
    return at;
  };
  if (!h->rms_att || !h->rms_ffn) return fail(RK_ERR_ARGS, "layer without norm weights");
  l->o_rms_att = put(h->rms_att, c->dim);
  l->o_rms_ffn = put(h->rms_ffn, c->dim);
  if (c->qkv_bias) {
    if (!h->bq || !h->bk || !h->bv) return fail(RK_ERR_ARGS, "qkv_bias without biases");
    l->o_bq = put(h->bq, qd);
    l->o_bk = put(h->bk, kvd);
    l->o_bv = put(h->bv, kvd);
  }
  if (c->qk_norm) {
    if (!h->q_norm || !h->k_norm) return fail(RK_ERR_ARGS, "qk_norm without norm weights");
    l->o_qn = put(h->q_norm, hs);
    l->o_kn = put(h->k_norm, hs);
  }
  return vectors_alloc(d, all.data(), (int64_t)all.size(), &l->vecs);
}

// Expected format of each matrix (Config.matType, model.go:105-113).
static int mat_fmt(const rk_config *c, bool sensitive) {
  switch (c->dtype) {
    case RK_DTYPE_F32: return RK_FMT_F32;
    case RK_DTYPE_BF16: return RK_FMT_BF16;
    case RK_DTYPE_Q8_0: return RK_FMT_Q8_0;
    case RK_DTYPE_Q4_0: return RK_FMT_Q4_0;
    default: return sensitive ? RK_FMT_Q8_0 : RK_FMT_Q4_0;
  }
}

// Row sharding over G GPUs (by whole kv heads, so attention stays local):
// shard r holds query heads [r·heads/G, …) and kv heads [r·kvHeads/G, …) of
// Wq / Wk / Wv, rows [r·D/G, …) of Wo and W2, and rows [r·H/G, …) of W1
// and W3; the inputs of every product stay whole. dims[i] = {rows, cols} of
// wq, wk, wv, wo, w1, w2, w3 in that order.
static int layer_dims(const rk_config *c, int G, int dims[7][2]) {
  const int hs = head_size(c), qd = c->heads * hs, kvd = c->kv_heads * hs, D = c->dim, H = c->hidden;
  if (G < 1 || c->kv_heads % G || D % G || H % G)
    return fail(RK_ERR_ARGS, "cannot shard kv heads %d, dim %d, hidden %d over %d", c->kv_heads, D, H, G);
  const int r[7][2] = {{qd / G, D}, {kvd / G, D}, {kvd / G, D}, {D / G, qd}, {H / G, D}, {D / G, H}, {H / G, D}};
  memcpy(dims, r, sizeof r);
  return RK_OK;
}

static int layer_upload(rk_device *d, const rk_config *c, int nshards, int shard, const rk_host_layer *h,
                        rk_layer **out) {
  if (!d || !c || !h || !out || shard < 0 || shard >= nshards) return fail(RK_ERR_ARGS, "bad argument");
  int rc = rk_config_validate(c);
  if (rc) return rc;
  int dims[7][2];
  if ((rc = layer_dims(c, nshards, dims))) return rc;
  Guard g(d);
  if ((rc = set_device(d))) return rc;
  auto *l = new rk_layer();
  l->d = d;
  l->c = *c;
  l->nshards = nshards;
  l->shard = shard;
  struct Spec {
    rk_matrix **dst;
    const rk_host_matrix *src;
    int rows, cols;
    bool sensitive;
  } specs[7] = {{&l->wq, &h->wq, dims[0][0], dims[0][1], false}, {&l->wk, &h->wk, dims[1][0], dims[1][1], false},
                {&l->wv, &h->wv, dims[2][0], dims[2][1], true},  {&l->wo, &h->wo, dims[3][0], dims[3][1], false},
                {&l->w1, &h->w1, dims[4][0], dims[4][1], false}, {&l->w2, &h->w2, dims[5][0], dims[5][1], true},
                {&l->w3, &h->w3, dims[6][0], dims[6][1], false}};
  for (auto &s : specs) {
    if (s.src->fmt != mat_fmt(c, s.sensitive)) {
      layer_release(l);
      return fail(RK_ERR_ARGS, "layer matrix format %d, want %d for dtype %d", s.src->fmt, mat_fmt(c, s.sensitive), c->dtype);
    }
    if ((rc = matrix_alloc(d, s.rows, s.cols, s.src->fmt, s.dst))) {
      layer_release(l);
      return rc;
    }
    cudaError_t e = cudaMemcpyAsync((*s.dst)->w, s.src->w, (*s.dst)->wbytes, cudaMemcpyHostToDevice, d->st);
    if (e == cudaSuccess && (*s.dst)->s)
      e = cudaMemcpyAsync((*s.dst)->s, s.src->scales, (*s.dst)->sbytes, cudaMemcpyHostToDevice, d->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
    if (e != cudaSuccess) {
      layer_release(l);
      return cuda_fail(e, "layer upload");
    }
  }
  if ((rc = layer_vectors(d, c, h, l))) {
    layer_release(l);
    return rc;
  }
  *out = l;
  return RK_OK;
}

extern "C" int rk_layer_upload(rk_device *d, const rk_config *c, const rk_host_layer *h, rk_layer **out) {
  return layer_upload(d, c, 1, 0, h, out);
}

extern "C" int rk_layer_upload_shard(rk_device *d, const rk_config *c, int nshards, int shard, const rk_host_layer *h,
                                     rk_layer **out) {
  return layer_upload(d, c, nshards, shard, h, out);
}

static int layer_from_device(rk_device *d, const rk_config *c, int nshards, int shard, const rk_host_layer *vectors,
                             rk_matrix *wq, rk_matrix *wk, rk_matrix *wv, rk_matrix *wo, rk_matrix *w1, rk_matrix *w2,
                             rk_matrix *w3, rk_layer **out) {
  if (!d || !c || !vectors || !out || shard < 0 || shard >= nshards) return fail(RK_ERR_ARGS, "bad argument");
  int rc = rk_config_validate(c);
  if (rc) return rc;
  int dims[7][2];
  if ((rc = layer_dims(c, nshards, dims))) return rc;
  struct Spec {
    rk_matrix *m;
    int rows, cols;
    bool sensitive;
  } specs[7] = {{wq, dims[0][0], dims[0][1], false}, {wk, dims[1][0], dims[1][1], false},
                {wv, dims[2][0], dims[2][1], true},  {wo, dims[3][0], dims[3][1], false},
                {w1, dims[4][0], dims[4][1], false}, {w2, dims[5][0], dims[5][1], true},
                {w3, dims[6][0], dims[6][1], false}};
  for (auto &s : specs)
    if (!s.m || s.m->d != d || s.m->rows != s.rows || s.m->cols != s.cols || s.m->fmt != mat_fmt(c, s.sensitive))
      return fail(RK_ERR_ARGS, "layer matrix of the wrong shape, format or device");
  Guard g(d);
  if ((rc = set_device(d))) return rc;
  auto *l = new rk_layer();
  l->d = d;
  l->c = *c;
  l->nshards = nshards;
  l->shard = shard;
  if ((rc = layer_vectors(d, c, vectors, l))) {
    delete l;
    return rc;
  }
  l->wq = wq;
  l->wk = wk;
  l->wv = wv;
  l->wo = wo;
  l->w1 = w1;
  l->w2 = w2;
  l->w3 = w3;
  *out = l;
  return RK_OK;
}

extern "C" int rk_layer_from_device(rk_device *d, const rk_config *c, const rk_host_layer *vectors, rk_matrix *wq,
                                    rk_matrix *wk, rk_matrix *wv, rk_matrix *wo, rk_matrix *w1, rk_matrix *w2,
                                    rk_matrix *w3, rk_layer **out) {
  return layer_from_device(d, c, 1, 0, vectors, wq, wk, wv, wo, w1, w2, w3, out);
}

extern "C" int rk_layer_from_device_shard(rk_device *d, const rk_config *c, int nshards, int shard,
                                          const rk_host_layer *vectors, rk_matrix *wq, rk_matrix *wk, rk_matrix *wv,
                                          rk_matrix *wo, rk_matrix *w1, rk_matrix *w2, rk_matrix *w3,
                                          rk_layer **out) {
  return layer_from_device(d, c, nshards, shard, vectors, wq, wk, wv, wo, w1, w2, w3, out);
}

extern "C" void rk_layer_free(rk_layer *l) {
  if (!l) return;
  rk_device *d = l->d;
  Guard g(d);
  layer_release(l);
}

struct rk_stage {
  rk_device *d = nullptr;
  rk_config c{};
  std::vector<rk_layer *> layers;
  int ctx = 0;
  int att_stride = 0;  // ctx rounded up to 4 floats (16-byte rows of scores)
  // Value caches are stored transposed (element i's positions contiguous,
  // v_pitch floats apart) when the attention runs as one fused kernel,
  // which then fetches a CTA's value slice with a few bulk copies; 0 keeps
  // the reference's [ctx][kvDim] rows.
  int v_pitch = 0;
  // Activations and scratch (gpustage.go:51-83).
  float *x = nullptr, *xb = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att_out = nullptr, *hb = nullptr,
        *hb2 = nullptr, *att = nullptr, *xs = nullptr, *cos_ = nullptr, *sin_ = nullptr, *io = nullptr;
  int8_t *qx = nullptr;
  int *xsum = nullptr, *pos_dev = nullptr, *tok_dev = nullptr;
  std::vector<float *> keys, vals;
  float *pin_io = nullptr;
  std::vector<void *> allocs;
  int64_t bytes = 0;
  cudaGraphExec_t graph = nullptr;
  int io_tokens = 64;  // gpuBatch, gpustage.go:17
  // ForwardMany's batched layers (stage_forward_many), when every product
  // takes the batched kernel: per-token rows of q, k, v, attOut, hb, hb2
  // (io_tokens each), the tokens' Q8_0 inputs, and their positions.
  bool many = false;
  // Independent sequences whose caches the stage holds (a batched decode
  // step, rk_stage_forward_batch): layer l's keys of sequence q start at
  // keys[l] + q·ctx·kvd, its values at vals[l] + q·kvd·v_pitch. Everything
  // else (rk_stage_forward, the decode graph, the Batch API) uses sequence 0.
  int nseq = 1;
  float *m_q = nullptr, *m_k = nullptr, *m_v = nullptr, *m_att = nullptr, *m_hb = nullptr, *m_hb2 = nullptr,
        *m_xs = nullptr;
  float *m_scores = nullptr;  // per-token score rows [io_tokens][heads][att_stride]
  int8_t *m_qx = nullptr;
  int *m_pos = nullptr, *pin_pos = nullptr;
  cudaEvent_t pos_copied = nullptr;  // the last copy out of pin_pos (recorded after it)
  // Row sharding (layer_dims): this process's rank of G; null/1 unsharded.
  rk_group *grp = nullptr;
  int G = 1, rank = 0;
  // The fused gathers (p2p): x, attOut and hb, their tagged copies (8-byte
  // words: value and tag) and the step epoch live in one allocation
  // `xbase`, mapped by every peer through CUDA IPC.
  int p2p = 0;
  // Chained products (k_matvec_chain): each layer's Wo, W1·W3, W2 and the
  // next layer's Q/K/V in one launch, handing their outputs on through the
  // tagged copies in `xbase` (on one GPU too, where the only peer is this
  // GPU). Decided when the step graph is recorded.
  int chain = 0;
  char *xbase = nullptr;
  size_t off_xll = 0, off_attll = 0, off_hbll = 0, off_epoch = 0;
  char *peer_base[kMaxPeers] = {};  // by rank; this rank's entry is xbase
};

static int stage_alloc(rk_stage *s, size_t bytes, void **p) {
  bytes = ((bytes + 255) & ~size_t(255)) + 256;
  cudaError_t e = cudaMalloc(p, bytes);
  if (e == cudaSuccess) e = cudaMemsetAsync(*p, 0, bytes, s->d->st);
  if (e != cudaSuccess) return cuda_fail(e, "stage allocation");
  s->allocs.push_back(*p);
  s->bytes += (int64_t)bytes;
  return RK_OK;
}

static void stage_release(rk_stage *s) {
  if (!s) return;
  cudaSetDevice(s->d->ordinal);
  cudaStreamSynchronize(s->d->st);
  if (s->graph) cudaGraphExecDestroy(s->graph);
  for (int g = 0; g < s->G && g < kMaxPeers; g++)
    if (s->peer_base[g] && s->peer_base[g] != s->xbase) cudaIpcCloseMemHandle(s->peer_base[g]);
  for (void *p : s->allocs) cudaFree(p);
  cudaFreeHost(s->pin_io);
  cudaFreeHost(s->pin_pos);
  if (s->pos_copied) cudaEventDestroy(s->pos_copied);
  s->d->used -= s->bytes;
  delete s;
}

// num.Recip32 (recip.go:38-67) of a positive integer-valued float, on the
// host: the Recip32(float32(n)) that rmsNorm multiplies by (model.go:633;
// gpustage.go:123-124). This file is compiled with -ffp-contract=off, so
// each operation rounds once.
static float host_recip32(float x) {
  float m = x;
  int e = 0;
  while (m >= 2.0f) {
    m = m * 0.5f;
    e++;
  }
  // float32(24.0/17) and float32(8.0/17), from the bit patterns the device
  // code uses (rk_common.cuh).
  float k24_17, k8_17;
  memcpy(&k24_17, &K_24_17, sizeof k24_17);
  memcpy(&k8_17, &K_8_17, sizeof k8_17);
  float r = k24_17 - k8_17 * m;
  for (int i = 0; i < 3; i++) {
    const float mr = m * r;
    const float t = 1.0f - mr;
    const float rt = r * t;
    r = r + rt;
  }
  return r * ldexpf(1.0f, -e);
}

// Advances a sharded stage's step epoch (the step number in the tags of its
// fused gathers' words).
__global__ void k_epoch(unsigned *epoch) {
  griddep_trigger();
  griddep_wait();
  if (threadIdx.x == 0) *epoch += 1;
}

// Records one position's pass through the stage's layers (gpustage.go:119-152
// in the order of Stage.Forward, model.go:537-611), reading the position
// from s->pos_dev. x is s->x.
// The arguments of layer li's post-processing (bias, QK-norm, RoPE, cache
// append; model.go:542-568) and attention (model.go:571-587) for one token
// whose q/k/v are given, at position *pos_dev, writing out (this rank's
// heads of attOut).
static void attention_args(const rk_stage *s, size_t li, float *q, float *k, float *v, float *out,
                           const int *pos_dev, QkvPostArgs *qp_out, AttnArgs *at_out) {
  const rk_config *c = &s->c;
  const rk_layer *l = s->layers[li];
  const float *vec = l->vecs->v;
  const int hs = head_size(c), G = s->G, heads_l = c->heads / G, kvh_l = c->kv_heads / G;
  const int h0 = s->rank * heads_l, kv0 = s->rank * kvh_l;
  QkvPostArgs qp{};
  qp.q = q;
  qp.k = k;
  qp.v = v;
  if (c->qkv_bias) {
    qp.bq = vec + l->o_bq + h0 * hs;
    qp.bk = vec + l->o_bk + kv0 * hs;
    qp.bv = vec + l->o_bv + kv0 * hs;
  }
  if (c->qk_norm) {
    qp.q_norm = vec + l->o_qn;
    qp.k_norm = vec + l->o_kn;
  }
  qp.cos_ = s->cos_;
  qp.sin_ = s->sin_;
  qp.key_cache = s->keys[li];
  qp.val_cache = s->vals[li];
  qp.v_pitch = s->v_pitch;
  qp.pos_dev = pos_dev;
  qp.heads = heads_l;
  qp.kv_heads = kvh_l;
  qp.hs = hs;
  qp.eps = cfg_eps(c);
  qp.recip_hs = host_recip32((float)hs);
  AttnArgs at{};
  at.q = q;
  at.keys = s->keys[li];
  at.vals = s->vals[li];
  at.v_pitch = s->v_pitch;
  at.att = s->att;
  at.out = out;
  at.positions_dev = pos_dev;
  at.positions_add = 1;
  at.max_positions = s->ctx;
  at.heads = heads_l;
  at.kv_heads = kvh_l;
  at.hs = hs;
  at.kv_dim = kvh_l * hs;
  at.att_stride = s->att_stride;
  at.inv_sqrt = (float)(1 / sqrt((double)hs));
  at.err = s->d->err_dev;
  *qp_out = qp;
  *at_out = at;
}

static int record_layers(rk_stage *s, cudaStream_t st) {
  rk_device *d = s->d;
  const rk_config *c = &s->c;
  const int hs = head_size(c), qd = c->heads * hs, D = c->dim, H = c->hidden;
  // This rank's part (everything when unsharded): query heads h0.., rows
  // r0.. of Wo/W2 (of D) and rH0.. of W1/W3 (of H).
  const int G = s->G, heads_l = c->heads / G;
  const int h0 = s->rank * heads_l, r0 = s->rank * (D / G), rH0 = s->rank * (H / G);
  auto gather = [&](float *buf, int total) -> int { return G > 1 ? group_gather(s->grp, buf, total / G, st) : RK_OK; };
  // Fused gathers (p2p): gather point slot = layer·4 + {0: attOut, 1: x
  // after Wo, 2: hb, 3: x after W2}. A point is fused when its producer
  // and consumer kernels both take part (quantized products that quantize
  // their own input, the single-kernel attention); the last layer's x
  // stays an NCCL all-gather, so whatever reads the stage's output reads
  // plain floats.
  auto epoch_of = [](rk_stage *st_) { return (unsigned *)(st_->xbase + st_->off_epoch); };
  unsigned *epoch = epoch_of(s);
  const int nslots = 4 * (int)s->layers.size();
  // The tagged copy of a vector (off_ll: its offset in the block) from
  // element `elem` on, in every rank's memory.
  auto put_for = [&](int slot, size_t off_ll, size_t elem) {
    GatherPut gp{};
    for (int g = 0; g < G; g++)
      gp.ll[gp.nll++] = (unsigned long long *)(s->peer_base[g] + off_ll) + elem;
    gp.epoch = epoch;
    gp.slot = slot;
    gp.nslots = nslots;
    return gp;
  };
  auto wait_for = [&](int slot, size_t off_ll) {
    GatherWait w{};
    w.ll = (const unsigned long long *)(s->xbase + off_ll);
    w.epoch = epoch;
    w.slot = slot;
    w.nslots = nslots;
    return w;
  };
  // A consumer reads a gathered input in one chunk of its prologue.
  auto fusable = [&](const rk_matrix *producer, const rk_matrix *consumer, int cols, bool norm) {
    return s->p2p && quantized_fmt(producer->fmt) && quantized_fmt(consumer->fmt) &&
           matvec_fused_ok(consumer->fmt, cols, norm) && cols <= (norm ? 8192 : 16384);
  };
  if (s->p2p) CK(launch_k(k_epoch, 1, 32, 0, st, epoch));
  const float eps = cfg_eps(c);
  const float recipD = host_recip32((float)D);
  // ms·(rmsNorm(x, norm_w) or x). A quantized product's CTAs quantize their
  // input themselves when it fits their shared memory; otherwise one
  // quantize launch fills the stage's scratch first. Float matrices get the
  // normalised input in xb.
  auto products = [&](int n, rk_matrix *const *ms, float *const *outs, const float *x, const float *norm_w, int cols,
                      int epi, const GatherPut *put = nullptr, const GatherWait *wait = nullptr) -> int {
    const float recip = host_recip32((float)cols);
    if (quantized_fmt(ms[0]->fmt)) {
      if (matvec_fused_ok(ms[0]->fmt, cols, norm_w != nullptr)) {
        Pro p;
        p.pro = norm_w ? PRO_NORM_QUANT : PRO_QUANT;
        p.norm_w = norm_w;
        p.recipN = recip;
        p.eps = eps;
        if (put) p.put = *put;
        if (wait) p.wait = *wait;
        return enqueue_matvecs(d, n, ms, outs, x, nullptr, nullptr, nullptr, epi, st, p);
      }
      // A gathered input needs the fused prologue (the gather points are
      // chosen so); the outputs still go to the peers when the point after
      // this product is fused, whatever the prologue.
      if (wait && wait->ll) return fail(RK_ERR_ARGS, "a gathered input for a product without the fused prologue");
      CK(launch_quantize_act(x, cols, norm_w, recip, eps, nullptr, s->qx, s->xs, s->xsum, st));
      Pro p;
      if (put) p.put = *put;
      return enqueue_matvecs(d, n, ms, outs, x, s->qx, s->xs, s->xsum, epi, st, p);
    }
    const float *in = x;
    if (norm_w) {
      CK(launch_rmsnorm(x, s->xb, norm_w, cols, 1, 0, recip, eps, st));
      in = s->xb;
    }
    return enqueue_matvecs(d, n, ms, outs, in, nullptr, nullptr, nullptr, epi, st);
  };
  // ---- Chained products: per layer the attention, then one launch of Wo,
  // W1·W3, W2 and the next layer's Q/K/V (layer 0's Q/K/V alone first).
  // Each step's output reaches the next through the tagged copies in the
  // stage's block (every rank's, when sharded). ----
  const int L = (int)s->layers.size();
  auto qkv_step = [&](int li, const GatherWait *w) {
    rk_layer *l = s->layers[li];
    MvArgs a{};
    a.fmt = l->wq->fmt;
    a.cols = D;
    a.epi = EPI_STORE;
    a.err = d->err_dev;
    a.part[0] = part_of(l->wq, s->q);
    a.part[1] = part_of(l->wk, s->k);
    a.part[2] = part_of(l->wv, s->v);
    a.nparts = 3;
    a.pro = PRO_NORM_QUANT;
    a.x = s->x;
    a.norm_w = l->vecs->v + l->o_rms_att;
    a.recipN = recipD;
    a.eps = eps;
    if (w) a.wait = *w;
    return a;
  };
  // The chain after layer li's attention; ok=false when some product
  // cannot take part.
  auto layer_chain = [&](int li, bool *ok) {
    rk_layer *l = s->layers[li];
    const float *vec = l->vecs->v;
    const int sl = 4 * li;
    const bool f_att = G > 1;
    ChainArgs ca{};
    MvArgs &wo = ca.step[0];
    wo.fmt = l->wo->fmt;
    wo.cols = qd;
    wo.epi = EPI_ADD;
    wo.err = d->err_dev;
    wo.part[0] = part_of(l->wo, s->x + r0);
    wo.nparts = 1;
    wo.pro = PRO_QUANT;
    wo.x = s->att_out;
    if (f_att) wo.wait = wait_for(sl, s->off_attll);
    wo.put = put_for(sl + 1, s->off_xll, r0);
    MvArgs &ff = ca.step[1];
    ff.fmt = l->w1->fmt;
    ff.cols = D;
    ff.epi = EPI_SILU;
    ff.err = d->err_dev;
    ff.part[0] = part_of(l->w1, s->hb + rH0);
    ff.part[1] = part_of(l->w3, s->hb2 + rH0);
    ff.nparts = 2;
    ff.pro = PRO_NORM_QUANT;
    ff.x = s->x;
    ff.norm_w = vec + l->o_rms_ffn;
    ff.recipN = recipD;
    ff.eps = eps;
    ff.wait = wait_for(sl + 1, s->off_xll);
    ff.put = put_for(sl + 2, s->off_hbll, rH0);
    MvArgs &w2 = ca.step[2];
    w2.fmt = l->w2->fmt;
    w2.cols = H;
    w2.epi = EPI_ADD_CANON;
    w2.err = d->err_dev;
    w2.part[0] = part_of(l->w2, s->x + r0);
    w2.nparts = 1;
    w2.pro = PRO_QUANT;
    w2.x = s->hb;
    w2.wait = wait_for(sl + 2, s->off_hbll);
    ca.nsteps = 3;
    if (li + 1 < L) {
      w2.put = put_for(sl + 3, s->off_xll, r0);
      const GatherWait wx = wait_for(sl + 3, s->off_xll);
      ca.step[3] = qkv_step(li + 1, &wx);
      ca.nsteps = 4;
    }
    // One format throughout; the W3 rows pair with W1's.
    *ok = l->w3->fmt == l->w1->fmt && matvec_chain_ok(ca, d->sms);
    for (int k = 0; k < ca.nsteps && *ok; k++)
      for (int p = 1; p < ca.step[k].nparts; p++) *ok = *ok && ca.step[k].part[p].rows > 0;
    if (li + 1 < L) {
      rk_layer *n = s->layers[li + 1];
      *ok = *ok && n->wk->fmt == n->wq->fmt && n->wv->fmt == n->wq->fmt;
    }
    return ca;
  };
  // Chains need the tagged copies on every rank: always on one GPU, and
  // with the fused gathers (peer memory mapped) when sharded; the
  // attention output of a sharded stage arrives as tagged words too.
  // They are opt-in (RK_CHAIN=1): measured on the same boxes, the
  // per-product graph, whose launches overlap through programmatic
  // dependent launch, is as fast or faster (Llama-3-8B Q8_0: 295 against
  // 292 tok/s on one B200, 359.6 against 354.6 on two, 429.6 against 407.9
  // on four).
  const char *chain_env = getenv("RK_CHAIN");
  const bool want_chain = chain_env && strcmp(chain_env, "1") == 0;
  bool chain = L > 0 && (G == 1 || (s->p2p && s->v_pitch > 0)) && want_chain;
  if (chain) {
    ChainArgs first{};
    first.step[0] = qkv_step(0, nullptr);
    first.nsteps = 1;
    rk_layer *l0 = s->layers[0];
    chain = matvec_chain_ok(first, d->sms) && l0->wk->fmt == l0->wq->fmt && l0->wv->fmt == l0->wq->fmt;
    for (int li = 0; li < L && chain; li++) {
      bool ok = false;
      layer_chain(li, &ok);
      chain = ok;
    }
    if (chain && G > 1) {
      // The sharded attention must store its output as tagged words.
      for (int li = 0; li < L && chain; li++) chain = fusable(s->layers[li]->wo, s->layers[li]->wo, qd, false);
    }
  }
  s->chain = chain ? 1 : 0;
  if (chain) {
    if (!s->p2p) CK(launch_k(k_epoch, 1, 32, 0, st, epoch_of(s)));
    ChainArgs first{};
    first.step[0] = qkv_step(0, nullptr);
    first.nsteps = 1;
    CK(launch_chain(d, first, st));
    for (int li = 0; li < L; li++) {
      QkvPostArgs qp;
      AttnArgs at;
      attention_args(s, li, s->q, s->k, s->v, s->att_out + h0 * hs, s->pos_dev, &qp, &at);
      if (G > 1) at.put = put_for(4 * li, s->off_attll, (size_t)h0 * hs);
      CK(launch_attention_post(qp, at, st));
      bool ok = false;
      const ChainArgs ca = layer_chain(li, &ok);
      CK(launch_chain(d, ca, st));
    }
    // A sharded stage's output x: every rank's rows, for whatever reads it.
    if (G > 1) return gather(s->x, D);
    return RK_OK;
  }

  for (size_t li = 0; li < s->layers.size(); li++) {
    rk_layer *l = s->layers[li];
    const float *vec = l->vecs->v;
    // q, k, v = Wq·xb, Wk·xb, Wv·xb with xb = rmsNorm(x, RmsAtt) (model.go:538-539).
    rk_matrix *qkv[3] = {l->wq, l->wk, l->wv};
    float *qkv_out[3] = {s->q, s->k, s->v};
    const int sl = 4 * (int)li;
    rk_layer *next = li + 1 < s->layers.size() ? s->layers[li + 1] : nullptr;
    const bool f_att = s->p2p && s->v_pitch > 0 && fusable(l->wo, l->wo, qd, false);
    const bool f_x1 = fusable(l->wo, l->w1, D, true);
    // The W1·W3 kernel reads x's tagged words and writes hb's; the peers
    // overwrite x's words (after W2) once they hold every hb row. That is
    // safe only when each of its CTAs owns a row, i.e. has finished reading
    // x before any peer can move on; otherwise hb goes through NCCL.
    const bool f_hb = fusable(l->w1, l->w2, H, false) && l->w1->rows >= d->sms;
    const bool f_x2 = next && fusable(l->w2, next->wq, D, true);
    const bool f_prev = li > 0 && fusable(s->layers[li - 1]->w2, l->wq, D, true);
    const GatherWait w_prev = f_prev ? wait_for(sl - 1, s->off_xll) : GatherWait{};
    int rc = products(3, qkv, qkv_out, s->x, vec + l->o_rms_att, D, EPI_STORE, nullptr, &w_prev);
    if (rc) return rc;
    // Bias, QK-norm, RoPE, cache append (model.go:542-568), then attention
    // over positions 0..pos (model.go:571-587).
    QkvPostArgs qp;
    AttnArgs at;
    attention_args(s, li, s->q, s->k, s->v, s->att_out + h0 * hs, s->pos_dev, &qp, &at);
    if (f_att) at.put = put_for(sl, s->off_attll, (size_t)h0 * hs);
    CK(launch_attention_post(qp, at, st));
    if (!f_att && (rc = gather(s->att_out, qd))) return rc;
    // x += Wo·attOut (model.go:588-594).
    {
      float *xo = s->x + r0;
      const GatherPut p1 = f_x1 ? put_for(sl + 1, s->off_xll, r0) : GatherPut{};
      const GatherWait w0 = f_att ? wait_for(sl, s->off_attll) : GatherWait{};
      if ((rc = products(1, &l->wo, &xo, s->att_out, nullptr, qd, EPI_ADD, &p1, &w0))) return rc;
    }
    if (!f_x1 && (rc = gather(s->x, D))) return rc;
    // hb = silu(W1·xb)·(W3·xb) with xb = rmsNorm(x, RmsFfn) (model.go:597-603):
    // row i of W1 and of W3 in one warp, SiLU·mul as the epilogue.
    {
      MvArgs a{};
      a.fmt = l->w1->fmt;
      a.cols = D;
      a.epi = EPI_SILU;
      a.err = d->err_dev;
      a.part[0] = part_of(l->w1, s->hb + rH0);
      a.part[1] = part_of(l->w3, s->hb2 + rH0);
      a.nparts = 2;
      const float *norm_w = vec + l->o_rms_ffn;
      if (quantized_fmt(a.fmt) && matvec_fused_ok(a.fmt, D, true)) {
        a.pro = PRO_NORM_QUANT;
        a.x = s->x;
        a.norm_w = norm_w;
        a.recipN = recipD;
        a.eps = eps;
        if (f_x1) a.wait = wait_for(sl + 1, s->off_xll);
        if (f_hb) a.put = put_for(sl + 2, s->off_hbll, rH0);
      } else if (quantized_fmt(a.fmt)) {
        if (f_x1) return fail(RK_ERR_ARGS, "a gathered input for a product without the fused prologue");
        CK(launch_quantize_act(s->x, D, norm_w, recipD, eps, nullptr, s->qx, s->xs, s->xsum, st));
        a.qx = s->qx;
        a.xs = s->xs;
        a.xsum = s->xsum;
        if (f_hb) a.put = put_for(sl + 2, s->off_hbll, rH0);  // (the epilogue stores them either way)
      } else {
        CK(launch_rmsnorm(s->x, s->xb, norm_w, D, 1, 0, recipD, eps, st));
        a.x = s->xb;
      }
      CK(launch_mv(d, a, st));
    }
    if (!f_hb && (rc = gather(s->hb, H))) return rc;
    // x = Canonical(x + W2·hb) (model.go:604-610).
    {
      float *xo = s->x + r0;
      const GatherPut p3 = f_x2 ? put_for(sl + 3, s->off_xll, r0) : GatherPut{};
      const GatherWait w2 = f_hb ? wait_for(sl + 2, s->off_hbll) : GatherWait{};
      if ((rc = products(1, &l->w2, &xo, s->hb, nullptr, H, EPI_ADD_CANON, &p3, &w2))) return rc;
    }
    if (!f_x2 && (rc = gather(s->x, D))) return rc;
  }
  return RK_OK;
}

// io[tok] -> x, or x -> io[tok] then tok += 1, pos += 1.
__global__ void k_stage_io(float *io, const int *tok, float *x, int dim, int dir) {
  griddep_trigger();
  griddep_wait();
  const long long t = *tok;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < dim; j += gridDim.x * blockDim.x) {
    if (dir == 0) x[j] = io[t * dim + j];
    else io[t * dim + j] = x[j];
  }
}
__global__ void k_advance(int *tok, int *pos) {
  griddep_trigger();
  griddep_wait();
  if (tok) *tok += 1;
  if (pos) *pos += 1;
}

// Records rec's launches into a graph; *nodes receives the number of this
// library's kernels in it (collectives are not counted).
static int capture(rk_device *d, std::function<int(cudaStream_t)> rec, cudaGraphExec_t *out, size_t *nodes = nullptr) {
  cudaGraph_t graph = nullptr;
  CK(cudaStreamBeginCapture(d->st, cudaStreamCaptureModeThreadLocal));
  // Kernels of a captured step use programmatic dependent launch: each may
  // start (and stream its weights) while its predecessor finishes.
  g_pdl = true;
  const long long k0 = g_kernel_launches;
  int rc = rec(d->st);
  g_pdl = false;
  if (nodes) *nodes = (size_t)(g_kernel_launches - k0);
  cudaError_t e = cudaStreamEndCapture(d->st, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(e, "graph capture");
  e = cudaGraphInstantiate(out, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return cuda_fail(e, "graph instantiate");
  return RK_OK;
}

// Maps every peer's exchange block (CUDA IPC; the handles and device
// ordinals travel through the group) when every peer is reachable by P2P,
// so that the stage's gathers can be fused into its kernels; otherwise (or
// with RK_GATHER=nccl) they stay NCCL all-gathers. Collective.
static int stage_p2p_setup(rk_stage *s) {
  const int G = s->G;
  s->peer_base[s->rank] = s->xbase;
  if (G > kMaxPeers) return RK_OK;
  const char *env = getenv("RK_GATHER");
  const bool want = !(env && strcmp(env, "nccl") == 0);
  struct Entry {
    cudaIpcMemHandle_t h;
    int ordinal, ok, pad[2];
  };
  static_assert(sizeof(Entry) % 4 == 0, "entry");
  constexpr int kFloats = sizeof(Entry) / 4;
  Entry mine{};
  mine.ordinal = s->d->ordinal;
  mine.ok = want && cudaIpcGetMemHandle(&mine.h, s->xbase) == cudaSuccess;
  cudaGetLastError();
  float *buf = nullptr;
  std::vector<Entry> all(G);
  CK(cudaMalloc(&buf, sizeof(Entry) * G));
  cudaError_t e = cudaMemcpy(buf + s->rank * kFloats, &mine, sizeof mine, cudaMemcpyHostToDevice);
  int rc = e == cudaSuccess ? group_gather(s->grp, buf, kFloats, s->d->st) : cuda_fail(e, "peer exchange");
  if (!rc) {
    e = cudaStreamSynchronize(s->d->st);
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), buf, sizeof(Entry) * G, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) rc = cuda_fail(e, "peer exchange");
  }
  cudaFree(buf);
  if (rc) return rc;
  bool ok = true;
  for (int g = 0; g < G; g++) {
    int can = 0;
    ok = ok && all[g].ok;
    if (g != s->rank && ok) ok = cudaDeviceCanAccessPeer(&can, s->d->ordinal, all[g].ordinal) == cudaSuccess && can;
  }
  // Every rank decides alike: all must have published a handle and see all peers.
  for (int g = 0; g < G && ok; g++) {
    if (g == s->rank) continue;
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, all[g].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = false;
      break;
    }
    s->peer_base[g] = (char *)p;
  }
  // Agree: fused gathers only if every rank mapped every peer.
  {
    float *fl = nullptr;
    std::vector<float> oks(G);
    const float me = ok ? 1.0f : 0.0f;
    CK(cudaMalloc(&fl, 4 * G));
    e = cudaMemcpy(fl + s->rank, &me, 4, cudaMemcpyHostToDevice);
    rc = e == cudaSuccess ? group_gather(s->grp, fl, 1, s->d->st) : cuda_fail(e, "peer agreement");
    if (!rc) {
      e = cudaStreamSynchronize(s->d->st);
      if (e == cudaSuccess) e = cudaMemcpy(oks.data(), fl, 4 * G, cudaMemcpyDeviceToHost);
      if (e != cudaSuccess) rc = cuda_fail(e, "peer agreement");
    }
    cudaFree(fl);
    if (rc) return rc;
    for (int g = 0; g < G; g++) ok = ok && oks[g] == 1.0f;
  }
  if (!ok) {
    for (int g = 0; g < G; g++)
      if (g != s->rank && s->peer_base[g]) {
        cudaIpcCloseMemHandle(s->peer_base[g]);
        s->peer_base[g] = nullptr;
      }
    cudaGetLastError();
  }
  s->p2p = ok ? 1 : 0;
  return RK_OK;
}

// Whether ForwardMany can run the stage's layers with batched products:
// unsharded, every matrix Q8_0 or Q4_0 and taken by the batched kernel.
static bool stage_many_ok(const rk_stage *s) {
  if (s->G != 1 || s->layers.empty()) return false;
  for (const rk_layer *l : s->layers)
    for (const rk_matrix *m : {l->wq, l->wk, l->wv, l->wo, l->w1, l->w3, l->w2})
      if (!mv_many_ok(m->fmt, m->rows, m->cols, m->w, m->s)) return false;
  return true;
}

// The batched attention's arguments for layer li, token 0 of a submission
// (per-token strides set). per_seq: token t belongs to sequence t (its own
// caches), else all tokens are one sequence's consecutive positions.
static void attention_many_args(const rk_stage *s, size_t li, bool per_seq, int max_positions, QkvPostArgs *qp,
                                AttnArgs *at) {
  const rk_config *c = &s->c;
  const int hs = head_size(c), qd = c->heads * hs, kvd = c->kv_heads * hs;
  attention_args(s, li, s->m_q, s->m_k, s->m_v, s->m_att, s->m_pos, qp, at);
  qp->tok_q = at->tok_q = at->tok_out = qd;
  qp->tok_kv = kvd;
  at->att = s->m_scores;
  at->tok_att = (long long)c->heads * s->att_stride;
  at->max_positions = max_positions;
  if (per_seq) {
    qp->tok_keys = at->tok_keys = (long long)s->ctx * kvd;
    qp->tok_vals = at->tok_vals = (long long)kvd * (s->v_pitch > 0 ? s->v_pitch : s->ctx);
  }
}

// Stage.ForwardMany (model.go:504-518) for the nt tokens in s->io at
// positions pos.., layer by layer. Each projection runs once for all nt
// tokens on the tensor cores (launch_mv_many); the bias / QK-norm / RoPE /
// cache append and the attention run token after token in position order,
// so token t's attention reads the cache rows appended before it, as the
// reference's token-by-token Forward does. Every element is computed by the
// same operations in the same order as in Forward.
//
// per_seq (a batched decode step, rk_stage_forward_batch): token t is the
// next token of sequence t, at position positions[t], with its own caches;
// every token's arithmetic is still the reference's Forward for that
// sequence.
static int stage_forward_many(rk_stage *s, const int *positions, int nt, bool per_seq) {
  rk_device *d = s->d;
  const rk_config *c = &s->c;
  cudaStream_t st = d->st;
  const int hs = head_size(c), qd = c->heads * hs, kvd = c->kv_heads * hs, D = c->dim, H = c->hidden;
  const float eps = cfg_eps(c), recipD = host_recip32((float)D);
  int max_pos = 0;
  // Submissions may be queued back to back (rk_model_generate's prompt):
  // the previous one's copy out of pin_pos must have run before the host
  // rewrites it, or that submission would see these positions.
  CK(cudaEventSynchronize(s->pos_copied));
  for (int t = 0; t < nt; t++) {
    s->pin_pos[t] = positions[t];
    max_pos = std::max(max_pos, positions[t] + 1);
  }
  CK(cudaMemcpyAsync(s->m_pos, s->pin_pos, sizeof(int) * nt, cudaMemcpyHostToDevice, st));
  CK(cudaEventRecord(s->pos_copied, st));
  // Up to three matrices that share the quantized input, in one launch
  // per format (a mixed-format model's Q4_0 and Q8_0 matrices apart).
  const auto products = [&](int cols, std::initializer_list<MmMat> mats) {
    for (const int fmt : {FMT_Q8_0, FMT_Q4_0}) {
      MmMat same[kMmMaxMats];
      int n = 0;
      for (const MmMat &m : mats)
        if (m.fmt == fmt) same[n++] = m;
      if (n == 0) continue;
      const cudaError_t e = launch_mv_many(n, same, cols, nt, s->m_qx, s->m_xs, s->io_tokens, d->err_dev, d->sms, st);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  };
  const auto mat = [](const rk_matrix *m, float *out, long long stride, int epi) {
    return MmMat{m->w, m->s, m->rows, out, stride, epi, m->fmt};
  };
  float *X = s->io;
  // When the attention runs batched, every kernel of the submission reads
  // its predecessor's results only after griddepcontrol.wait, so they are
  // launched with programmatic dependent launch, as a captured decode step
  // is: each starts while its predecessor finishes. The token-by-token
  // attention is launched without it: its fused scores kernel copies key
  // rows before that wait, which is safe only after the previous token's
  // kernels have completed.
  bool batched_attention = false;
  {
    QkvPostArgs qp;
    AttnArgs at;
    attention_many_args(s, 0, per_seq, max_pos, &qp, &at);
    batched_attention = attention_many_ok(at);
  }
  if (per_seq && !batched_attention) return fail(RK_ERR_ARGS, "batched decode needs the batched attention kernels");
  struct PdlScope {
    bool old;
    explicit PdlScope(bool on) : old(g_pdl) { g_pdl = on; }
    ~PdlScope() { g_pdl = old; }
  } pdl_scope(batched_attention);
  for (size_t li = 0; li < s->layers.size(); li++) {
    const rk_layer *l = s->layers[li];
    const float *vec = l->vecs->v;
    // q, k, v = Wq·xb, Wk·xb, Wv·xb with xb = rmsNorm(x, RmsAtt) (model.go:538-539).
    CK(launch_quantize_many(X, nt, D, vec + l->o_rms_att, recipD, eps, s->m_qx, s->m_xs, s->io_tokens, st));
    CK(products(D, {mat(l->wq, s->m_q, qd, EPI_STORE), mat(l->wk, s->m_k, kvd, EPI_STORE),
                    mat(l->wv, s->m_v, kvd, EPI_STORE)}));
    // Bias, QK-norm, RoPE, cache append and attention (model.go:542-587):
    // all tokens' appends, then all tokens' attention, in three launches;
    // shapes the batched kernels do not take go token by token.
    QkvPostArgs qp;
    AttnArgs at;
    attention_many_args(s, li, per_seq, max_pos, &qp, &at);
    if (batched_attention) {
      CK(launch_attention_many(qp, at, nt, st));
    } else {
      for (int t = 0; t < nt; t++) {
        attention_args(s, li, s->m_q + (size_t)t * qd, s->m_k + (size_t)t * kvd, s->m_v + (size_t)t * kvd,
                       s->m_att + (size_t)t * qd, s->m_pos + t, &qp, &at);
        CK(launch_attention_post(qp, at, st));
      }
    }
    // x += Wo·attOut (model.go:588-594).
    CK(launch_quantize_many(s->m_att, nt, qd, nullptr, 0.0f, 0.0f, s->m_qx, s->m_xs, s->io_tokens, st));
    CK(products(qd, {mat(l->wo, X, D, EPI_ADD)}));
    // hb = silu(W1·xb)·(W3·xb) with xb = rmsNorm(x, RmsFfn) (model.go:597-603).
    CK(launch_quantize_many(X, nt, D, vec + l->o_rms_ffn, recipD, eps, s->m_qx, s->m_xs, s->io_tokens, st));
    CK(products(D, {mat(l->w1, s->m_hb, H, EPI_STORE), mat(l->w3, s->m_hb2, H, EPI_STORE)}));
    CK(launch_silu_mul_many(s->m_hb, s->m_hb2, (long long)nt * H, d->sms, st));
    // x = Canonical(x + W2·hb) (model.go:604-610).
    CK(launch_quantize_many(s->m_hb, nt, H, nullptr, 0.0f, 0.0f, s->m_qx, s->m_xs, s->io_tokens, st));
    CK(products(H, {mat(l->w2, X, D, EPI_ADD_CANON)}));
  }
  return RK_OK;
}

static int stage_new(rk_device *d, const rk_config *c, rk_layer *const *layers, int n, int ctx, rk_group *grp,
                     rk_stage **out, int nseq = 1) {
  if (!d || !c || !out || n < 0 || (n > 0 && !layers) || ctx <= 0) return fail(RK_ERR_ARGS, "bad argument");
  int rc = rk_config_validate(c);
  if (rc) return rc;
  ctx = std::min(ctx, c->seq_len);
  const int G = grp ? grp->n : 1, rank = grp ? grp->rank : 0;
  if (grp && grp->d != d) return fail(RK_ERR_ARGS, "group on another device");
  int dims[7][2];
  if ((rc = layer_dims(c, G, dims))) return rc;
  for (int i = 0; i < n; i++) {
    if (!layers[i] || layers[i]->d != d) return fail(RK_ERR_ARGS, "layer %d not on this device", i);
    if (layers[i]->nshards != G || layers[i]->shard != rank)
      return fail(RK_ERR_ARGS, "layer %d is shard %d of %d, the stage is rank %d of %d", i, layers[i]->shard,
                  layers[i]->nshards, rank, G);
  }
  Guard g(d);
  if ((rc = set_device(d))) return rc;
  auto *s = new rk_stage();
  s->d = d;
  s->c = *c;
  s->layers.assign(layers, layers + n);
  s->ctx = ctx;
  s->grp = grp;
  s->G = G;
  s->rank = rank;
  s->nseq = nseq;
  const int hs = head_size(c), qd = c->heads * hs, kvd = c->kv_heads * hs / G, D = c->dim, H = c->hidden;
  const int widest = std::max(D, std::max(qd, H));
  void *p;
  auto A = [&](size_t bytes, void **dst) { return stage_alloc(s, bytes, dst); };
#define ALLOC(field, bytes)                   \
  do {                                        \
    if ((rc = A((bytes), &p))) goto fail_;    \
    s->field = (decltype(s->field))p;         \
  } while (0)
  {
    // The gathered (or chained) activations, their tagged copies and the
    // epoch in one block.
    auto a16 = [](size_t b) { return (b + 15) & ~size_t(15); };
    const size_t ox = 0, oatt = ox + a16(4 * (size_t)D), ohb = oatt + a16(4 * (size_t)qd);
    s->off_xll = ohb + a16(4 * (size_t)H);
    s->off_attll = s->off_xll + a16(8 * (size_t)D);
    s->off_hbll = s->off_attll + a16(8 * (size_t)qd);
    s->off_epoch = s->off_hbll + a16(8 * (size_t)H);
    if ((rc = A(s->off_epoch + 16, &p))) goto fail_;
    s->xbase = (char *)p;
    s->x = (float *)(s->xbase + ox);
    s->att_out = (float *)(s->xbase + oatt);
    s->hb = (float *)(s->xbase + ohb);
    // (stage_alloc zeroes it: tags of epoch 0, which no step uses, since
    // the step graph advances the epoch first.)
    s->peer_base[s->rank] = s->xbase;
  }
  ALLOC(xb, 4 * (size_t)D);
  ALLOC(q, 4 * (size_t)(qd / G));
  ALLOC(k, 4 * (size_t)kvd);
  ALLOC(v, 4 * (size_t)kvd);
  ALLOC(hb2, 4 * (size_t)H);
  s->att_stride = (ctx + 3) & ~3;
  s->v_pitch = attention_fused_ok(c->heads / G, c->kv_heads / G, hs, ctx) ? s->att_stride : 0;
  ALLOC(att, 4 * (size_t)(c->heads / G) * s->att_stride);
  ALLOC(qx, (size_t)widest);
  ALLOC(xs, 4 * (size_t)(widest / 32 + 1));
  ALLOC(xsum, 4 * (size_t)(widest / 32 + 1));
  ALLOC(cos_, 4 * (size_t)ctx * (hs / 2));
  ALLOC(sin_, 4 * (size_t)ctx * (hs / 2));
  ALLOC(io, 4 * (size_t)s->io_tokens * D);
  ALLOC(pos_dev, 4);
  ALLOC(tok_dev, 4);
  for (int i = 0; i < n; i++) {
    if ((rc = A(4 * (size_t)nseq * ctx * kvd, &p))) goto fail_;
    s->keys.push_back((float *)p);
    if ((rc = A(4 * (size_t)nseq * (s->v_pitch > 0 ? s->v_pitch : ctx) * kvd, &p))) goto fail_;
    s->vals.push_back((float *)p);
  }
  s->many = stage_many_ok(s);
  if (s->many) {
    const size_t T = (size_t)s->io_tokens;
    ALLOC(m_q, 4 * T * qd);
    ALLOC(m_k, 4 * T * kvd);
    ALLOC(m_v, 4 * T * kvd);
    ALLOC(m_att, 4 * T * qd);
    ALLOC(m_hb, 4 * T * H);
    ALLOC(m_hb2, 4 * T * H);
    ALLOC(m_qx, T * widest);
    ALLOC(m_xs, 4 * T * (widest / 32));
    ALLOC(m_pos, 4 * T);
    ALLOC(m_scores, 4 * T * c->heads * s->att_stride);
    cudaError_t e = cudaMallocHost(&s->pin_pos, 4 * T);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->pos_copied, cudaEventDisableTiming);
    if (e != cudaSuccess) {
      rc = cuda_fail(e, "stage staging");
      goto fail_;
    }
  }
  if (nseq > 1) {
    QkvPostArgs qp;
    AttnArgs at;
    if (nseq > s->io_tokens || !s->many || (attention_many_args(s, 0, true, ctx, &qp, &at), !attention_many_ok(at))) {
      rc = fail(RK_ERR_ARGS,
                "a stage of %d sequences needs at most %d of them, an unsharded all-Q8_0 stage whose widths are "
                "multiples of 128, and head width 64 or 128",
                nseq, s->io_tokens);
      goto fail_;
    }
  }
#undef ALLOC
  {
    cudaError_t e = cudaMallocHost(&s->pin_io, 4 * (size_t)s->io_tokens * D);
    if (e != cudaSuccess) {
      rc = cuda_fail(e, "stage staging");
      goto fail_;
    }
    const double theta = c->rope_theta > 0 ? c->rope_theta : 10000.0;
    e = launch_rope_table(theta, hs, ctx, s->cos_, s->sin_, d->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
    if (e != cudaSuccess) {
      rc = cuda_fail(e, "rope table");
      goto fail_;
    }
  }
  if (G > 1 && (rc = stage_p2p_setup(s))) goto fail_;
  d->used += s->bytes;
  rc = capture(
      d,
      [s, D](cudaStream_t st) {
        CK(launch_k(k_stage_io, (D + 255) / 256, 256, 0, st, s->io, (const int *)s->tok_dev, s->x, D, 0));
        int r = record_layers(s, st);
        if (r) return r;
        CK(launch_k(k_stage_io, (D + 255) / 256, 256, 0, st, s->io, (const int *)s->tok_dev, s->x, D, 1));
        CK(launch_k(k_advance, 1, 1, 0, st, s->tok_dev, s->pos_dev));
        CK(cudaGetLastError());
        return RK_OK;
      },
      &s->graph);
  if (rc) {
    stage_release(s);
    return rc;
  }
  *out = s;
  return RK_OK;
fail_:
  d->used += s->bytes;
  stage_release(s);
  return rc;
}

extern "C" int rk_stage_new(rk_device *d, const rk_config *c, rk_layer *const *layers, int n, int ctx, rk_stage **out) {
  return stage_new(d, c, layers, n, ctx, nullptr, out);
}

extern "C" int rk_stage_fused_gathers(const rk_stage *s) { return s && s->G > 1 ? s->p2p : 0; }
extern "C" int rk_stage_chained(const rk_stage *s) { return s ? s->chain : 0; }

extern "C" int rk_stage_new_group(rk_device *d, const rk_config *c, rk_layer *const *layers, int n, int ctx,
                                  rk_group *g, rk_stage **out) {
  if (!g) return fail(RK_ERR_ARGS, "null group");
  return stage_new(d, c, layers, n, ctx, g, out);
}

extern "C" void rk_stage_free(rk_stage *s) {
  if (!s) return;
  rk_device *d = s->d;
  Guard g(d);
  stage_release(s);
}

extern "C" int rk_stage_positions(const rk_stage *s) { return s ? s->ctx : 0; }

extern "C" int rk_stage_batched(const rk_stage *s) { return s && s->many ? 1 : 0; }

extern "C" int rk_stage_new_batch(rk_device *d, const rk_config *c, rk_layer *const *layers, int n, int ctx, int nseq,
                                  rk_stage **out) {
  if (nseq < 1) return fail(RK_ERR_ARGS, "bad sequence count %d", nseq);
  return stage_new(d, c, layers, n, ctx, nullptr, out, nseq);
}

extern "C" int rk_stage_forward_batch(rk_stage *s, float *xs, const int *positions, int nseq) {
  if (!s || nseq < 0 || (nseq > 0 && (!xs || !positions))) return fail(RK_ERR_ARGS, "bad argument");
  if (nseq > s->nseq) return fail(RK_ERR_ARGS, "%d sequences on a stage of %d", nseq, s->nseq);
  if (nseq == 0) return RK_OK;
  for (int q = 0; q < nseq; q++)
    if (positions[q] < 0 || positions[q] >= s->ctx)
      return fail(RK_ERR_ARGS, "position %d of sequence %d outside the stage's %d", positions[q], q, s->ctx);
  if (s->nseq == 1) return rk_stage_forward(s, xs, positions[0], 1);
  rk_device *d = s->d;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  const size_t bytes = sizeof(float) * (size_t)nseq * s->c.dim;
  memcpy(s->pin_io, xs, bytes);
  CK(cudaMemcpyAsync(s->io, s->pin_io, bytes, cudaMemcpyHostToDevice, d->st));
  if ((rc = stage_forward_many(s, positions, nseq, true))) return rc;
  CK(cudaMemcpyAsync(s->pin_io, s->io, bytes, cudaMemcpyDeviceToHost, d->st));
  if ((rc = sync_dev(d))) return rc;
  memcpy(xs, s->pin_io, bytes);
  return RK_OK;
}

extern "C" int rk_stage_forward(rk_stage *s, float *xs, int pos, int tokens) {
  if (!s || (tokens > 0 && !xs) || tokens < 0) return fail(RK_ERR_ARGS, "bad argument");
  if (pos < 0 || pos + tokens > s->ctx) return fail(RK_ERR_ARGS, "positions [%d, %d) outside the stage's %d", pos, pos + tokens, s->ctx);
  rk_device *d = s->d;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  const int D = s->c.dim;
  for (int start = 0; start < tokens; start += s->io_tokens) {
    const int nt = std::min(s->io_tokens, tokens - start);
    memcpy(s->pin_io, xs + (size_t)start * D, sizeof(float) * (size_t)nt * D);
    CK(cudaMemcpyAsync(s->io, s->pin_io, sizeof(float) * (size_t)nt * D, cudaMemcpyHostToDevice, d->st));
    if (s->many && nt > 1) {
      int positions[64];
      for (int t = 0; t < nt; t++) positions[t] = pos + start + t;
      if ((rc = stage_forward_many(s, positions, nt, false))) return rc;
    } else {
      const int hdr[2] = {0, pos + start};
      CK(cudaMemcpyAsync(s->tok_dev, &hdr[0], sizeof(int), cudaMemcpyHostToDevice, d->st));
      CK(cudaMemcpyAsync(s->pos_dev, &hdr[1], sizeof(int), cudaMemcpyHostToDevice, d->st));
      for (int t = 0; t < nt; t++) CK(cudaGraphLaunch(s->graph, d->st));
    }
    CK(cudaMemcpyAsync(s->pin_io, s->io, sizeof(float) * (size_t)nt * D, cudaMemcpyDeviceToHost, d->st));
    if ((rc = sync_dev(d))) return rc;
    memcpy(xs + (size_t)start * D, s->pin_io, sizeof(float) * (size_t)nt * D);
  }
  return RK_OK;
}

// ---------------------------------------------------------------------------
// Head, Embed
// ---------------------------------------------------------------------------
struct rk_head {
  rk_device *d = nullptr;
  rk_config c{};
  rk_matrix *wcls = nullptr;  // not owned
  float *rms = nullptr, *x = nullptr, *xb = nullptr, *xs = nullptr, *logits = nullptr;
  int8_t *qx = nullptr;
  int *xsum = nullptr;
  float *pin = nullptr;
  int64_t bytes = 0;
  rk_group *grp = nullptr;  // sharded: wcls holds rows [rank·V/G, …) and the logits are gathered
};

static void head_release(rk_head *h) {
  if (!h) return;
  cudaSetDevice(h->d->ordinal);
  cudaStreamSynchronize(h->d->st);
  for (void *p : {(void *)h->rms, (void *)h->x, (void *)h->xb, (void *)h->xs, (void *)h->logits, (void *)h->qx,
                  (void *)h->xsum})
    cudaFree(p);
  cudaFreeHost(h->pin);
  h->d->used -= h->bytes;
  delete h;
}

static int head_new(rk_device *d, const rk_config *c, const float *rms_final, rk_matrix *wcls, rk_group *grp,
                    rk_head **out) {
  if (!d || !c || !rms_final || !wcls || !out) return fail(RK_ERR_ARGS, "null argument");
  int rc = rk_config_validate(c);
  if (rc) return rc;
  const int G = grp ? grp->n : 1;
  if (c->vocab % G) return fail(RK_ERR_ARGS, "cannot shard vocabulary %d over %d", c->vocab, G);
  if (wcls->d != d || wcls->rows != c->vocab / G || wcls->cols != c->dim)
    return fail(RK_ERR_ARGS, "classifier of the wrong shape");
  if (grp && grp->d != d) return fail(RK_ERR_ARGS, "group on another device");
  Guard g(d);
  if ((rc = set_device(d))) return rc;
  auto *h = new rk_head();
  h->d = d;
  h->c = *c;
  h->wcls = wcls;
  h->grp = grp;
  const size_t D = (size_t)c->dim, V = (size_t)c->vocab;
  cudaError_t e = cudaMalloc(&h->rms, 4 * D);
  if (e == cudaSuccess) e = cudaMalloc(&h->x, 4 * D);
  if (e == cudaSuccess) e = cudaMalloc(&h->xb, 4 * D);
  if (e == cudaSuccess) e = cudaMalloc(&h->xs, 4 * (D / 32 + 1));
  if (e == cudaSuccess) e = cudaMalloc(&h->xsum, 4 * (D / 32 + 1));
  if (e == cudaSuccess) e = cudaMalloc(&h->qx, D + 16);
  if (e == cudaSuccess) e = cudaMalloc(&h->logits, 4 * V);
  if (e == cudaSuccess) e = cudaMallocHost(&h->pin, 4 * std::max(D, V));
  if (e == cudaSuccess) e = cudaMemcpy(h->rms, rms_final, 4 * D, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    head_release(h);
    return cuda_fail(e, "head allocation");
  }
  h->bytes = (int64_t)(4 * D * 3 + 8 * (D / 32 + 1) + D + 16 + 4 * V);
  d->used += h->bytes;
  *out = h;
  return RK_OK;
}

extern "C" int rk_head_new(rk_device *d, const rk_config *c, const float *rms_final, rk_matrix *wcls, rk_head **out) {
  return head_new(d, c, rms_final, wcls, nullptr, out);
}

extern "C" int rk_head_new_group(rk_device *d, const rk_config *c, const float *rms_final, rk_matrix *wcls,
                                 rk_group *g, rk_head **out) {
  if (!g) return fail(RK_ERR_ARGS, "null group");
  return head_new(d, c, rms_final, wcls, g, out);
}

extern "C" void rk_head_free(rk_head *h) {
  if (!h) return;
  rk_device *d = h->d;
  Guard g(d);
  head_release(h);
}

// rmsNorm(xn, x, RmsFinal) then Wcls·xn into h->logits (model.go:667-673).
static int record_head(rk_head *h, const float *x, cudaStream_t st) {
  const int D = h->c.dim;
  const float recipD = host_recip32((float)D);
  const float eps = cfg_eps(&h->c);
  MvArgs a{};
  a.fmt = h->wcls->fmt;
  a.cols = D;
  a.epi = EPI_STORE;
  a.err = h->d->err_dev;
  if (quantized_fmt(h->wcls->fmt) && matvec_fused_ok(h->wcls->fmt, D, true)) {
    // Every CTA computes rmsNorm + quantize8 of x itself.
    a.pro = PRO_NORM_QUANT;
    a.x = x;
    a.norm_w = h->rms;
    a.recipN = recipD;
    a.eps = eps;
  } else if (quantized_fmt(h->wcls->fmt)) {
    CK(launch_quantize_act(x, D, h->rms, recipD, eps, nullptr, h->qx, h->xs, h->xsum, st));
    a.qx = h->qx;
    a.xs = h->xs;
    a.xsum = h->xsum;
  } else {
    CK(launch_rmsnorm(x, h->xb, h->rms, D, 1, 0, recipD, eps, st));
    a.x = h->xb;
  }
  const int G = h->grp ? h->grp->n : 1;
  a.part[0] = part_of(h->wcls, h->logits + (size_t)(h->grp ? h->grp->rank : 0) * (h->c.vocab / G));
  a.nparts = 1;
  CK(launch_mv(h->d, a, st));
  if (G > 1) return group_gather(h->grp, h->logits, (size_t)(h->c.vocab / G), st);
  return RK_OK;
}

extern "C" int rk_head_logits(rk_head *h, const float *x, float *logits) {
  if (!h || !x || !logits) return fail(RK_ERR_ARGS, "null argument");
  rk_device *d = h->d;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  const int D = h->c.dim, V = h->c.vocab;
  memcpy(h->pin, x, 4 * (size_t)D);
  CK(cudaMemcpyAsync(h->x, h->pin, 4 * (size_t)D, cudaMemcpyHostToDevice, d->st));
  if ((rc = record_head(h, h->x, d->st))) return rc;
  CK(cudaMemcpyAsync(h->pin, h->logits, 4 * (size_t)V, cudaMemcpyDeviceToHost, d->st));
  if ((rc = sync_dev(d))) return rc;
  memcpy(logits, h->pin, 4 * (size_t)V);
  return RK_OK;
}

extern "C" int rk_embed(rk_matrix *table, int token, float *x) {
  if (!table || !x) return fail(RK_ERR_ARGS, "null argument");
  if (token < 0 || token >= table->rows) return fail(RK_ERR_ARGS, "token %d outside the table's %d rows", token, table->rows);
  rk_device *d = table->d;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  memcpy(d->pin_in, &token, sizeof token);
  CK(cudaMemcpyAsync(d->mv_xsum, d->pin_in, sizeof(int), cudaMemcpyHostToDevice, d->st));
  CK(launch_embed(table->fmt, table->w, table->s, table->rows, table->cols, d->mv_xsum, d->mv_x, d->err_dev, d->st));
  CK(cudaMemcpyAsync(d->pin_out, d->mv_x, 4 * (size_t)table->cols, cudaMemcpyDeviceToHost, d->st));
  if ((rc = sync_dev(d))) return rc;
  memcpy(x, d->pin_out, 4 * (size_t)table->cols);
  return RK_OK;
}

// ---------------------------------------------------------------------------
// Whole-model decode
// ---------------------------------------------------------------------------
struct rk_model {
  rk_device *d = nullptr;
  rk_matrix *embed = nullptr;
  rk_stage *stage = nullptr;
  rk_head *head = nullptr;
  int *token_dev = nullptr, *next_dev = nullptr;
  int *prompt_dev = nullptr;  // a batched prompt chunk's tokens (64)
  unsigned long long *key_dev = nullptr;  // argmax key (0 between steps)
  int *pin_tok = nullptr;
  float *pin_logits = nullptr;
  cudaGraphExec_t graph = nullptr;
  int launches = 0;
};

__global__ void k_feed_token(const int *next, int *token) {
  griddep_trigger();
  griddep_wait();
  *token = *next;
}

static int record_model(rk_model *m, cudaStream_t st) {
  rk_stage *s = m->stage;
  CK(launch_embed(m->embed->fmt, m->embed->w, m->embed->s, m->embed->rows, s->c.dim, m->token_dev, s->x,
                  m->d->err_dev, st));
  int rc = record_layers(s, st);
  if (rc) return rc;
  if ((rc = record_head(m->head, s->x, st))) return rc;
  CK(launch_argmax_multi(m->head->logits, s->c.vocab, m->key_dev, m->next_dev, m->token_dev, st));
  CK(launch_k(k_advance, 1, 1, 0, st, (int *)nullptr, s->pos_dev));
  CK(cudaGetLastError());
  return RK_OK;
}

static void model_release(rk_model *m) {
  if (!m) return;
  cudaSetDevice(m->d->ordinal);
  cudaStreamSynchronize(m->d->st);
  if (m->graph) cudaGraphExecDestroy(m->graph);
  cudaFree(m->token_dev);
  cudaFree(m->prompt_dev);
  cudaFree(m->next_dev);
  cudaFree(m->key_dev);
  cudaFreeHost(m->pin_tok);
  cudaFreeHost(m->pin_logits);
  delete m;
}

extern "C" int rk_model_new(rk_device *d, rk_matrix *embed, rk_stage *stage, rk_head *head, rk_model **out) {
  if (!d || !embed || !stage || !head || !out) return fail(RK_ERR_ARGS, "null argument");
  if (embed->d != d || stage->d != d || head->d != d) return fail(RK_ERR_ARGS, "model parts on different devices");
  if (embed->rows != stage->c.vocab || embed->cols != stage->c.dim) return fail(RK_ERR_ARGS, "embedding table of the wrong shape");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  auto *m = new rk_model();
  m->d = d;
  m->embed = embed;
  m->stage = stage;
  m->head = head;
  // The graph embeds *token_dev (argmax writes the next one at the end of a
  // step), so a replay before any rk_model_step starts from token 0.
  cudaError_t e = cudaMalloc(&m->token_dev, 16);
  if (e == cudaSuccess) e = cudaMemset(m->token_dev, 0, 16);
  if (e == cudaSuccess) e = cudaMalloc(&m->key_dev, 16);
  if (e == cudaSuccess) e = cudaMemset(m->key_dev, 0, 16);
  if (e == cudaSuccess) e = cudaMalloc(&m->next_dev, 16);
  if (e == cudaSuccess) e = cudaMemset(m->next_dev, 0, 16);
  if (e == cudaSuccess) e = cudaMalloc(&m->prompt_dev, sizeof(int) * 64);
  if (e == cudaSuccess) e = cudaMallocHost(&m->pin_tok, 64);
  if (e == cudaSuccess) e = cudaMallocHost(&m->pin_logits, 4 * (size_t)stage->c.vocab);
  if (e != cudaSuccess) {
    model_release(m);
    return cuda_fail(e, "model allocation");
  }
  size_t nodes = 0;
  if ((rc = capture(d, [m](cudaStream_t st) { return record_model(m, st); }, &m->graph, &nodes))) {
    model_release(m);
    return rc;
  }
  m->launches = (int)nodes;
  *out = m;
  return RK_OK;
}

extern "C" void rk_model_free(rk_model *m) {
  if (!m) return;
  rk_device *d = m->d;
  Guard g(d);
  model_release(m);
}

extern "C" int rk_model_kernel_count(rk_model *m, int *launches_per_step) {
  if (!m || !launches_per_step) return fail(RK_ERR_ARGS, "null argument");
  *launches_per_step = m->launches;
  return RK_OK;
}

extern "C" int rk_model_step(rk_model *m, int token, int pos, float *logits, int *next) {
  if (!m) return fail(RK_ERR_ARGS, "null model");
  rk_stage *s = m->stage;
  if (pos < 0 || pos >= s->ctx) return fail(RK_ERR_ARGS, "position %d outside the stage's %d", pos, s->ctx);
  if (token < 0 || token >= s->c.vocab) return fail(RK_ERR_ARGS, "token %d outside the vocabulary", token);
  rk_device *d = m->d;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  m->pin_tok[0] = token;
  m->pin_tok[1] = pos;
  CK(cudaMemcpyAsync(m->token_dev, &m->pin_tok[0], 4, cudaMemcpyHostToDevice, d->st));
  CK(cudaMemcpyAsync(s->pos_dev, &m->pin_tok[1], 4, cudaMemcpyHostToDevice, d->st));
  CK(cudaGraphLaunch(m->graph, d->st));
  if (logits) CK(cudaMemcpyAsync(m->pin_logits, m->head->logits, 4 * (size_t)s->c.vocab, cudaMemcpyDeviceToHost, d->st));
  CK(cudaMemcpyAsync(&m->pin_tok[2], m->next_dev, 4, cudaMemcpyDeviceToHost, d->st));
  if ((rc = sync_dev(d))) return rc;
  if (logits) memcpy(logits, m->pin_logits, 4 * (size_t)s->c.vocab);
  if (next) *next = m->pin_tok[2];
  return RK_OK;
}

extern "C" int rk_model_generate(rk_model *m, const int *prompt, int n_prompt, int n_new, int *out_tokens,
                                 float *out_logits) {
  if (!m || !prompt || n_prompt <= 0 || n_new < 0 || (n_new > 0 && !out_tokens)) return fail(RK_ERR_ARGS, "bad argument");
  rk_stage *s = m->stage;
  const int steps = n_prompt + n_new - 1;
  if (steps > s->ctx) return fail(RK_ERR_ARGS, "generation of %d positions exceeds the stage's %d", steps, s->ctx);
  const int V = s->c.vocab;
  for (int i = 0; i < n_prompt; i++)
    if (prompt[i] < 0 || prompt[i] >= V) return fail(RK_ERR_ARGS, "prompt token %d outside the vocabulary", prompt[i]);
  rk_device *d = m->d;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  // Without per-position logits, the prompt's tokens but the last run
  // through the stage's ForwardMany (batched products when the stage takes
  // them; bits as Forward token by token), in chunks of the stage's
  // io_tokens with at least two tokens each; the step graph then takes the
  // last prompt token and the generated ones.
  int first = 0;
  if (!out_logits && s->many && n_prompt > 2) {
    first = n_prompt - 1;
    if (first % s->io_tokens == 1) first--;
  }
  const int D = s->c.dim;
  int *pin = nullptr;
  CK(cudaMallocHost(&pin, sizeof(int) * (size_t)(n_prompt + n_new + 2)));
  memcpy(pin, prompt, sizeof(int) * n_prompt);
  pin[n_prompt + n_new] = first;
  auto run = [&]() -> int {
    for (int start = 0; start < first; start += s->io_tokens) {
      const int nt = std::min(s->io_tokens, first - start);
      int positions[64];
      CK(cudaMemcpyAsync(m->prompt_dev, &pin[start], sizeof(int) * nt, cudaMemcpyHostToDevice, d->st));
      for (int t = 0; t < nt; t++) {
        positions[t] = start + t;
        CK(launch_embed(m->embed->fmt, m->embed->w, m->embed->s, m->embed->rows, D, m->prompt_dev + t,
                        s->io + (size_t)t * D, d->err_dev, d->st));
      }
      int r = stage_forward_many(s, positions, nt, false);
      if (r) return r;
    }
    CK(cudaMemcpyAsync(s->pos_dev, &pin[n_prompt + n_new], 4, cudaMemcpyHostToDevice, d->st));
    for (int i = first; i < steps; i++) {
      // Prompt tokens are fed from the host; generated ones are already in
      // token_dev (k_feed_token).
      if (i < n_prompt) CK(cudaMemcpyAsync(m->token_dev, &pin[i], 4, cudaMemcpyHostToDevice, d->st));
      CK(cudaGraphLaunch(m->graph, d->st));
      if (i >= n_prompt - 1) CK(cudaMemcpyAsync(&pin[n_prompt + (i - (n_prompt - 1))], m->next_dev, 4, cudaMemcpyDeviceToHost, d->st));
      if (out_logits) {
        CK(cudaMemcpyAsync(m->pin_logits, m->head->logits, 4 * (size_t)V, cudaMemcpyDeviceToHost, d->st));
        int r = sync_dev(d);
        if (r) return r;
        memcpy(out_logits + (size_t)i * V, m->pin_logits, 4 * (size_t)V);
      }
    }
    return sync_dev(d);
  };
  rc = run();
  if (rc == RK_OK && n_new > 0) memcpy(out_tokens, pin + n_prompt, sizeof(int) * n_new);
  cudaFreeHost(pin);
  return rc;
}

// ---------------------------------------------------------------------------
// tensor/1 matmul
// ---------------------------------------------------------------------------
static int tensor_check(int dtype, int m, int k, int n) {
  if (dtype == RK_TENSOR_I32) return fail(RK_ERR_ARGS, "matmul of int32 tensors");
  if (dtype != RK_TENSOR_F32 && dtype != RK_TENSOR_I8) return fail(RK_ERR_ARGS, "unknown dtype %d", dtype);
  if (m <= 0 || k <= 0 || n <= 0 || m > (1 << 24) || k > (1 << 24) || n > (1 << 24))
    return fail(RK_ERR_ARGS, "matmul shape %d×%d·%d out of range", m, k, n);
  return RK_OK;
}

extern "C" int rk_tensor_matmul_device(rk_device *d, int dtype, int transposed, int m, int k, int n, const void *a_dev,
                                       const void *b_dev, void *c_dev) {
  if (!d || !a_dev || !b_dev || !c_dev) return fail(RK_ERR_ARGS, "null argument");
  int rc = tensor_check(dtype, m, k, n);
  if (rc) return rc;
  if ((rc = set_device(d))) return rc;
  CK(launch_tensor_matmul(dtype, transposed, m, k, n, a_dev, b_dev, c_dev, d->sms, d->err_dev, d->st));
  return RK_OK;
}

extern "C" int rk_tensor_matmul(rk_device *d, int dtype, int transposed, int m, int k, int n, const void *a,
                                const void *b, void *c) {
  if (!d || !a || !b || !c) return fail(RK_ERR_ARGS, "null argument");
  int rc = tensor_check(dtype, m, k, n);
  if (rc) return rc;
  Guard g(d);
  if ((rc = set_device(d))) return rc;
  const size_t es = dtype == RK_TENSOR_F32 ? 4 : 1;
  const size_t ab = es * (size_t)m * k, bb = es * (size_t)k * n, cb = 4 * (size_t)m * n;
  void *da = nullptr, *db = nullptr, *dc = nullptr;
  cudaError_t e = cudaMalloc(&da, ab);
  if (e == cudaSuccess) e = cudaMalloc(&db, bb);
  if (e == cudaSuccess) e = cudaMalloc(&dc, cb);
  if (e == cudaSuccess) e = cudaMemcpyAsync(da, a, ab, cudaMemcpyHostToDevice, d->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(db, b, bb, cudaMemcpyHostToDevice, d->st);
  if (e == cudaSuccess) e = launch_tensor_matmul(dtype, transposed, m, k, n, da, db, dc, d->sms, d->err_dev, d->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(c, dc, cb, cudaMemcpyDeviceToHost, d->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  cudaFree(da);
  cudaFree(db);
  cudaFree(dc);
  if (e != cudaSuccess) return cuda_fail(e, "tensor matmul");
  return check_dev_err(d);
}

// rakkan_tensor_v1's element and row operations (tensor.go:341-486): host
// buffers in and out through device copies, the reference's argument checks
// (tenErrArgs) as RK_ERR_ARGS.
static int tensor_elemwise(rk_device *d, size_t in_a, const void *a, size_t in_b, const void *b, size_t out_bytes,
                           void *c, const char *what,
                           const std::function<cudaError_t(const void *, const void *, void *, cudaStream_t)> &run) {
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  void *da = nullptr, *db = nullptr, *dc = nullptr;
  cudaError_t e = cudaMalloc(&da, std::max<size_t>(in_a, 16));
  if (e == cudaSuccess && b) e = cudaMalloc(&db, std::max<size_t>(in_b, 16));
  if (e == cudaSuccess) e = cudaMalloc(&dc, std::max<size_t>(out_bytes, 16));
  if (e == cudaSuccess && in_a) e = cudaMemcpyAsync(da, a, in_a, cudaMemcpyHostToDevice, d->st);
  if (e == cudaSuccess && b && in_b) e = cudaMemcpyAsync(db, b, in_b, cudaMemcpyHostToDevice, d->st);
  if (e == cudaSuccess) e = run(da, db, dc, d->st);
  if (e == cudaSuccess && out_bytes) e = cudaMemcpyAsync(c, dc, out_bytes, cudaMemcpyDeviceToHost, d->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  cudaFree(da);
  cudaFree(db);
  cudaFree(dc);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return check_dev_err(d);
}

static bool ten_shape_ok(int rows, int cols) { return rows > 0 && cols > 0 && (long long)rows * cols <= (1LL << 31); }

extern "C" int rk_tensor_add(rk_device *d, int dtype, int rows, int cols, const void *a, const void *b, int b_rows,
                             void *c) {
  if (!d || !a || !b || !c || !ten_shape_ok(rows, cols)) return fail(RK_ERR_ARGS, "bad argument");
  if (dtype == RK_TENSOR_I8 || (dtype != RK_TENSOR_F32 && dtype != RK_TENSOR_I32) || (b_rows != rows && b_rows != 1))
    return fail(RK_ERR_ARGS, "add: dtype or shape mismatch");
  const size_t n = (size_t)rows * cols;
  return tensor_elemwise(d, 4 * n, a, 4 * (size_t)b_rows * cols, b, 4 * n, c, "tensor add",
                         [&](const void *da, const void *db, void *dc, cudaStream_t st) {
                           return launch_tensor_add(dtype == RK_TENSOR_F32 ? 0 : 1, rows, cols, da, db, b_rows, dc, st);
                         });
}

extern "C" int rk_tensor_scale(rk_device *d, int dtype, int rows, int cols, const void *a, float k, float *c) {
  if (!d || !a || !c || !ten_shape_ok(rows, cols)) return fail(RK_ERR_ARGS, "bad argument");
  if (dtype != RK_TENSOR_F32 && dtype != RK_TENSOR_I32) return fail(RK_ERR_ARGS, "scale: int8 input");
  const size_t n = (size_t)rows * cols;
  return tensor_elemwise(d, 4 * n, a, 0, nullptr, 4 * n, c, "tensor scale",
                         [&](const void *da, const void *, void *dc, cudaStream_t st) {
                           return launch_tensor_scale(dtype == RK_TENSOR_F32 ? 0 : 1, (long long)n, da, k, (float *)dc, st);
                         });
}

extern "C" int rk_tensor_relu(rk_device *d, int dtype, int rows, int cols, const void *a, void *c) {
  if (!d || !a || !c || !ten_shape_ok(rows, cols)) return fail(RK_ERR_ARGS, "bad argument");
  if (dtype != RK_TENSOR_F32 && dtype != RK_TENSOR_I32) return fail(RK_ERR_ARGS, "relu: int8 input");
  const size_t n = (size_t)rows * cols;
  return tensor_elemwise(d, 4 * n, a, 0, nullptr, 4 * n, c, "tensor relu",
                         [&](const void *da, const void *, void *dc, cudaStream_t st) {
                           return launch_tensor_relu(dtype == RK_TENSOR_F32 ? 0 : 1, (long long)n, da, dc, st);
                         });
}

extern "C" int rk_tensor_softmax(rk_device *d, int dtype, int rows, int cols, const float *a, float *c) {
  if (!d || !a || !c || !ten_shape_ok(rows, cols)) return fail(RK_ERR_ARGS, "bad argument");
  if (dtype != RK_TENSOR_F32) return fail(RK_ERR_ARGS, "softmax: not f32");
  const size_t n = (size_t)rows * cols;
  return tensor_elemwise(d, 4 * n, a, 0, nullptr, 4 * n, c, "tensor softmax",
                         [&](const void *da, const void *, void *dc, cudaStream_t st) {
                           return launch_tensor_softmax(rows, cols, (const float *)da, (float *)dc, st);
                         });
}

extern "C" int rk_tensor_quantize(rk_device *d, int dtype, int rows, int cols, const float *a, float k, int8_t *c) {
  if (!d || !a || !c || !ten_shape_ok(rows, cols)) return fail(RK_ERR_ARGS, "bad argument");
  if (dtype != RK_TENSOR_F32 || !(k > 0.0f)) return fail(RK_ERR_ARGS, "quantize: not f32, or scale not positive");
  const size_t n = (size_t)rows * cols;
  return tensor_elemwise(d, 4 * n, a, 0, nullptr, n, c, "tensor quantize",
                         [&](const void *da, const void *, void *dc, cudaStream_t st) {
                           return launch_tensor_quantize((long long)n, (const float *)da, k, (int8_t *)dc, st);
                         });
}

extern "C" int rk_tensor_argmax(rk_device *d, int dtype, int rows, int cols, const void *a, int32_t *out) {
  if (!d || !a || !out || !ten_shape_ok(rows, cols)) return fail(RK_ERR_ARGS, "bad argument");
  if (dtype != RK_TENSOR_F32 && dtype != RK_TENSOR_I32) return fail(RK_ERR_ARGS, "argmax: int8 input");
  const size_t n = (size_t)rows * cols;
  return tensor_elemwise(d, 4 * n, a, 0, nullptr, 4 * (size_t)rows, out, "tensor argmax",
                         [&](const void *da, const void *, void *dc, cudaStream_t st) {
                           return launch_tensor_argmax(dtype == RK_TENSOR_F32 ? 0 : 1, rows, cols, da, (int *)dc, st);
                         });
}


// ---------------------------------------------------------------------------
// rakkan_tensor_v1's tensor table on the device (tensor.go:92-158, 186-275,
// 286-505): tensors live in device memory by handle, so a guest's chain of
// operations (matmul -> add -> relu ...) stays on the GPU; only from_memory /
// from_blob upload and to_memory / argmax download. Each operation makes a
// new tensor, as the reference's do, within the table's byte budget.
// ---------------------------------------------------------------------------
namespace {
struct DevTensor {
  int dtype = 0, rows = 0, cols = 0;
  void *p = nullptr;
  int64_t bytes = 0;
};
int64_t ten_elem_size(int dtype) { return dtype == RK_TENSOR_F32 || dtype == RK_TENSOR_I32 ? 4 : dtype == RK_TENSOR_I8 ? 1 : 0; }
constexpr int kMaxTensorDim = 1 << 24;  // maxTensorDim, tensor.go:60
}  // namespace

struct rk_tensors {
  rk_device *d = nullptr;
  int64_t budget = 0, used = 0;
  std::map<int, DevTensor> table;
  int next = 0;
};

extern "C" int rk_tensors_new(rk_device *d, int64_t budget_bytes, rk_tensors **out) {
  if (!d || !out || budget_bytes < 0) return fail(RK_ERR_ARGS, "bad argument");
  auto *t = new rk_tensors();
  t->d = d;
  t->budget = budget_bytes;
  *out = t;
  return RK_OK;
}

extern "C" void rk_tensors_free(rk_tensors *t) {
  if (!t) return;
  Guard g(t->d);
  cudaSetDevice(t->d->ordinal);
  cudaStreamSynchronize(t->d->st);
  for (auto &kv : t->table) cudaFree(kv.second.p);
  t->d->used -= t->used;
  delete t;
}

extern "C" int64_t rk_tensors_used(const rk_tensors *t) { return t ? t->used : 0; }

// newTensor (tensor.go:119-141): a zeroed tensor within the budget, or 0
// (bad type or shape: *why = RK_ERR_ARGS; over the budget: RK_ERR_TOO_BIG).
static DevTensor *tt_new(rk_tensors *t, int dtype, int rows, int cols, DevTensor *out, int *why) {
  const int64_t es = ten_elem_size(dtype);
  if (es == 0 || rows <= 0 || cols <= 0 || rows > kMaxTensorDim || cols > kMaxTensorDim) {
    *why = RK_ERR_ARGS;
    return nullptr;
  }
  const int64_t n = (int64_t)rows * cols * es;
  if (t->used + n > t->budget) {
    *why = RK_ERR_TOO_BIG;
    return nullptr;
  }
  out->dtype = dtype;
  out->rows = rows;
  out->cols = cols;
  out->bytes = n;
  cudaError_t e = cudaMalloc(&out->p, std::max<int64_t>(n, 16));
  if (e == cudaSuccess) e = cudaMemsetAsync(out->p, 0, n, t->d->st);
  if (e != cudaSuccess) {
    cudaFree(out->p);
    cudaGetLastError();
    *why = RK_ERR_NOMEM;
    return nullptr;
  }
  t->used += n;
  t->d->used += n;
  return out;
}

static void tt_drop(rk_tensors *t, DevTensor &x) {
  cudaFree(x.p);
  t->used -= x.bytes;
  t->d->used -= x.bytes;
  x.p = nullptr;
}

static int tt_add(rk_tensors *t, const DevTensor &x) {
  t->table[++t->next] = x;
  return t->next;
}

static DevTensor *tt_get(rk_tensors *t, int h) {
  auto it = t->table.find(h);
  return it == t->table.end() ? nullptr : &it->second;
}

// Runs a kernel sequence into a fresh result tensor; returns its handle, or
// the error (the result is dropped).
static int tt_result(rk_tensors *t, DevTensor &c, cudaError_t e, const char *what) {
  rk_device *d = t->d;
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  if (e != cudaSuccess) {
    tt_drop(t, c);
    return cuda_fail(e, what);
  }
  int rc = check_dev_err(d);
  if (rc) {
    tt_drop(t, c);
    return rc;
  }
  return tt_add(t, c);
}

// Uploads raw little-endian bytes into a new tensor (decodeInto: float32
// NaNs canonicalised on the device).
static int tt_upload(rk_tensors *t, const void *raw, int dtype, int rows, int cols, int too_big_code) {
  DevTensor c;
  int why = 0;
  if (!tt_new(t, dtype, rows, cols, &c, &why)) {
    if (why == RK_ERR_TOO_BIG) return fail(too_big_code, "tensor of %d×%d over the budget", rows, cols);
    if (why == RK_ERR_NOMEM) return fail(RK_ERR_NOMEM, "device allocation failed");
    return fail(RK_ERR_ARGS, "bad tensor type or shape");
  }
  cudaError_t e = cudaMemcpyAsync(c.p, raw, c.bytes, cudaMemcpyHostToDevice, t->d->st);
  if (e == cudaSuccess && dtype == RK_TENSOR_F32) e = launch_tensor_canon(c.bytes / 4, (float *)c.p, t->d->st);
  return tt_result(t, c, e, "tensor upload");
}

extern "C" int rk_tensors_from_memory(rk_tensors *t, const void *src, int dtype, int rows, int cols) {
  if (!t || !src) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(t->d);
  int rc = set_device(t->d);
  if (rc) return rc;
  // tenFromMemory reports a tensor it cannot make as tenErrArgs (tensor.go:206-209).
  return tt_upload(t, src, dtype, rows, cols, RK_ERR_ARGS);
}

extern "C" int rk_tensors_from_blob(rk_tensors *t, const void *blob, int64_t blob_size, int64_t offset, int dtype,
                                    int rows, int cols) {
  if (!t || (!blob && blob_size > 0) || blob_size < 0 || offset < 0) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(t->d);
  int rc = set_device(t->d);
  if (rc) return rc;
  // tenFromBlob (tensor.go:220-242): the tensor is made first (tenErrTooBig),
  // then the blob must hold it from `offset` on (tenErrBlob).
  const int64_t es = ten_elem_size(dtype);
  if (es == 0 || rows <= 0 || cols <= 0 || rows > kMaxTensorDim || cols > kMaxTensorDim)
    return fail(RK_ERR_TOO_BIG, "bad tensor type or shape");
  const int64_t n = (int64_t)rows * cols * es;
  if (t->used + n > t->budget) return fail(RK_ERR_TOO_BIG, "tensor of %d×%d over the budget", rows, cols);
  // (offset is the guest's: compared without forming offset + n, which a
  // huge offset would overflow)
  if (offset > blob_size || n > blob_size - offset)
    return fail(RK_ERR_BLOB, "blob of %lld bytes too short for %lld bytes at %lld", (long long)blob_size,
                (long long)n, (long long)offset);
  return tt_upload(t, static_cast<const char *>(blob) + offset, dtype, rows, cols, RK_ERR_TOO_BIG);
}

extern "C" int64_t rk_tensors_to_memory(rk_tensors *t, int h, void *dst, int64_t n) {
  if (!t) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(t->d);
  DevTensor *x = tt_get(t, h);
  if (!x || !dst || n < x->bytes) return fail(RK_ERR_ARGS, "to_memory: bad handle or buffer too small");
  int rc = set_device(t->d);
  if (rc) return rc;
  CK(cudaMemcpy(dst, x->p, x->bytes, cudaMemcpyDeviceToHost));
  return x->bytes;
}

extern "C" int rk_tensors_dim(rk_tensors *t, int h, int which) {
  if (!t || which < 0 || which > 2) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(t->d);
  DevTensor *x = tt_get(t, h);
  if (!x) return fail(RK_ERR_ARGS, "bad handle");
  return which == 0 ? x->rows : which == 1 ? x->cols : x->dtype;
}

extern "C" int rk_tensors_release(rk_tensors *t, int h) {
  if (!t) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(t->d);
  DevTensor *x = tt_get(t, h);
  if (!x) return fail(RK_ERR_ARGS, "bad handle");
  cudaSetDevice(t->d->ordinal);
  cudaStreamSynchronize(t->d->st);
  tt_drop(t, *x);
  t->table.erase(h);
  return RK_OK;
}

extern "C" int rk_tensors_matmul(rk_tensors *t, int ha, int hb, int transposed) {
  if (!t) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(t->d);
  DevTensor *a = tt_get(t, ha), *b = tt_get(t, hb);
  if (!a || !b || a->dtype != b->dtype || a->dtype == RK_TENSOR_I32) return fail(RK_ERR_ARGS, "matmul: bad operands");
  const int m = a->rows, k = a->cols, n = transposed ? b->rows : b->cols;
  if ((transposed ? b->cols : b->rows) != k) return fail(RK_ERR_ARGS, "matmul: inner dimensions differ");
  int rc = set_device(t->d);
  if (rc) return rc;
  DevTensor c;
  int why = 0;
  if (!tt_new(t, a->dtype == RK_TENSOR_I8 ? RK_TENSOR_I32 : RK_TENSOR_F32, m, n, &c, &why))
    return fail(why == RK_ERR_NOMEM ? RK_ERR_NOMEM : RK_ERR_TOO_BIG, "matmul: result over the budget");
  const cudaError_t e = launch_tensor_matmul(a->dtype, transposed ? 1 : 0, m, k, n, a->p, b->p, c.p, t->d->sms,
                                             t->d->err_dev, t->d->st);
  return tt_result(t, c, e, "tensor matmul");
}

extern "C" int rk_tensors_add(rk_tensors *t, int ha, int hb) {
  if (!t) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(t->d);
  DevTensor *a = tt_get(t, ha), *b = tt_get(t, hb);
  if (!a || !b || a->dtype != b->dtype || a->dtype == RK_TENSOR_I8 || a->cols != b->cols ||
      (b->rows != a->rows && b->rows != 1))
    return fail(RK_ERR_ARGS, "add: bad operands");
  int rc = set_device(t->d);
  if (rc) return rc;
  DevTensor c;
  int why = 0;
  if (!tt_new(t, a->dtype, a->rows, a->cols, &c, &why)) return fail(RK_ERR_TOO_BIG, "add: result over the budget");
  const cudaError_t e =
      launch_tensor_add(a->dtype == RK_TENSOR_F32 ? 0 : 1, a->rows, a->cols, a->p, b->p, b->rows, c.p, t->d->st);
  return tt_result(t, c, e, "tensor add");
}

// scale, relu, softmax and quantize: one input tensor, one result.
static int tt_unary(rk_tensors *t, int h, bool ok_i8, bool ok_i32, bool f32_only, int out_dtype_f32, int out_dtype_i32,
                    const char *what, const std::function<cudaError_t(const DevTensor &, DevTensor &)> &run) {
  if (!t) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(t->d);
  DevTensor *a = tt_get(t, h);
  if (!a || (a->dtype == RK_TENSOR_I8 && !ok_i8) || (a->dtype == RK_TENSOR_I32 && !ok_i32) ||
      (f32_only && a->dtype != RK_TENSOR_F32))
    return fail(RK_ERR_ARGS, "%s: bad operand", what);
  int rc = set_device(t->d);
  if (rc) return rc;
  DevTensor c;
  int why = 0;
  const int od = a->dtype == RK_TENSOR_F32 ? out_dtype_f32 : out_dtype_i32;
  if (!tt_new(t, od, a->rows, a->cols, &c, &why)) return fail(RK_ERR_TOO_BIG, "%s: result over the budget", what);
  return tt_result(t, c, run(*a, c), what);
}

extern "C" int rk_tensors_scale(rk_tensors *t, int h, float k) {
  return tt_unary(t, h, false, true, false, RK_TENSOR_F32, RK_TENSOR_F32, "scale",
                  [&](const DevTensor &a, DevTensor &c) {
                    return launch_tensor_scale(a.dtype == RK_TENSOR_F32 ? 0 : 1, (long long)a.rows * a.cols, a.p, k,
                                               (float *)c.p, t->d->st);
                  });
}

extern "C" int rk_tensors_relu(rk_tensors *t, int h) {
  return tt_unary(t, h, false, true, false, RK_TENSOR_F32, RK_TENSOR_I32, "relu",
                  [&](const DevTensor &a, DevTensor &c) {
                    return launch_tensor_relu(a.dtype == RK_TENSOR_F32 ? 0 : 1, (long long)a.rows * a.cols, a.p, c.p,
                                              t->d->st);
                  });
}

extern "C" int rk_tensors_softmax(rk_tensors *t, int h) {
  return tt_unary(t, h, false, false, true, RK_TENSOR_F32, RK_TENSOR_F32, "softmax",
                  [&](const DevTensor &a, DevTensor &c) {
                    return launch_tensor_softmax(a.rows, a.cols, (const float *)a.p, (float *)c.p, t->d->st);
                  });
}

extern "C" int rk_tensors_quantize(rk_tensors *t, int h, float k) {
  if (!(k > 0.0f)) return fail(RK_ERR_ARGS, "quantize: scale not positive");
  return tt_unary(t, h, false, false, true, RK_TENSOR_I8, RK_TENSOR_I8, "quantize",
                  [&](const DevTensor &a, DevTensor &c) {
                    return launch_tensor_quantize((long long)a.rows * a.cols, (const float *)a.p, k, (int8_t *)c.p,
                                                  t->d->st);
                  });
}

extern "C" int rk_tensors_argmax(rk_tensors *t, int h, int32_t *dst, int64_t n) {
  if (!t) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(t->d);
  DevTensor *a = tt_get(t, h);
  if (!a || a->dtype == RK_TENSOR_I8 || !dst || n < (int64_t)a->rows * 4)
    return fail(RK_ERR_ARGS, "argmax: bad operand or buffer too small");
  int rc = set_device(t->d);
  if (rc) return rc;
  int *out = nullptr;
  cudaError_t e = cudaMalloc(&out, 4 * (size_t)a->rows);
  if (e == cudaSuccess)
    e = launch_tensor_argmax(a->dtype == RK_TENSOR_F32 ? 0 : 1, a->rows, a->cols, a->p, out, t->d->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dst, out, 4 * (size_t)a->rows, cudaMemcpyDeviceToHost, t->d->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(t->d->st);
  cudaFree(out);
  if (e != cudaSuccess) return cuda_fail(e, "tensor argmax");
  return a->rows;
}

// ---------------------------------------------------------------------------
// Device-side import and the seeded generator
// ---------------------------------------------------------------------------
static int matrix_generate(rk_device *d, long long first, int rows, int cols, int fmt, uint64_t seed, uint64_t tid,
                           float scale, rk_matrix **out);

extern "C" int rk_matrix_generate(rk_device *d, int rows, int cols, int fmt, uint64_t seed, uint64_t tid, float scale,
                                  rk_matrix **out) {
  return matrix_generate(d, 0, rows, cols, fmt, seed, tid, scale, out);
}

extern "C" int rk_matrix_generate_rows(rk_device *d, int rows_total, int row0, int rows, int cols, int fmt,
                                       uint64_t seed, uint64_t tid, float scale, rk_matrix **out) {
  if (row0 < 0 || rows < 0 || row0 + rows > rows_total) return fail(RK_ERR_ARGS, "rows out of range");
  return matrix_generate(d, (long long)row0 * cols, rows, cols, fmt, seed, tid, scale, out);
}

// Elements [first, first + rows·cols) of the tensor's stream as a matrix.
static int matrix_generate(rk_device *d, long long first, int rows, int cols, int fmt, uint64_t seed, uint64_t tid,
                           float scale, rk_matrix **out) {
  if (!d || !out) return fail(RK_ERR_ARGS, "null argument");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  rk_matrix *m = nullptr;
  if ((rc = matrix_alloc(d, rows, cols, fmt, &m))) return rc;
  const long long n = (long long)rows * cols;
  // Generate in slices of at most 256 Mi floats to bound the scratch.
  const long long slice = std::min<long long>(n, 1ll << 28);
  float *tmp = nullptr;
  uint8_t *stale = nullptr;
  cudaError_t e = cudaMalloc(&tmp, sizeof(float) * (size_t)slice);
  if (e == cudaSuccess && fmt == RK_FMT_Q4_0) e = cudaMalloc(&stale, (size_t)(slice / 32 + 1));
  for (long long off = 0; e == cudaSuccess && off < n; off += slice) {
    const long long cnt = std::min(slice, n - off);
    e = launch_gen_normal(seed, tid, first + off, cnt, scale, tmp, d->st);
    if (e != cudaSuccess) break;
    switch (fmt) {
      case RK_FMT_F32: e = cudaMemcpyAsync(m->w + 4 * off, tmp, 4 * (size_t)cnt, cudaMemcpyDeviceToDevice, d->st); break;
      case RK_FMT_Q8_0: e = launch_quantize_q8_w(tmp, cnt, (int8_t *)m->w + off, m->s + off / 32, d->st); break;
      case RK_FMT_Q4_0:
        // Slices are whole numbers of blocks; a stale block at a slice start
        // would need the previous slice's last block (not for finite weights).
        e = launch_quantize_q4_w(tmp, cnt, m->w + off / 2, m->s + off / 32, stale, d->st);
        break;
      case RK_FMT_BF16: e = launch_to_bf16(tmp, cnt, reinterpret_cast<uint16_t *>(m->w) + off, d->st); break;
      default: e = cudaErrorInvalidValue;
    }
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  cudaFree(tmp);
  cudaFree(stale);
  if (e != cudaSuccess) {
    matrix_release(m);
    return cuda_fail(e, "matrix generation");
  }
  *out = m;
  return RK_OK;
}

extern "C" int rk_generate_normal(rk_device *d, uint64_t seed, uint64_t tid, int64_t offset, int64_t n, float scale,
                                  float *out) {
  if (!d || !out || n < 0) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  float *tmp = nullptr;
  CK(cudaMalloc(&tmp, 4 * (size_t)std::max<int64_t>(n, 1)));
  cudaError_t e = launch_gen_normal(seed, tid, offset, n, scale, tmp, d->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, tmp, 4 * (size_t)n, cudaMemcpyDeviceToHost, d->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  cudaFree(tmp);
  if (e != cudaSuccess) return cuda_fail(e, "generate");
  return RK_OK;
}

extern "C" int rk_quantize(rk_device *d, int fmt, const float *w, int64_t n, void *q, float *scales) {
  if (!d || !w || !q || !scales || n < 0 || n % 32) return fail(RK_ERR_ARGS, "bad argument");
  if (!quantized_fmt(fmt)) return fail(RK_ERR_ARGS, "not a quantized format");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  float *dw = nullptr, *ds = nullptr;
  uint8_t *dq = nullptr, *stale = nullptr;
  const size_t qb = fmt == RK_FMT_Q8_0 ? (size_t)n : (size_t)n / 2;
  cudaError_t e = cudaMalloc(&dw, 4 * (size_t)std::max<int64_t>(n, 1));
  if (e == cudaSuccess) e = cudaMalloc(&dq, std::max<size_t>(qb, 1));
  if (e == cudaSuccess) e = cudaMalloc(&ds, 4 * (size_t)(n / 32 + 1));
  if (e == cudaSuccess) e = cudaMalloc(&stale, (size_t)(n / 32 + 1));
  if (e == cudaSuccess) e = cudaMemcpyAsync(dw, w, 4 * (size_t)n, cudaMemcpyHostToDevice, d->st);
  if (e == cudaSuccess)
    e = fmt == RK_FMT_Q8_0 ? launch_quantize_q8_w(dw, n, (int8_t *)dq, ds, d->st)
                           : launch_quantize_q4_w(dw, n, dq, ds, stale, d->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(q, dq, qb, cudaMemcpyDeviceToHost, d->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(scales, ds, 4 * (size_t)(n / 32), cudaMemcpyDeviceToHost, d->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  cudaFree(dw);
  cudaFree(dq);
  cudaFree(ds);
  cudaFree(stale);
  if (e != cudaSuccess) return cuda_fail(e, "quantize");
  return RK_OK;
}

// ---------------------------------------------------------------------------
// Measurement helpers
// ---------------------------------------------------------------------------
// Reads a buffer twice L2's size, so the timed kernel starts with L2 full of
// clean lines that are not its own (a write-based flush would leave dirty
// lines whose write-back would land inside the timed kernel).
__global__ void k_flush_read(const int4 *p, long long n, int *sink) {
  int acc = 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int4 v = p[i];
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  if (acc == 0x7fffffff) *sink = acc;  // never true for the zeroed buffer; keeps the loads
}

static int ensure_flush(rk_device *d) {
  if (d->flush) return RK_OK;
  d->flush_bytes = (size_t)256 << 20;  // twice the 126 MB L2
  CK(cudaMalloc(&d->flush, d->flush_bytes));
  CK(cudaMemset(d->flush, 0, d->flush_bytes));
  return RK_OK;
}

extern "C" int rk_bench_matvec(rk_matrix *m, int iters, int flags, float *ms_per_launch) {
  if (!m || iters <= 0 || !ms_per_launch) return fail(RK_ERR_ARGS, "bad argument");
  rk_device *d = m->d;
  const int flush = flags & RK_BENCH_FLUSH;
  Pro pro;
  if ((flags & RK_BENCH_FUSED) && quantized_fmt(m->fmt) && matvec_fused_ok(m->fmt, m->cols, false)) pro.pro = PRO_QUANT;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  if (flush && (rc = ensure_flush(d))) return rc;
  CK(cudaMemsetAsync(d->mv_x, 0, 4 * (size_t)m->cols, d->st));
  if (quantized_fmt(m->fmt))
    CK(launch_quantize_act(d->mv_x, m->cols, nullptr, 0.0f, 0.0f, nullptr, d->mv_qx, d->mv_xs, d->mv_xsum, d->st));
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  float total = 0.0f;
  float *out = d->mv_out;
  for (int i = 0; i < iters + 1; i++) {
    if (flush) k_flush_read<<<d->sms * 4, 512, 0, d->st>>>((const int4 *)d->flush, (long long)(d->flush_bytes / 16), d->err_dev + 1);
    CK(cudaEventRecord(e0, d->st));
    if ((rc = enqueue_matvecs(d, 1, &m, &out, d->mv_x, d->mv_qx, d->mv_xs, d->mv_xsum, EPI_STORE, d->st, pro)))
      return rc;
    CK(cudaEventRecord(e1, d->st));
    CK(cudaEventSynchronize(e1));
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    if (i > 0) total += ms;  // the first launch is a warm-up
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if ((rc = check_dev_err(d))) return rc;
  *ms_per_launch = total / iters;
  return RK_OK;
}

extern "C" int rk_bench_matvec_many(rk_matrix *m, int n, int iters, int flags, float *ms_per_launch) {
  if (!m || n <= 0 || iters <= 0 || !ms_per_launch) return fail(RK_ERR_ARGS, "bad argument");
  if (!mv_many_ok(m->fmt, m->rows, m->cols, m->w, m->s))
    return fail(RK_ERR_ARGS, "the batched kernel takes Q8_0 and Q4_0 matrices of a multiple of 128 columns");
  rk_device *d = m->d;
  const int flush = flags & RK_BENCH_FLUSH;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  if (flush && (rc = ensure_flush(d))) return rc;
  const size_t cols = (size_t)m->cols, rows = (size_t)m->rows;
  const int xs_pitch = (n + 3) & ~3;  // the batched kernel's block-major input scales
  float *dx = nullptr, *dxs = nullptr, *dout = nullptr;
  int8_t *dqx = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  float total = 0.0f;
  // Seeded inputs, quantized once; then each timed launch is the batched
  // product alone (L2 flushed first when asked).
  cudaError_t e = cudaMalloc(&dx, 4 * n * cols);
  if (e == cudaSuccess) e = cudaMalloc(&dqx, n * cols);
  if (e == cudaSuccess) e = cudaMalloc(&dxs, 4 * (size_t)xs_pitch * (cols / 32));
  if (e == cudaSuccess) e = cudaMalloc(&dout, 4 * n * rows);
  if (e == cudaSuccess) e = launch_fill_hash(DT_F32, dx, (long long)(n * cols), 7u, d->st);
  if (e == cudaSuccess) e = launch_quantize_many(dx, n, m->cols, nullptr, 0.0f, 0.0f, dqx, dxs, xs_pitch, d->st);
  if (e == cudaSuccess) e = cudaEventCreate(&e0);
  if (e == cudaSuccess) e = cudaEventCreate(&e1);
  const MmMat mat{m->w, m->s, m->rows, dout, (long long)rows, EPI_STORE, m->fmt};
  for (int i = 0; e == cudaSuccess && i < iters + 1; i++) {
    if (flush) k_flush_read<<<d->sms * 4, 512, 0, d->st>>>((const int4 *)d->flush, (long long)(d->flush_bytes / 16), d->err_dev + 1);
    e = cudaEventRecord(e0, d->st);
    if (e == cudaSuccess) e = launch_mv_many(1, &mat, m->cols, n, dqx, dxs, xs_pitch, d->err_dev, d->sms, d->st);
    if (e == cudaSuccess) e = cudaEventRecord(e1, d->st);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0.0f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    if (i > 0) total += ms;  // the first launch is a warm-up
  }
  rc = e == cudaSuccess ? check_dev_err(d) : cuda_fail(e, "batched matvec bench");
  cudaStreamSynchronize(d->st);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  for (void *p : {(void *)dx, (void *)dqx, (void *)dxs, (void *)dout}) cudaFree(p);
  if (rc) return rc;
  *ms_per_launch = total / iters;
  return RK_OK;
}

extern "C" int rk_bench_tensor(rk_device *d, int dtype, int transposed, int m, int k, int n, int iters, int flags,
                               float *ms_per_product) {
  if (!d || iters <= 0 || !ms_per_product) return fail(RK_ERR_ARGS, "bad argument");
  int rc = tensor_check(dtype, m, k, n);
  if (rc) return rc;
  Guard g(d);
  if ((rc = set_device(d))) return rc;
  const int flush = flags & RK_BENCH_FLUSH;
  if (flush && (rc = ensure_flush(d))) return rc;
  const size_t es = dtype == RK_TENSOR_F32 ? 4 : 1;
  void *da = nullptr, *db = nullptr, *dc = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  float total = 0.0f;
  cudaError_t e = cudaMalloc(&da, es * (size_t)m * k);
  if (e == cudaSuccess) e = cudaMalloc(&db, es * (size_t)k * n);
  if (e == cudaSuccess) e = cudaMalloc(&dc, 4 * (size_t)m * n);
  if (e == cudaSuccess) e = launch_fill_hash(dtype, da, (long long)m * k, 1u, d->st);
  if (e == cudaSuccess) e = launch_fill_hash(dtype, db, (long long)k * n, 2u, d->st);
  if (e == cudaSuccess) e = cudaEventCreate(&e0);
  if (e == cudaSuccess) e = cudaEventCreate(&e1);
  for (int i = 0; i < iters + 1 && e == cudaSuccess; i++) {
    if (flush)
      k_flush_read<<<d->sms * 4, 512, 0, d->st>>>((const int4 *)d->flush, (long long)(d->flush_bytes / 16),
                                                  d->err_dev + 1);
    e = cudaEventRecord(e0, d->st);
    if (e == cudaSuccess) e = launch_tensor_matmul(dtype, transposed, m, k, n, da, db, dc, d->sms, d->err_dev, d->st);
    if (e == cudaSuccess) e = cudaEventRecord(e1, d->st);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0.0f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    if (i > 0) total += ms;  // the first product is a warm-up
  }
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaFree(da);
  cudaFree(db);
  cudaFree(dc);
  if (e != cudaSuccess) return cuda_fail(e, "tensor bench");
  if ((rc = check_dev_err(d))) return rc;
  *ms_per_product = total / iters;
  return RK_OK;
}

extern "C" int rk_bench_model(rk_model *m, int pos, int iters, float *ms_per_step) {
  if (!m || iters <= 0 || !ms_per_step) return fail(RK_ERR_ARGS, "bad argument");
  rk_device *d = m->d;
  if (pos < 0 || pos >= m->stage->ctx) return fail(RK_ERR_ARGS, "position out of range");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  m->pin_tok[4] = pos;
  CK(cudaMemcpyAsync(m->stage->pos_dev, &m->pin_tok[4], 4, cudaMemcpyHostToDevice, d->st));
  CK(cudaEventRecord(e0, d->st));
  for (int i = 0; i < iters; i++) {
    // Each step re-runs position pos (its KV entry is rewritten), so every
    // timed step attends over pos+1 positions.
    CK(cudaMemcpyAsync(m->stage->pos_dev, &m->pin_tok[4], 4, cudaMemcpyHostToDevice, d->st));
    CK(cudaGraphLaunch(m->graph, d->st));
  }
  CK(cudaEventRecord(e1, d->st));
  CK(cudaEventSynchronize(e1));
  float ms = 0.0f;
  CK(cudaEventElapsedTime(&ms, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if ((rc = check_dev_err(d))) return rc;
  *ms_per_step = ms / iters;
  return RK_OK;
}

extern "C" int rk_model_profile(rk_model *m, int pos, int iters, rk_profile *out) {
  if (!m || iters <= 0 || !out) return fail(RK_ERR_ARGS, "bad argument");
  rk_device *d = m->d;
  if (pos < 0 || pos >= m->stage->ctx) return fail(RK_ERR_ARGS, "position out of range");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  std::vector<ProfLaunch> launches;
  cudaEvent_t s0, s1;
  CK(cudaEventCreate(&s0));
  CK(cudaEventCreate(&s1));
  m->pin_tok[4] = pos;
  g_prof = &launches;
  CK(cudaEventRecord(s0, d->st));
  for (int i = 0; i < iters && rc == RK_OK; i++) {
    cudaError_t e = cudaMemcpyAsync(m->stage->pos_dev, &m->pin_tok[4], 4, cudaMemcpyHostToDevice, d->st);
    if (e != cudaSuccess) rc = cuda_fail(e, "profile");
    if (rc == RK_OK) rc = record_model(m, d->st);
  }
  g_prof = nullptr;
  CK(cudaEventRecord(s1, d->st));
  CK(cudaEventSynchronize(s1));
  if (rc == RK_OK) rc = check_dev_err(d);
  float total = 0.0f, mv = 0.0f;
  double bytes = 0;
  cudaEventElapsedTime(&total, s0, s1);
  for (auto &l : launches) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, l.e0, l.e1);
    mv += ms;
    bytes += l.bytes;
    cudaEventDestroy(l.e0);
    cudaEventDestroy(l.e1);
  }
  cudaEventDestroy(s0);
  cudaEventDestroy(s1);
  if (rc) return rc;
  out->step_ms = total / iters;
  out->matvec_ms = mv / iters;
  out->matvec_bytes = bytes / iters;
  out->matvec_launches = (int)(launches.size() / iters);
  out->launches = m->launches;
  return RK_OK;
}

extern "C" int rk_stage_fill_cache(rk_stage *s, int positions, uint64_t seed) {
  return rk_stage_fill_cache_from(s, positions, seed, 0);
}

extern "C" int rk_stage_fill_cache_from(rk_stage *s, int positions, uint64_t seed, int first_layer) {
  if (!s || positions < 0 || positions > s->ctx || first_layer < 0) return fail(RK_ERR_ARGS, "bad argument");
  rk_device *d = s->d;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  // Position t's cache row is elements [t·kvd, …) of the layer's stream;
  // this rank holds columns [c0, c0 + kvd_l) (its kv heads).
  const int kvd = s->c.kv_heads * head_size(&s->c), kvd_l = kvd / s->G, c0 = s->rank * kvd_l;
  // A stage of several sequences gets the same rows in every sequence's caches.
  const size_t kstride = (size_t)s->ctx * kvd_l, vstride = (size_t)kvd_l * (s->v_pitch > 0 ? s->v_pitch : s->ctx);
  for (int q = 0; q < s->nseq; q++)
    for (size_t l = 0; l < s->layers.size(); l++) {
      float *keys = s->keys[l] + q * kstride, *vals = s->vals[l] + q * vstride;
      const unsigned long long gl = (unsigned long long)first_layer + l;  // the whole model's layer index
      CK(launch_gen_normal_2d(seed, 0xA0000ull + 2 * gl, positions, kvd, c0, kvd_l, kvd_l, 1, 1.0f, keys, d->st));
      if (s->v_pitch > 0)
        CK(launch_gen_normal_2d(seed, 0xA0001ull + 2 * gl, positions, kvd, c0, kvd_l, 1, s->v_pitch, 1.0f, vals,
                                d->st));
      else
        CK(launch_gen_normal_2d(seed, 0xA0001ull + 2 * gl, positions, kvd, c0, kvd_l, kvd_l, 1, 1.0f, vals, d->st));
    }
  return sync_dev(d);
}

// MatMulBF16 (num/matvec.go:124-147): out[i·m + j] = DotBF16(row j of w,
// row i of x), what MatVecBF16 gives each row of x, so each row of x is one
// bf16 matvec launch (the kernel's lane order and tree are DotBF16's).
extern "C" int rk_matmul_bf16(rk_matrix *w, int n, const float *x, float *out) {
  if (!w || n < 0 || (n > 0 && (!x || !out))) return fail(RK_ERR_ARGS, "bad argument");
  if (w->fmt != RK_FMT_BF16) return fail(RK_ERR_ARGS, "MatMulBF16 needs a bfloat16 matrix");
  if (n == 0) return RK_OK;
  rk_device *d = w->d;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  const size_t k = (size_t)w->cols, m = (size_t)w->rows;
  float *dx = nullptr, *dout = nullptr;
  cudaError_t e = cudaMalloc(&dx, 4 * k * n);
  if (e == cudaSuccess) e = cudaMalloc(&dout, 4 * m * n);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dx, x, 4 * k * n, cudaMemcpyHostToDevice, d->st);
  for (int i = 0; i < n && e == cudaSuccess; i++) {
    float *o = dout + m * i;
    rc = enqueue_matvecs(d, 1, &w, &o, dx + k * i, nullptr, nullptr, nullptr, EPI_STORE);
    if (rc) break;
  }
  if (e == cudaSuccess && !rc) e = cudaMemcpyAsync(out, dout, 4 * m * n, cudaMemcpyDeviceToHost, d->st);
  if (e == cudaSuccess && !rc) e = cudaStreamSynchronize(d->st);
  cudaFree(dx);
  cudaFree(dout);
  if (rc) return rc;
  if (e != cudaSuccess) return cuda_fail(e, "bf16 matmul");
  return check_dev_err(d);
}

// num.ToBF16 (matvec.go:23-29): round to nearest even, a NaN kept NaN.
static uint16_t host_to_bf16(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  if (f != f) return (uint16_t)((b >> 16) | 0x40);
  return (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}

// MeasureSpeed (llm/speed.go:16-47) on a device: a 4096×4096 bfloat16
// matrix of the reference's LCG values, x[i] = (i mod 17)/17; one warm-up
// product, then the median of seven timed ones (each a whole MulVec call,
// host to host, as the reference times it); GB of weights per second.
extern "C" int rk_measure_speed(rk_device *d, double *gbps) {
  if (!d || !gbps) return fail(RK_ERR_ARGS, "null argument");
  constexpr int rows = 4096, cols = 4096;
  std::vector<uint16_t> w((size_t)rows * cols);
  uint32_t seed = 1;
  for (auto &v : w) {
    seed = seed * 1664525u + 1013904223u;
    const float f = (float)((int32_t)(seed >> 8) - (1 << 23)) / (float)(1 << 30);
    v = host_to_bf16(f);
  }
  std::vector<float> x(cols), out(rows);
  for (int i = 0; i < cols; i++) x[i] = (float)(i % 17) / 17.0f;
  rk_matrix *m = nullptr;
  int rc = rk_matrix_upload(d, rows, cols, RK_FMT_BF16, w.data(), nullptr, &m);
  if (rc) return rc;
  std::vector<double> times;
  for (int it = 0; it < 8 && !rc; it++) {
    const auto t0 = std::chrono::steady_clock::now();
    rc = rk_matrix_mulvec(m, out.data(), x.data());
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (it > 0) times.push_back(dt);
  }
  rk_matrix_free(m);
  if (rc) return rc;
  std::sort(times.begin(), times.end());
  *gbps = 2.0 * rows * cols / times[times.size() / 2] / 1e9;
  return RK_OK;
}

// ---------------------------------------------------------------------------
// The reference's model part formats (internal/llm/shard.go:165-300): a
// part's tensors in order, little-endian; a matrix in its own type (float32,
// bfloat16, or the scales then the values when quantized). Decoded into host
// views, then uploaded as Layer.toDevice / Matrix.toDevice do.
// ---------------------------------------------------------------------------
struct PartDecoder {  // shard.go:187-240
  const uint8_t *p;
  int64_t left;
  bool bad = false;
  std::vector<std::vector<float>> floats;  // aligned copies of the part's float arrays
  const uint8_t *take(int64_t n) {
    if (bad || n < 0 || n > left) {
      bad = true;
      return nullptr;
    }
    const uint8_t *r = p;
    p += n;
    left -= n;
    return r;
  }
  const float *vec(int64_t n) {
    const uint8_t *b = take(4 * n);
    if (!b) return nullptr;
    floats.emplace_back((size_t)n);
    memcpy(floats.back().data(), b, 4 * (size_t)n);
    return floats.back().data();
  }
  rk_host_matrix mat(int64_t n, int fmt) {
    rk_host_matrix m{};
    m.fmt = fmt;
    switch (fmt) {
      case RK_FMT_Q8_0: m.scales = vec(n / 32); m.w = take(n); break;
      case RK_FMT_Q4_0: m.scales = vec(n / 32); m.w = take(n / 2); break;
      case RK_FMT_BF16: m.w = take(2 * n); break;
      default: m.w = take(4 * n); break;
    }
    return m;
  }
  bool done() const { return !bad && left == 0; }
};

// Config.embedType (model.go:96-101): the embedding table and a separate
// classifier stay q8_0 in quantized models.
static int embed_fmt(const rk_config *c) {
  return c->dtype == RK_DTYPE_F32 ? RK_FMT_F32 : c->dtype == RK_DTYPE_BF16 ? RK_FMT_BF16 : RK_FMT_Q8_0;
}

extern "C" int rk_layer_load_part(rk_device *d, const rk_config *c, const void *part, int64_t bytes, rk_layer **out) {
  if (!d || !c || !part || bytes < 0 || !out) return fail(RK_ERR_ARGS, "null argument");
  int rc = rk_config_validate(c);
  if (rc) return rc;
  const int64_t D = c->dim, hs = head_size(c), q = (int64_t)c->heads * hs, kv = (int64_t)c->kv_heads * hs, H = c->hidden;
  const int m = mat_fmt(c, false), sens = mat_fmt(c, true);
  PartDecoder dec{(const uint8_t *)part, bytes};
  rk_host_layer h{};  // Layer.tensors order, model.go:328-343
  h.rms_att = dec.vec(D);
  h.wq = dec.mat(q * D, m);
  h.wk = dec.mat(kv * D, m);
  h.wv = dec.mat(kv * D, sens);
  h.wo = dec.mat(D * q, m);
  h.rms_ffn = dec.vec(D);
  h.w1 = dec.mat(H * D, m);
  h.w2 = dec.mat(D * H, sens);
  h.w3 = dec.mat(H * D, m);
  if (c->qkv_bias) {
    h.bq = dec.vec(q);
    h.bk = dec.vec(kv);
    h.bv = dec.vec(kv);
  }
  if (c->qk_norm) {
    h.q_norm = dec.vec(hs);
    h.k_norm = dec.vec(hs);
  }
  if (!dec.done()) return fail(RK_ERR_ARGS, "model part has the wrong size");
  return rk_layer_upload(d, c, &h, out);
}

extern "C" int rk_embed_load_part(rk_device *d, const rk_config *c, const void *part, int64_t bytes, rk_matrix **out) {
  if (!d || !c || !part || bytes < 0 || !out) return fail(RK_ERR_ARGS, "null argument");
  int rc = rk_config_validate(c);
  if (rc) return rc;
  PartDecoder dec{(const uint8_t *)part, bytes};
  const rk_host_matrix e = dec.mat((int64_t)c->vocab * c->dim, embed_fmt(c));  // LoadEmbed, shard.go:282-287
  if (!dec.done()) return fail(RK_ERR_ARGS, "model part has the wrong size");
  return rk_matrix_upload(d, c->vocab, c->dim, e.fmt, e.w, e.scales, out);
}

extern "C" int rk_head_load_part(rk_device *d, const rk_config *c, const void *part, int64_t bytes, rk_matrix *embed,
                                 rk_matrix **wcls_out, rk_head **out) {
  if (!d || !c || !part || bytes < 0 || !out || !wcls_out) return fail(RK_ERR_ARGS, "null argument");
  int rc = rk_config_validate(c);
  if (rc) return rc;
  *wcls_out = nullptr;
  PartDecoder dec{(const uint8_t *)part, bytes};  // LoadHead, shard.go:292-300
  const float *rms = dec.vec(c->dim);
  rk_host_matrix w{};
  if (!c->shared_classifier) w = dec.mat((int64_t)c->vocab * c->dim, embed_fmt(c));
  if (!dec.done()) return fail(RK_ERR_ARGS, "model part has the wrong size");
  rk_matrix *wcls = embed;
  if (!c->shared_classifier) {
    if ((rc = rk_matrix_upload(d, c->vocab, c->dim, w.fmt, w.w, w.scales, &wcls))) return rc;
  } else if (!embed) {
    return fail(RK_ERR_ARGS, "a shared classifier needs the embedding table");
  }
  if ((rc = rk_head_new(d, c, rms, wcls, out))) {
    if (wcls != embed) rk_matrix_free(wcls);
    return rc;
  }
  if (wcls != embed) *wcls_out = wcls;
  return RK_OK;
}

// ---------------------------------------------------------------------------
// Layer pipeline: the stage plan (planStages, internal/llm/plan.go:122-207)
// and one rank's part of a pipelined step.
// ---------------------------------------------------------------------------
extern "C" int rk_plan_stages(const int64_t *cost, const int64_t *mem, int layers, const double *speed,
                              const int64_t *capacity, const int64_t *free_mem, int nodes, int stages, int *nspans,
                              int *span_node, int *span_from, int *span_to) {
  if (!cost || !mem || layers <= 0 || !speed || !capacity || nodes < 0 || !nspans || !span_node || !span_from ||
      !span_to)
    return fail(RK_ERR_ARGS, "bad argument");
  // fits(n, from, to): the node holds layers [from, to) (the reference's
  // nodeFit over memory, here the layers' bytes against the node's).
  std::vector<int64_t> msum(layers + 1, 0), sum(layers + 1, 0);
  for (int i = 0; i < layers; i++) {
    msum[i + 1] = msum[i] + mem[i];
    sum[i + 1] = sum[i] + cost[i];
  }
  auto fits = [&](int n, int from, int to) { return msum[to] - msum[from] <= capacity[n]; };
  // Nodes that hold at least one layer, fastest first (then more free
  // memory, then lower index: sortNodes, plan.go:103-113).
  std::vector<int> order;
  for (int n = 0; n < nodes; n++)
    for (int i = 0; i < layers; i++)
      if (fits(n, i, i + 1)) {
        order.push_back(n);
        break;
      }
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
    if (speed[a] != speed[b]) return speed[a] > speed[b];
    const int64_t fa = free_mem ? free_mem[a] : 0, fb = free_mem ? free_mem[b] : 0;
    if (fa != fb) return fa > fb;
    return a < b;
  });
  struct Span {
    int from, to, node;
  };
  std::vector<Span> out;
  if (stages <= 0) {
    // The fastest nodes take as many layers as they hold (plan.go:141-156).
    int at = 0;
    for (int n : order) {
      if (at == layers) break;
      int k = 0;
      while (k < layers - at && fits(n, at, at + k + 1)) k++;
      if (k > 0) {
        out.push_back({at, at + k, n});
        at += k;
      }
    }
    if (at < layers || out.empty()) return fail(RK_ERR_ARGS, "the model's %d layers do not fit the nodes", layers);
  } else {
    const int use = std::min(std::min(stages, (int)order.size()), layers);
    order.resize(use);
    if (order.empty()) return fail(RK_ERR_ARGS, "no node holds a layer");
    // Cut the layers, in node order, into stages within `bound` (seconds
    // per token: bytes over speed), each later node keeping a layer.
    auto cut = [&](double bound, std::vector<Span> *res) {
      int at = 0;
      for (int j = 0; j < use; j++) {
        const int n = order[j], left = use - j - 1;
        int k = 0;
        while (at + k < layers - left && fits(n, at, at + k + 1) &&
               (double)(sum[at + k + 1] - sum[at]) / std::max(speed[n], 1e-9) <= bound)
          k++;
        if (k == 0) return false;
        if (res) res->push_back({at, at + k, n});
        at += k;
      }
      return at >= layers;
    };
    std::vector<double> bounds;
    for (int n : order)
      for (int i = 0; i < layers; i++)
        for (int j = i + 1; j <= layers; j++) bounds.push_back((double)(sum[j] - sum[i]) / std::max(speed[n], 1e-9));
    std::sort(bounds.begin(), bounds.end());
    bounds.erase(std::unique(bounds.begin(), bounds.end()), bounds.end());
    // Go's lower-bound search over "cut succeeds" (slices.BinarySearchFunc),
    // as the reference does. Where capacities make cutting non-monotone in
    // the bound, its answer is still the reference's.
    size_t lo = 0, hi = bounds.size();
    while (lo < hi) {
      const size_t mid = (lo + hi) / 2;
      if (cut(bounds[mid], nullptr)) hi = mid;
      else lo = mid + 1;
    }
    if (lo == bounds.size())
      return fail(RK_ERR_ARGS, "the model's %d layers do not fit the %d fastest nodes", layers, use);
    cut(bounds[lo], &out);
  }
  const int cap = *nspans;
  if ((int)out.size() > cap) {
    *nspans = (int)out.size();
    return fail(RK_ERR_ARGS, "%d spans do not fit the %d given", (int)out.size(), cap);
  }
  *nspans = (int)out.size();
  for (size_t i = 0; i < out.size(); i++) {
    span_node[i] = out[i].node;
    span_from[i] = out[i].from;
    span_to[i] = out[i].to;
  }
  return RK_OK;
}

struct rk_pipeline {
  rk_device *d = nullptr;
  rk_group *grp = nullptr;
  rk_matrix *embed = nullptr;  // first rank
  rk_stage *stage = nullptr;
  rk_head *head = nullptr;  // last rank
  int *token_dev = nullptr, *next_dev = nullptr;
  unsigned long long *key_dev = nullptr;
  int *pin_tok = nullptr;
  float *pin_logits = nullptr;
  cudaGraphExec_t graph = nullptr;
};

static void pipeline_release(rk_pipeline *p) {
  if (!p) return;
  cudaSetDevice(p->d->ordinal);
  cudaStreamSynchronize(p->d->st);
  if (p->graph) cudaGraphExecDestroy(p->graph);
  cudaFree(p->token_dev);
  cudaFree(p->next_dev);
  cudaFree(p->key_dev);
  cudaFreeHost(p->pin_tok);
  cudaFreeHost(p->pin_logits);
  delete p;
}

// One rank's step: x from the previous rank (or the embedding of *token_dev
// on the first), this rank's layers, x on to the next rank (or the head and
// argmax on the last), then the next token from the last rank to all.
static int record_pipeline(rk_pipeline *p, cudaStream_t st) {
  rk_stage *s = p->stage;
  rk_group *g = p->grp;
  const int D = s->c.dim, last = g->n - 1;
  ncclResult_t r;
  if (g->rank == 0) {
    CK(launch_embed(p->embed->fmt, p->embed->w, p->embed->s, p->embed->rows, D, p->token_dev, s->x, p->d->err_dev, st));
  } else if ((r = nccl().recv(s->x, D, ncclFloat32, g->rank - 1, g->comm, st)) != ncclSuccess) {
    return nccl_fail(r, "pipeline receive");
  }
  int rc = record_layers(s, st);
  if (rc) return rc;
  if (g->rank < last) {
    if ((r = nccl().send(s->x, D, ncclFloat32, g->rank + 1, g->comm, st)) != ncclSuccess)
      return nccl_fail(r, "pipeline send");
  } else {
    if ((rc = record_head(p->head, s->x, st))) return rc;
    CK(launch_argmax_multi(p->head->logits, s->c.vocab, p->key_dev, p->next_dev, nullptr, st));
  }
  if ((r = nccl().broadcast(p->next_dev, p->next_dev, 1, ncclInt32, last, g->comm, st)) != ncclSuccess)
    return nccl_fail(r, "pipeline token broadcast");
  CK(cudaGetLastError());
  return RK_OK;
}

extern "C" int rk_pipeline_new(rk_group *g, rk_matrix *embed, rk_stage *stage, rk_head *head, rk_pipeline **out) {
  if (!g || !stage || !out) return fail(RK_ERR_ARGS, "null argument");
  if (g->n < 2) return fail(RK_ERR_ARGS, "a pipeline needs at least two ranks");
  if (stage->d != g->d || stage->G != 1) return fail(RK_ERR_ARGS, "the stage must be a whole (unsharded) stage on the group's device");
  const bool first = g->rank == 0, last = g->rank == g->n - 1;
  if (first != (embed != nullptr)) return fail(RK_ERR_ARGS, "the first rank, and only it, passes the embedding table");
  if (last != (head != nullptr)) return fail(RK_ERR_ARGS, "the last rank, and only it, passes the head");
  if (embed && (embed->d != g->d || embed->rows != stage->c.vocab || embed->cols != stage->c.dim))
    return fail(RK_ERR_ARGS, "embedding table of the wrong shape or device");
  if (head && (head->d != g->d || head->grp)) return fail(RK_ERR_ARGS, "the head must be a whole head on the group's device");
  rk_device *d = g->d;
  Guard gd(d);
  int rc = set_device(d);
  if (rc) return rc;
  auto *p = new rk_pipeline();
  p->d = d;
  p->grp = g;
  p->embed = embed;
  p->stage = stage;
  p->head = head;
  cudaError_t e = cudaMalloc(&p->token_dev, 16);
  if (e == cudaSuccess) e = cudaMemset(p->token_dev, 0, 16);
  if (e == cudaSuccess) e = cudaMalloc(&p->next_dev, 16);
  if (e == cudaSuccess) e = cudaMemset(p->next_dev, 0, 16);
  if (e == cudaSuccess) e = cudaMalloc(&p->key_dev, 16);
  if (e == cudaSuccess) e = cudaMemset(p->key_dev, 0, 16);
  if (e == cudaSuccess) e = cudaMallocHost(&p->pin_tok, 64);
  if (e == cudaSuccess && last) e = cudaMallocHost(&p->pin_logits, 4 * (size_t)stage->c.vocab);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->st);
  if (e != cudaSuccess) {
    pipeline_release(p);
    return cuda_fail(e, "pipeline allocation");
  }
  if ((rc = capture(d, [p](cudaStream_t st) { return record_pipeline(p, st); }, &p->graph))) {
    pipeline_release(p);
    return rc;
  }
  *out = p;
  return RK_OK;
}

extern "C" void rk_pipeline_free(rk_pipeline *p) {
  if (!p) return;
  rk_device *d = p->d;
  Guard g(d);
  pipeline_release(p);
}

extern "C" int rk_pipeline_step(rk_pipeline *p, int token, int pos, float *logits, int *next) {
  if (!p) return fail(RK_ERR_ARGS, "null pipeline");
  rk_stage *s = p->stage;
  if (pos < 0 || pos >= s->ctx) return fail(RK_ERR_ARGS, "position %d outside the stage's %d", pos, s->ctx);
  if (token < 0 || token >= s->c.vocab) return fail(RK_ERR_ARGS, "token %d outside the vocabulary", token);
  rk_device *d = p->d;
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  p->pin_tok[0] = token;
  p->pin_tok[1] = pos;
  CK(cudaMemcpyAsync(p->token_dev, &p->pin_tok[0], 4, cudaMemcpyHostToDevice, d->st));
  CK(cudaMemcpyAsync(s->pos_dev, &p->pin_tok[1], 4, cudaMemcpyHostToDevice, d->st));
  CK(cudaGraphLaunch(p->graph, d->st));
  const bool last = p->grp->rank == p->grp->n - 1;
  if (logits && last)
    CK(cudaMemcpyAsync(p->pin_logits, p->head->logits, 4 * (size_t)s->c.vocab, cudaMemcpyDeviceToHost, d->st));
  CK(cudaMemcpyAsync(&p->pin_tok[2], p->next_dev, 4, cudaMemcpyDeviceToHost, d->st));
  if ((rc = sync_dev(d))) return rc;
  if (logits && last) memcpy(logits, p->pin_logits, 4 * (size_t)s->c.vocab);
  if (next) *next = p->pin_tok[2];
  return RK_OK;
}

extern "C" int rk_bench_pipeline(rk_pipeline *p, int pos, int iters, float *ms_per_step) {
  if (!p || iters <= 0 || !ms_per_step) return fail(RK_ERR_ARGS, "bad argument");
  rk_device *d = p->d;
  if (pos < 0 || pos >= p->stage->ctx) return fail(RK_ERR_ARGS, "position out of range");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  p->pin_tok[4] = pos;
  p->pin_tok[5] = 0;
  CK(cudaMemcpyAsync(p->token_dev, &p->pin_tok[5], 4, cudaMemcpyHostToDevice, d->st));
  CK(cudaEventRecord(e0, d->st));
  for (int i = 0; i < iters; i++) {
    CK(cudaMemcpyAsync(p->stage->pos_dev, &p->pin_tok[4], 4, cudaMemcpyHostToDevice, d->st));
    CK(cudaGraphLaunch(p->graph, d->st));
  }
  CK(cudaEventRecord(e1, d->st));
  CK(cudaEventSynchronize(e1));
  float ms = 0.0f;
  CK(cudaEventElapsedTime(&ms, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if ((rc = check_dev_err(d))) return rc;
  *ms_per_step = ms / iters;
  return RK_OK;
}

// ---------------------------------------------------------------------------
// Accessors for rk_noalloc.cu (C++ linkage, not part of the C ABI).
// ---------------------------------------------------------------------------
namespace rk {
int internal_fail(int code, const char *msg) { return fail(code, "%s", msg); }

int internal_matrix_view(const rk_matrix *m, int *device, int *rows, int *cols, int *fmt, const void **w,
                         const float **scales, void **stream, int **err_word, int *sms) {
  if (!m) return fail(RK_ERR_ARGS, "null matrix");
  *device = m->d->ordinal;
  *rows = m->rows;
  *cols = m->cols;
  *fmt = m->fmt;
  *w = m->w;
  *scales = m->s;
  *stream = m->d->st;
  *err_word = m->d->err_dev;
  *sms = m->d->sms;
  return RK_OK;
}

// The matrix's device mutex, held by rk_matrix_mulvec_noalloc for its whole
// call as every other entry point holds it.
void internal_device_lock(const rk_matrix *m) { m->d->mu.lock(); }
void internal_device_unlock(const rk_matrix *m) { m->d->mu.unlock(); }

// Reads and clears the device error word, with check_dev_err's mapping of
// the word to a status (call with the device mutex held, after a sync).
int internal_check_dev_err(const rk_matrix *m) { return check_dev_err(m->d); }
}  // namespace rk

extern "C" int rk_sample_argmax(rk_device *d, const float *logits, int n, int *index) {
  if (!d || !logits || !index || n <= 0 || n > RK_MAX_ROWS) return fail(RK_ERR_ARGS, "bad argument");
  Guard g(d);
  int rc = set_device(d);
  if (rc) return rc;
  memcpy(d->pin_out, logits, sizeof(float) * (size_t)n);
  CK(cudaMemcpyAsync(d->mv_out, d->pin_out, sizeof(float) * (size_t)n, cudaMemcpyHostToDevice, d->st));
  // The key and the index use the device scratch of MulVecs (mv_xsum).
  unsigned long long *key = reinterpret_cast<unsigned long long *>(d->mv_xsum);
  CK(cudaMemsetAsync(key, 0, sizeof *key, d->st));
  CK(launch_argmax_multi(d->mv_out, n, key, d->mv_xsum + 2, nullptr, d->st));
  CK(cudaMemcpyAsync(d->pin_in, d->mv_xsum + 2, sizeof(int), cudaMemcpyDeviceToHost, d->st));
  if ((rc = sync_dev(d))) return rc;
  memcpy(index, d->pin_in, sizeof(int));
  return RK_OK;
}
