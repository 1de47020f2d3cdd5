// Library plumbing: version, per-thread error messages, device facts and the
// library-owned reduction workspace.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "common.cuh"

namespace {
thread_local char g_message[512] = "";
thread_local int g_status = LC_OK;

std::mutex g_mutex;
std::map<std::pair<int, cudaStream_t>, lc::ReduceWorkspace> g_workspaces;
struct Scratch {
  void *ptr = nullptr;
  size_t bytes = 0;
};
std::map<std::tuple<int, cudaStream_t, int>, Scratch> g_scratch;
int *g_error_words[64] = {nullptr};
int g_sms[64] = {0};
}  // namespace

namespace lc {

int fail(int code, const char *fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_message, sizeof(g_message), fmt, args);
  va_end(args);
  g_status = code;
  return code;
}

int check_cuda(cudaError_t err, const char *what) {
  if (err == cudaSuccess) return LC_OK;
  return fail(LC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

int check_launch(const char *what) { return check_cuda(cudaGetLastError(), what); }

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (g_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

int reduce_workspace(cudaStream_t stream, ReduceWorkspace *out) {
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  std::lock_guard<std::mutex> lock(g_mutex);
  auto key = std::make_pair(dev, stream);
  auto it = g_workspaces.find(key);
  if (it != g_workspaces.end()) {
    *out = it->second;
    return LC_OK;
  }
  void *mem = nullptr;
  const size_t bytes = kMaxPartials * sizeof(double) + 256;
  if (cudaMalloc(&mem, bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(LC_ERR_NOMEM, "reduction workspace: cudaMalloc(%zu) failed", bytes);
  }
  // synchronous memset: the counter must read zero before any kernel uses it
  if (int rc = check_cuda(cudaMemset(mem, 0, bytes), "workspace memset")) {
    cudaFree(mem);
    return rc;
  }
  ReduceWorkspace ws;
  ws.partials = static_cast<double *>(mem);
  ws.counter = reinterpret_cast<unsigned int *>(static_cast<char *>(mem) +
                                                kMaxPartials * sizeof(double));
  g_workspaces.emplace(key, ws);
  *out = ws;
  return LC_OK;
}

int scratch_buffer(cudaStream_t stream, int slot, size_t bytes, void **out) {
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  std::lock_guard<std::mutex> lock(g_mutex);
  Scratch &sc = g_scratch[std::make_tuple(dev, stream, slot)];
  if (sc.bytes < bytes) {
    if (sc.ptr) {
      // the stream may still read the old buffer
      if (int rc = check_cuda(cudaStreamSynchronize(stream), "scratch: stream")) return rc;
      cudaFree(sc.ptr);
      sc.ptr = nullptr;
      sc.bytes = 0;
    }
    void *mem = nullptr;
    if (cudaMalloc(&mem, bytes) != cudaSuccess) {
      cudaGetLastError();
      return fail(LC_ERR_NOMEM, "scratch: cudaMalloc(%zu) failed", bytes);
    }
    sc.ptr = mem;
    sc.bytes = bytes;
  }
  *out = sc.ptr;
  return LC_OK;
}

int device_error_word(int **out) {
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(LC_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_error_words[dev]) {
    void *mem = nullptr;
    if (cudaMalloc(&mem, 256) != cudaSuccess) {
      cudaGetLastError();
      return fail(LC_ERR_NOMEM, "device error word: cudaMalloc failed");
    }
    if (int rc = check_cuda(cudaMemset(mem, 0, 256), "error word memset")) {
      cudaFree(mem);
      return rc;
    }
    g_error_words[dev] = static_cast<int *>(mem);
  }
  *out = g_error_words[dev];
  return LC_OK;
}

}  // namespace lc

extern "C" int lc_device_status(void *stream) {
  int *word = nullptr;
  if (int rc = lc::device_error_word(&word)) return rc;
  cudaStream_t s = lc::as_stream(stream);
  if (int rc = lc::check_cuda(cudaStreamSynchronize(s), "lc_device_status: stream")) return rc;
  int value = 0;
  if (int rc = lc::check_cuda(cudaMemcpy(&value, word, sizeof(int), cudaMemcpyDeviceToHost),
                              "lc_device_status: read"))
    return rc;
  if (value == 0) return LC_OK;
  cudaMemset(word, 0, sizeof(int));
  return lc::fail(LC_ERR_TIMEOUT,
                  "a bounded device wait gave up (code %d: 1 producer, 2 mma, 3 epilogue, "
                  "4 softmax, 5 correction)",
                  value);
}

extern "C" int lc_version(void) { return 1 * 10000 + 0 * 100 + 0; }

extern "C" int lc_last_error(char *buf, size_t len) {
  if (buf && len) {
    strncpy(buf, g_message, len - 1);
    buf[len - 1] = '\0';
  }
  return g_status;
}
