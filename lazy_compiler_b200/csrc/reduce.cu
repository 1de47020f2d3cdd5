// Whole-array FP32 sum and mean.
//
// The reference lowers r01/r02/r03 to ONE CTA of 128 threads
// (problems/r02_big_sum/meta.json grid [1,1,1]): a strided fp32 accumulate
// (ptx_backend.py:1496-1554 loop), a shfl.sync.bfly butterfly (:1668-1703
// shuffle) and a 4-slot shared tree (:1705-1744 tree); r03 divides by the
// count buffer.  At 2^24 elements that is 131,072 dependent loads per thread
// on one of 148 SMs.
//
// Here one launch covers the whole array: a grid of up to 2 CTAs x 512
// threads per SM strides over the array with 128-bit streaming loads, each
// thread keeps an error-free compensated fp32 sum (TwoSum), the block tree
// combines in f64 and writes one f64 partial per CTA, and the last CTA to
// finish (atomic ticket after a fence) adds the partials in a fixed order and
// writes the fp32 result.  The order of every addition is fixed by the grid,
// so the result is deterministic; the f64 combine makes it the correctly
// rounded fp32 value of the exact sum in all but tie cases.
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace lc {
namespace {

constexpr int kThreads = 512;
constexpr int kBlocksPerSm = 2;
constexpr int kUnroll = 4;

__device__ __forceinline__ void accumulate(CompSum &acc, const float *__restrict__ x, int64_t n) {
  const int64_t nvec = n >> 2;
  const float4 *xv = reinterpret_cast<const float4 *>(x);
  const int64_t tile = (int64_t)kThreads * kUnroll;
  for (int64_t base = (int64_t)blockIdx.x * tile; base < nvec; base += (int64_t)gridDim.x * tile) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * kThreads + threadIdx.x;
      v[u] = i < nvec ? ld_stream(xv + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      acc.add(v[u].x);
      acc.add(v[u].y);
      acc.add(v[u].z);
      acc.add(v[u].w);
    }
  }
  if (blockIdx.x == 0) {
    const int64_t i = (nvec << 2) + threadIdx.x;
    if (i < n) acc.add(x[i]);
  }
}

__device__ __forceinline__ void accumulate_scalar(CompSum &acc, const float *__restrict__ x,
                                                  int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    acc.add(x[i]);
}

// Peer-memory exchange of the shard sums of one range-sharded reduction (one
// process per GPU).  Every rank owns one mailbox in its own device memory,
// with a call counter (the epoch) that only its own kernels touch.  The last
// CTA of a rank's reduction takes epoch e = counter + 1, stores its f64 shard
// sum into slot [e & 1][rank] of every rank's mailbox (its own included) over
// NVLink and raises the flag next to it with a system-scope release; it then
// waits (bounded) until all flags of that slot in its own mailbox carry e,
// adds the shard sums in rank order (so every rank computes the same value)
// and stores e back as the counter.  The epoch lives on the device, so the
// call can be replayed from a CUDA graph.  Two slots alternate by epoch
// parity: a rank can only write epoch e+2 into a peer's mailbox after that
// peer wrote epoch e+1, i.e. after the peer's kernel of epoch e (and its reads
// of slot e & 1) finished, so no slot is overwritten while it is read.
struct PeerBox {
  double partial[2][LC_PEER_MAX_RANKS];
  unsigned int flag[2][LC_PEER_MAX_RANKS];
  unsigned int epoch;
};
static_assert(sizeof(PeerBox) <= LC_PEER_MAILBOX_BYTES, "mailbox layout exceeds its allocation");
struct PeerSet {
  PeerBox *box[LC_PEER_MAX_RANKS];
  int world, rank;
  int *err;
};
constexpr uint64_t kPeerWaitLimitNs = 5000000000ull;  // ranks may reach the kernel seconds apart
constexpr int kErrTimeoutPeer = 7;

__device__ __forceinline__ void st_release_sys(unsigned int *p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int *p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_f64(double *p, double v) {
  asm volatile("st.relaxed.sys.global.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}
__device__ __forceinline__ double ld_relaxed_sys_f64(const double *p) {
  double v;
  asm volatile("ld.relaxed.sys.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Run by the first warp of the last CTA: exchange `total` with the peers and
// return the sum over all ranks (NaN if a peer did not arrive in time).
__device__ double peer_exchange(double total, const PeerSet &peers) {
  PeerBox *mine = peers.box[peers.rank];
  const int t = threadIdx.x;
  unsigned int epoch = 0;
  if (t == 0) epoch = *reinterpret_cast<volatile unsigned int *>(&mine->epoch) + 1u;
  epoch = __shfl_sync(0xffffffffu, epoch, 0);
  const unsigned int slot = epoch & 1u;
  double value = 0.0;
  bool ok = true;
  if (t < peers.world) {
    PeerBox *dst = peers.box[t];
    st_relaxed_sys_f64(&dst->partial[slot][peers.rank], total);
    st_release_sys(&dst->flag[slot][peers.rank], epoch);  // orders the store above
    const unsigned int *flag = &mine->flag[slot][t];
    ok = ld_acquire_sys(flag) == epoch;
    if (!ok) {
      const uint64_t start = globaltimer_ns();
      for (uint32_t i = 1; !ok; ++i) {
        ok = ld_acquire_sys(flag) == epoch;
        if (!ok && (i & 63) == 0 && globaltimer_ns() - start > kPeerWaitLimitNs) break;
      }
    }
    if (ok) value = ld_relaxed_sys_f64(&mine->partial[slot][t]);
    else if (peers.err) atomicCAS(peers.err, 0, kErrTimeoutPeer);
  }
  const bool failed = __any_sync(0xffffffffu, !ok);
  double sum = 0.0;
  for (int r = 0; r < peers.world; ++r) sum += __shfl_sync(0xffffffffu, value, r);  // rank order
  if (t == 0) *reinterpret_cast<volatile unsigned int *>(&mine->epoch) = epoch;
  return failed ? __longlong_as_double(0x7ff8000000000000ll) : sum;
}

// mode 0: out = sum; mode 1: out = sum / count[0]; mode 2: partial_out = sum (f64);
// mode 3: out = (sum over the ranks of `peers`) [/ count[0] when count != NULL]
template <bool VEC>
__global__ void __launch_bounds__(kThreads, kBlocksPerSm) sum_kernel(const float *__restrict__ x, int64_t n,
                                                       double *__restrict__ partials,
                                                       unsigned int *__restrict__ counter,
                                                       int mode, const float *__restrict__ count,
                                                       float *__restrict__ out,
                                                       double *__restrict__ partial_out,
                                                       const PeerSet peers) {
  __shared__ double scratch[32];
  __shared__ bool is_last;
  pdl_wait();     // x and the workspace may be the previous kernel's
  pdl_trigger();  // the next kernel may be scheduled while this one drains
  CompSum acc;
  if (VEC) accumulate(acc, x, n);
  else accumulate_scalar(acc, x, n);
  const double block_total = block_sum<double>(acc.value(), scratch);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = block_total;
    // the ticket releases this CTA's partial and, for the last CTA, acquires all of them
    unsigned int ticket;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(ticket) : "l"(counter) : "memory");
    is_last = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last || threadIdx.x >= 32) return;
  // the last CTA's first warp adds the partials in a fixed order (lane-strided, then
  // the butterfly), so the result does not depend on which CTA finished last
  double t = 0.0;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += 32) t += __ldcg(partials + i);
  double total = warp_sum(t);
  if (mode == 3) total = peer_exchange(total, peers);
  if (threadIdx.x == 0) {
    if (mode == 0) out[0] = (float)total;
    else if (mode == 1) out[0] = (float)(total / (double)__ldg(count));
    else if (mode == 2) partial_out[0] = total;
    else out[0] = count ? (float)(total / (double)__ldg(count)) : (float)total;
    *counter = 0u;  // ready for the next launch on this workspace
  }
}

__global__ void finalize_kernel(const double *__restrict__ total, const float *__restrict__ count,
                                float *__restrict__ out) {
  const double t = *total;
  out[0] = count ? (float)(t / (double)*count) : (float)t;
}

int launch_sum(const char *name, const float *x, int64_t n, int mode, const float *count,
               float *out, double *partial_out, void *stream, const PeerSet *peers = nullptr) {
  if (n < 0 || (!x && n > 0)) return fail(LC_ERR_INVALID, "%s: null input or negative length", name);
  if ((mode < 2 || mode == 3) && !out) return fail(LC_ERR_INVALID, "%s: null output", name);
  if (mode == 1 && !count) return fail(LC_ERR_INVALID, "%s: null count", name);
  if (mode == 2 && !partial_out) return fail(LC_ERR_INVALID, "%s: null partial", name);
  cudaStream_t s = as_stream(stream);
  ReduceWorkspace ws;
  if (int rc = reduce_workspace(s, &ws)) return rc;
  const bool vec = aligned(x, 16);
  const int64_t per_block = vec ? (int64_t)kThreads * kUnroll * 4 : (int64_t)kThreads;
  int64_t blocks = (n + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * kBlocksPerSm;
  if (blocks > cap) blocks = cap;
  if (blocks > kMaxPartials) blocks = kMaxPartials;
  if (blocks < 1) blocks = 1;
  PeerSet none{};
  const PeerSet &p = peers ? *peers : none;
  cudaError_t e = vec ? launch_pdl(sum_kernel<true>, dim3((unsigned)blocks), dim3(kThreads), 0, s, x, n,
                                    ws.partials, ws.counter, mode, count, out, partial_out, p)
                      : launch_pdl(sum_kernel<false>, dim3((unsigned)blocks), dim3(kThreads), 0, s, x, n,
                                    ws.partials, ws.counter, mode, count, out, partial_out, p);
  if (e != cudaSuccess) return check_cuda(e, name);
  return check_launch(name);
}

}  // namespace
}  // namespace lc

// ---------------------------------------------------------------- no-allocation variant
//
// lc_sum_f32 keeps its per-CTA partials in a workspace the library creates
// with cudaMalloc on the first call per (device, stream).  Some callers cannot
// let a library allocate: applications whose device memory is entirely owned
// by their own allocator (a framework's caching pool, or a service that
// reserves the GPU's memory at start-up), and launch paths that must not pay
// cudaMalloc's implicit device-wide synchronisation.  lc_sum_f32_noalloc runs
// the same kernel with its scratch in this fixed-size device array instead.
// Every device on which the library's module has been loaded holds the array
// (LC_SUM_NOALLOC_SCRATCH_BYTES) until the process exits; all calls share it,
// so calls that overlap on the GPU (different streams, or other threads) race
// on it.  The array bounds the number of CTAs (one f64 partial each), not n.
namespace {
static __device__ __align__(256) unsigned char
    g_sum_noalloc_scratch[LC_SUM_NOALLOC_MAX_BLOCKS * sizeof(double) + 256];

std::mutex g_noalloc_mutex;
unsigned char *g_noalloc_address[64] = {nullptr};

// Device address of g_sum_noalloc_scratch on the current device.  Host code
// only sees a host-side stand-in under that name, so the address is looked up
// once per device (with that device current) and cached for the life of the
// process; a device reset would invalidate it, and the library must not
// outlive one.  The lookup also loads the module on the device under lazy
// loading, so the first call per device must precede any stream capture.
int noalloc_scratch(unsigned char **out) {
  int dev = 0;
  if (int rc = lc::check_cuda(cudaGetDevice(&dev), "lc_sum_f32_noalloc: cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64)
    return lc::fail(LC_ERR_UNSUPPORTED, "lc_sum_f32_noalloc: device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_address[dev]) {
    void *ptr = nullptr;
    if (int rc = lc::check_cuda(cudaGetSymbolAddress(&ptr, g_sum_noalloc_scratch),
                                "lc_sum_f32_noalloc: cudaGetSymbolAddress"))
      return rc;
    g_noalloc_address[dev] = static_cast<unsigned char *>(ptr);
  }
  *out = g_noalloc_address[dev];
  return LC_OK;
}
}  // namespace

extern "C" int lc_sum_f32_noalloc(const float *x, float *out, int64_t n, void *stream) {
  using namespace lc;
  if (n < 0 || (!x && n > 0) || !out)
    return fail(LC_ERR_INVALID, "lc_sum_f32_noalloc: null buffer or negative length");
  if (n > LC_SUM_NOALLOC_MAX_N)
    return fail(LC_ERR_UNSUPPORTED,
                "lc_sum_f32_noalloc: n = %lld exceeds the maximum of %lld elements; use lc_sum_f32",
                (long long)n, (long long)LC_SUM_NOALLOC_MAX_N);
  unsigned char *scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  double *partials = reinterpret_cast<double *>(scratch);
  unsigned int *counter =
      reinterpret_cast<unsigned int *>(scratch + LC_SUM_NOALLOC_MAX_BLOCKS * sizeof(double));
  cudaStream_t s = as_stream(stream);
  const bool vec = aligned(x, 16);
  const int64_t per_block = vec ? (int64_t)kThreads * kUnroll * 4 : (int64_t)kThreads;
  int64_t blocks = (n + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * kBlocksPerSm;
  if (blocks > cap) blocks = cap;
  // grid-stride and int64-indexed: a grid clamped to the array's partials covers any n
  if (blocks > LC_SUM_NOALLOC_MAX_BLOCKS) blocks = LC_SUM_NOALLOC_MAX_BLOCKS;
  if (blocks < 1) blocks = 1;
  // the CTA ticket counter must start at zero; the array keeps the last call's contents
  if (int rc = check_cuda(cudaMemsetAsync(counter, 0, sizeof(unsigned int), s),
                          "lc_sum_f32_noalloc: clear counter"))
    return rc;
  if (vec)
    sum_kernel<true><<<(int)blocks, kThreads, 0, s>>>(x, n, partials, counter, 0, nullptr, out,
                                                      nullptr, PeerSet{});
  else
    sum_kernel<false><<<(int)blocks, kThreads, 0, s>>>(x, n, partials, counter, 0, nullptr, out,
                                                       nullptr, PeerSet{});
  return check_launch("lc_sum_f32_noalloc");
}

extern "C" int lc_sum_f32(const float *x, float *out, int64_t n, void *stream) {
  return lc::launch_sum("lc_sum_f32", x, n, 0, nullptr, out, nullptr, stream);
}

extern "C" int lc_mean_f32(const float *x, const float *count, float *out, int64_t n,
                           void *stream) {
  return lc::launch_sum("lc_mean_f32", x, n, 1, count, out, nullptr, stream);
}

extern "C" int lc_sum_partial_f32(const float *x, int64_t n, double *partial, void *stream) {
  return lc::launch_sum("lc_sum_partial_f32", x, n, 2, nullptr, nullptr, partial, stream);
}

extern "C" int lc_sum_finalize(const double *total, const float *count, float *out,
                               void *stream) {
  if (!total || !out) return lc::fail(LC_ERR_INVALID, "lc_sum_finalize: null buffer");
  lc::finalize_kernel<<<1, 1, 0, lc::as_stream(stream)>>>(total, count, out);
  return lc::check_launch("lc_sum_finalize");
}

// ---------------------------------------------------------------- peer mailboxes

namespace {
std::mutex g_peer_mutex;
void *g_peer_mailbox[64] = {nullptr};
}  // namespace

extern "C" int lc_peer_mailbox(void **mailbox, unsigned char *handle) {
  using namespace lc;
  if (!mailbox || !handle) return fail(LC_ERR_INVALID, "lc_peer_mailbox: null argument");
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "lc_peer_mailbox: cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(LC_ERR_UNSUPPORTED, "lc_peer_mailbox: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_peer_mutex);
  if (!g_peer_mailbox[dev]) {
    void *mem = nullptr;
    if (cudaMalloc(&mem, LC_PEER_MAILBOX_BYTES) != cudaSuccess) {
      cudaGetLastError();
      return fail(LC_ERR_NOMEM, "lc_peer_mailbox: cudaMalloc(%d) failed", LC_PEER_MAILBOX_BYTES);
    }
    // flags and the epoch counter start at 0; the first call uses epoch 1
    if (int rc = check_cuda(cudaMemset(mem, 0, LC_PEER_MAILBOX_BYTES), "lc_peer_mailbox: memset")) {
      cudaFree(mem);
      return rc;
    }
    g_peer_mailbox[dev] = mem;
  }
  cudaIpcMemHandle_t h;
  if (int rc = check_cuda(cudaIpcGetMemHandle(&h, g_peer_mailbox[dev]), "lc_peer_mailbox: cudaIpcGetMemHandle"))
    return rc;
  memcpy(handle, &h, LC_PEER_HANDLE_BYTES);
  *mailbox = g_peer_mailbox[dev];
  return LC_OK;
}

extern "C" int lc_peer_open(const unsigned char *handle, void **peer_mailbox) {
  using namespace lc;
  if (!handle || !peer_mailbox) return fail(LC_ERR_INVALID, "lc_peer_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, LC_PEER_HANDLE_BYTES);
  return check_cuda(cudaIpcOpenMemHandle(peer_mailbox, h, cudaIpcMemLazyEnablePeerAccess),
                    "lc_peer_open: cudaIpcOpenMemHandle");
}

extern "C" int lc_peer_close(void *peer_mailbox) {
  if (!peer_mailbox) return lc::fail(LC_ERR_INVALID, "lc_peer_close: null mailbox");
  return lc::check_cuda(cudaIpcCloseMemHandle(peer_mailbox), "lc_peer_close: cudaIpcCloseMemHandle");
}

extern "C" int lc_peer_reset(void *stream) {
  using namespace lc;
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "lc_peer_reset: cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(LC_ERR_UNSUPPORTED, "lc_peer_reset: device %d out of range", dev);
  void *box = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_peer_mutex);
    box = g_peer_mailbox[dev];
  }
  if (!box) return LC_OK;
  return check_cuda(cudaMemsetAsync(box, 0, LC_PEER_MAILBOX_BYTES, as_stream(stream)), "lc_peer_reset");
}

extern "C" int lc_sum_peer_f32(const float *x, int64_t n, const float *count, float *out,
                               void *const *mailboxes, int world, int rank, void *stream) {
  using namespace lc;
  if (!mailboxes || world < 1 || world > LC_PEER_MAX_RANKS || rank < 0 || rank >= world)
    return fail(LC_ERR_INVALID, "lc_sum_peer_f32: bad rank %d of %d (at most %d ranks)", rank, world,
                LC_PEER_MAX_RANKS);
  PeerSet peers{};
  for (int r = 0; r < world; ++r) {
    if (!mailboxes[r]) return fail(LC_ERR_INVALID, "lc_sum_peer_f32: null mailbox of rank %d", r);
    if (!aligned(mailboxes[r], 16)) return fail(LC_ERR_ALIGN, "lc_sum_peer_f32: unaligned mailbox");
    peers.box[r] = static_cast<PeerBox *>(mailboxes[r]);
  }
  peers.world = world;
  peers.rank = rank;
  if (int rc = device_error_word(&peers.err)) return rc;
  return launch_sum("lc_sum_peer_f32", x, n, 3, count, out, nullptr, stream, &peers);
}
