// abi.cu -- the library's C ABI (include/anima_rt.h, include/anima_attn.h).
//
// Two layers:
//  * anima_attn_*: device pointers + stream, asynchronous, int status codes.
//  * anima_rt_*:   drop-in replacements of the reference runtime's extern "C" entries
//    (anima_rt/src/anima_rt.cpp:11-173): fp32 host pointers, bool returns.  Each call
//    copies its operands into a device workspace owned by the library, runs the
//    kernels on the library's stream, copies the result back and synchronises.
//    Calls are serialised by one mutex (one workspace); like the reference they are
//    safe to call from several threads.
#include <sched.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <initializer_list>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "anima_rt.h"
#include "common.cuh"

namespace anima {
int attn_fwd_launch(const AnimaAttnArgs* a, int* status, int sm_count, cudaStream_t st,
                    void* const* peers = nullptr, int n_peers = 0, int peer_rows = 0,
                    long long peer_row_stride = 0, int peer_head0 = 0);
int qkv_projection_scatter_launch(const AnimaQkvProjArgs* a, int rows, int row0,
                                  void* const* dest, int n_dest, int* status, int sm_count,
                                  cudaStream_t st);
int attn_fwd_pair_launch(const AnimaAttnArgs* a, int* status, cudaStream_t st);
size_t attn_workspace_bytes(int B, int H, int S_q, int S_kv, unsigned flags, int sm_count);
int attn_schedule_mode(int B, int H, int S_q, int S_kv, unsigned flags, int sm_count);
int selftest_wait_launch(int* status, unsigned timeout_us, cudaStream_t st);
int ln_modulate_launch(const float* x, const float* scale, const float* shift, long long mod_stride,
                       void* y, int out_dtype, long long rows, int rows_per_b, int D, float eps,
                       int sm_count, cudaStream_t st);
int gate_residual_launch(float* x, const float* gate, long long gate_stride, const float* y,
                         long long rows, int rows_per_b, int D, int sm_count, cudaStream_t st);
int gate_residual_ln_modulate_launch(float* x, const float* gate, long long gate_stride,
                                     const void* y, int y_dtype, const float* scale,
                                     const float* shift, long long mod_stride, void* h,
                                     int out_dtype, long long rows, int rows_per_b, int D,
                                     float eps, int sm_count, cudaStream_t st);
int gelu16_launch(const void* x, void* y, int dtype, long long n, int sm_count, cudaStream_t st);
int attn_fwd_launch_noalloc(const AnimaAttnArgs* a, int* status, int sm_count, void* scratch,
                            cudaStream_t st, const char** why);
cudaError_t noalloc_scratch_address(void** ptr);
int prologue_launch(const AnimaPrologueArgs* a, int sm_count, cudaStream_t st);
int rmsnorm_launch(const float* x, const float* w, float* y, long long m, int d, float eps,
                   int sm_count, cudaStream_t st);
int rope_launch(const float* t, const float* f, float* out, int N, int S, int D, int sm_count,
                cudaStream_t st);
int rope_strided_launch(const float* t, const long long* ts, const float* f, float* out,
                        const long long* os, int O, int S, int Hn, int D, int sm_count,
                        cudaStream_t st);
int act_launch(int which, const float* x, float* y, long long n, int sm_count, cudaStream_t st);
int qkv_projection_launch(const AnimaQkvProjArgs* a, int* status, int sm_count, cudaStream_t st);
int gemm_gelu_launch(const void* x, const void* w, void* y, int M, int N, int K, int dtype,
                     int* status, int sm_count, cudaStream_t st);
int layernorm_launch(const float* x, float* y, long long m, int d, float eps, int sm_count,
                     cudaStream_t st);
int softmax_launch(const float* x, float* y, long long outer, int dim, int sm_count,
                   cudaStream_t st);
int gemm_nt_launch(const float* A, const void* Bm, bool b_bf16, float* C, int M, int N, int K,
                   cudaStream_t st);
}  // namespace anima

using namespace anima;

namespace {

thread_local std::string g_last_error;

void set_error(const std::string& s) { g_last_error = s; }

constexpr int kMaxDevices = 64;

// The status word: first error a kernel recorded on this device (0 = clean).  It is a
// static device variable, so no entry of the library allocates device memory for it;
// each device that loads the library has its own copy, zero at load.
__device__ int g_status_word;

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  int cc = 0;
  int* status = nullptr;          // device address of g_status_word on this device
  void* noalloc_scratch = nullptr;  // device address of the no-allocation scratch array
};
DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

// Per-device bookkeeping for the current device; nullptr (with error set) on failure.
DeviceState* current_device(int* rc) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    *rc = ANIMA_ERR_CUDA;
    set_error("no usable CUDA device");
    return nullptr;
  }
  DeviceState& d = g_dev[dev];
  if (d.ready) return &d;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!d.ready) {
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      *rc = ANIMA_ERR_CUDA;
      set_error("cudaDeviceGetAttribute failed");
      return nullptr;
    }
    if (major != 10) {
      *rc = ANIMA_ERR_UNSUPPORTED;
      set_error("anima_attn kernels are built for sm_100a (B200); device is sm_" +
                std::to_string(major * 10 + minor));
      return nullptr;
    }
    // The symbol's address on this device (the device is current); a host-side
    // `&g_status_word` would be a host stand-in, not a device address.
    int* st = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&st), g_status_word) != cudaSuccess || !st) {
      cudaGetLastError();
      *rc = ANIMA_ERR_CUDA;
      set_error("cudaGetSymbolAddress of the device status word failed");
      return nullptr;
    }
    d.sm_count = sms;
    d.cc = major * 10 + minor;
    d.status = st;
    d.ready = true;
  }
  return &d;
}

// Device address of the no-allocation scratch on the current device (looked up once per
// device, under the same lock as the rest of the device state); nullptr on failure.
void* noalloc_scratch(DeviceState* d) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!d->noalloc_scratch) {
    void* ptr = nullptr;
    if (noalloc_scratch_address(&ptr) != cudaSuccess || !ptr) {
      cudaGetLastError();
      return nullptr;
    }
    d->noalloc_scratch = ptr;
  }
  return d->noalloc_scratch;
}

const char* code_name(int rc) {
  switch (rc) {
    case ANIMA_OK: return "ok";
    case ANIMA_ERR_ARG: return "bad argument";
    case ANIMA_ERR_SHAPE: return "unsupported shape";
    case ANIMA_ERR_CUDA: return "CUDA error";
    case ANIMA_ERR_TIMEOUT: return "device-side wait timed out";
    case ANIMA_ERR_UNSUPPORTED: return "unsupported device";
    case ANIMA_ERR_NOMEM: return "out of device memory";
  }
  return "unknown error";
}

// ---------------------------------------------------------------- anima_rt state
constexpr int kRtMaxChunks = 64;
// Page-locked staging of pageable caller arrays (see "host staging" below): slots of
// kStageSlot bytes, kStageIn of them for host->device pieces, kStageOut for device->host.
// Measured at B=2, H=16, L=4096 (16 host threads, pageable fp32 arrays in and out):
// 4 MiB x (6 + 4) slots 5.2-5.3 ms per anima_rt_run_attention call; 2 MiB x (6 + 4) 6.8,
// 2 MiB x (12 + 6) 5.7, 4 MiB x (12 + 6) 6.2, 8 MiB x (6 + 4) 6.3, 1 MiB x (16 + 8) 6.6;
// the driver's own pageable copies 24.2.
#ifndef ANIMA_STAGE_SLOT_MB
#define ANIMA_STAGE_SLOT_MB 4
#endif
constexpr size_t kStageSlot = size_t(ANIMA_STAGE_SLOT_MB) << 20;
#ifndef ANIMA_STAGE_IN
#define ANIMA_STAGE_IN 6
#define ANIMA_STAGE_OUT 4
#endif
constexpr int kStageIn = ANIMA_STAGE_IN, kStageOut = ANIMA_STAGE_OUT;
constexpr int kStageSlots = kStageIn + kStageOut;
struct RtState {
  bool inited = false;
  cudaStream_t stream = nullptr;          // kernels
  cudaStream_t in = nullptr, out = nullptr;  // host->device and device->host copies
  cudaEvent_t ev_in[kRtMaxChunks] = {}, ev_done[kRtMaxChunks] = {};
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int device = -1;
  char* ring = nullptr;                      // kStageSlots * kStageSlot page-locked bytes
  cudaEvent_t ev_slot[kStageSlots] = {};     // last copy that used each slot
  unsigned next_in = 0, next_out = 0;        // round-robin slot counters
};
RtState g_rt;
std::recursive_mutex g_rt_mu;

bool rt_fail(const std::string& what) {
  set_error(what);
  return false;
}

// Make sure the stream exists on the current device and the workspace holds `bytes`.
bool rt_prepare(size_t bytes) {
  int rc = ANIMA_OK;
  if (!current_device(&rc)) return false;
  int dev = -1;
  cudaGetDevice(&dev);
  if (g_rt.device != dev) {  // first use, or the caller switched devices
    if (g_rt.ws) cudaFree(g_rt.ws);
    for (cudaStream_t* s : {&g_rt.stream, &g_rt.in, &g_rt.out}) {
      if (*s) cudaStreamDestroy(*s);
      *s = nullptr;
    }
    for (int c = 0; c < kRtMaxChunks; ++c) {
      if (g_rt.ev_in[c]) cudaEventDestroy(g_rt.ev_in[c]);
      if (g_rt.ev_done[c]) cudaEventDestroy(g_rt.ev_done[c]);
      g_rt.ev_in[c] = g_rt.ev_done[c] = nullptr;
    }
    for (cudaEvent_t& e : g_rt.ev_slot) {
      if (e) cudaEventDestroy(e);
      e = nullptr;
    }
    g_rt.ws = nullptr;
    g_rt.ws_bytes = 0;
    g_rt.device = -1;
    for (cudaStream_t* s : {&g_rt.stream, &g_rt.in, &g_rt.out})
      if (cudaStreamCreateWithFlags(s, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        return rt_fail("cudaStreamCreate failed");
      }
    for (int c = 0; c < kRtMaxChunks; ++c)
      if (cudaEventCreateWithFlags(&g_rt.ev_in[c], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&g_rt.ev_done[c], cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        return rt_fail("cudaEventCreate failed");
      }
    for (cudaEvent_t& e : g_rt.ev_slot)
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        return rt_fail("cudaEventCreate failed");
      }
    g_rt.device = dev;
  }
  if (bytes > g_rt.ws_bytes) {
    if (g_rt.ws) cudaFree(g_rt.ws);
    g_rt.ws = nullptr;
    g_rt.ws_bytes = 0;
    if (cudaMalloc(&g_rt.ws, bytes) != cudaSuccess) {
      cudaGetLastError();
      return rt_fail("cudaMalloc of " + std::to_string(bytes) + " bytes failed");
    }
    g_rt.ws_bytes = bytes;
  }
  return true;
}

size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

bool rt_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return true;
  cudaGetLastError();
  return rt_fail(std::string(what) + ": " + cudaGetErrorString(e));
}

bool rt_finish(const char* what) {
  if (!rt_check(cudaStreamSynchronize(g_rt.stream), what)) return false;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  int code = 0;
  if (!rt_check(cudaMemcpy(&code, d->status, sizeof(int), cudaMemcpyDeviceToHost), what))
    return false;
  if (code != 0) {
    cudaMemset(d->status, 0, sizeof(int));
    return rt_fail(std::string(what) + ": " + code_name(code));
  }
  return true;
}

// ---------------------------------------------------------------- host staging
// The reference's callers pass ordinary (pageable) numpy arrays.  The CUDA driver copies
// pageable memory through its own bounce buffer on the calling thread, about 10 GB/s
// here, and a device->host copy into pageable memory does not return before the copy is
// done, which stalls the chunk pipeline.  Large pageable arrays are therefore copied
// through the library's page-locked ring instead: host threads gather a piece of rows
// into a slot while the copy engine moves the previous slots, and device->host pieces
// land in slots that the threads scatter into the caller's array.  Page-locked (and
// device) pointers keep the direct copies.  ANIMA_RT_STAGE=0 turns the staging off.

// Persistent host threads for the gathers and scatters.  run(fn) calls fn(t, T) for
// t = 0..T-1 on T threads, the caller being thread 0, and returns when all are done.
// Between jobs a worker spins for up to kSpinUs before it sleeps on the condition
// variable: the pieces of one call follow each other within microseconds, and a sleeping
// thread takes tens of microseconds to wake.
class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool* pool = new CopyPool();  // never destroyed: idle workers end with the process
    return *pool;
  }
  void run(const std::function<void(int, int)>& fn) {
    if (nworkers_ == 0 || getpid() != pid_) {  // a forked child has no workers
      fn(0, 1);
      return;
    }
    job_.store(&fn, std::memory_order_relaxed);
    pending_.store(nworkers_, std::memory_order_relaxed);
    {
      std::lock_guard<std::mutex> lk(mu_);  // a worker about to sleep sees the new generation
      gen_.fetch_add(1, std::memory_order_release);
    }
    cv_.notify_all();
    fn(0, nworkers_ + 1);
    while (pending_.load(std::memory_order_acquire) != 0) std::this_thread::yield();
  }

 private:
  static constexpr int kSpinUs = 2000;
  CopyPool() {
    int n = 1;
    cpu_set_t set;
    if (sched_getaffinity(0, sizeof(set), &set) == 0) n = CPU_COUNT(&set);
    // One process per GPU (torchrun sets LOCAL_WORLD_SIZE): the processes of this host
    // share its cores, so each takes its share.
    if (const char* w = std::getenv("LOCAL_WORLD_SIZE")) n /= std::max(1, std::atoi(w));
    if (const char* e = std::getenv("ANIMA_RT_COPY_THREADS")) n = std::atoi(e);
    n = std::max(1, std::min(n, 16));
    nworkers_ = n - 1;
    pid_ = getpid();
    for (int i = 0; i < nworkers_; ++i) std::thread([this, i] { work(i + 1); }).detach();
  }
  void work(int id) {
    unsigned long seen = 0;
    for (;;) {
      unsigned long g;
      const auto t0 = std::chrono::steady_clock::now();
      while ((g = gen_.load(std::memory_order_acquire)) == seen) {
        if (std::chrono::steady_clock::now() - t0 > std::chrono::microseconds(kSpinUs)) {
          std::unique_lock<std::mutex> lk(mu_);
          cv_.wait(lk, [&] { return gen_.load(std::memory_order_acquire) != seen; });
        }
      }
      seen = g;
      (*job_.load(std::memory_order_relaxed))(id, nworkers_ + 1);
      pending_.fetch_sub(1, std::memory_order_acq_rel);
    }
  }
  std::mutex mu_;
  std::condition_variable cv_;
  std::atomic<const std::function<void(int, int)>*> job_{nullptr};
  std::atomic<unsigned long> gen_{0};
  std::atomic<int> pending_{0};
  int nworkers_ = 0;
  pid_t pid_ = 0;
};

bool staging_enabled() {
  const char* e = std::getenv("ANIMA_RT_STAGE");
  return !(e && e[0] == '0');
}

// True for memory the copy engine reads without the driver's bounce buffer: page-locked
// host memory (cudaHostAlloc, cudaHostRegister, torch's pin_memory) and device memory.
bool direct_copyable(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type != cudaMemoryTypeUnregistered;
}

// Copies below this size go straight to the driver; the ring pays off above it.
constexpr size_t kStageMin = size_t(1) << 20;
static_assert(kStageSlot >= kStageMin, "a staged copy fills at least one row per slot");

// The ring, allocated on first use.  If the host cannot page-lock it, the copies go to the
// driver instead (slower, same result) and the allocation is not retried.
bool stage_ring() {
  static bool failed = false;
  if (g_rt.ring) return true;
  if (failed) return false;
  void* p = nullptr;
  if (cudaHostAlloc(&p, kStageSlots * kStageSlot, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    failed = true;
    return false;
  }
  g_rt.ring = static_cast<char*>(p);
  return true;
}

// rows x width bytes with pitches: rows [r0, r0+n) of src to the packed buffer dst, or
// the packed buffer src to rows of dst, split over the copy threads.
void copy_rows(char* dst, size_t dpitch, const char* src, size_t spitch, size_t width, size_t n) {
  CopyPool::get().run([&](int t, int T) {
    if (dpitch == width && spitch == width) {  // contiguous: split by bytes
      const size_t total = width * n, lo = total * t / T, hi = total * (t + 1) / T;
      if (hi > lo) std::memcpy(dst + lo, src + lo, hi - lo);
      return;
    }
    const size_t lo = n * t / T, hi = n * (t + 1) / T;
    for (size_t r = lo; r < hi; ++r) std::memcpy(dst + r * dpitch, src + r * spitch, width);
  });
}

// Host -> device copy of `rows` rows of `width` bytes (pitches in bytes) on stream s.
// Asynchronous for the caller's array as soon as it returns: every row has been read.
bool h2d_rows(char* dst, size_t dpitch, const char* src, size_t spitch, size_t width,
              size_t rows, cudaStream_t s, bool direct, const char* who) {
  if (!rows || !width) return true;
  if (direct || !staging_enabled() || width * rows < kStageMin || width > kStageSlot ||
      !stage_ring())
    return rt_check(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows,
                                      cudaMemcpyHostToDevice, s), who);
  const size_t per = kStageSlot / width;
  for (size_t r0 = 0; r0 < rows; r0 += per) {
    const size_t n = std::min(per, rows - r0);
    const int slot = (int)(g_rt.next_in++ % kStageIn);
    char* buf = g_rt.ring + slot * kStageSlot;
    // the slot's previous host->device copy has read it
    if (!rt_check(cudaEventSynchronize(g_rt.ev_slot[slot]), who)) return false;
    copy_rows(buf, width, src + r0 * spitch, spitch, width, n);
    if (!rt_check(cudaMemcpy2DAsync(dst + r0 * dpitch, dpitch, buf, width, width, n,
                                    cudaMemcpyHostToDevice, s), who) ||
        !rt_check(cudaEventRecord(g_rt.ev_slot[slot], s), who))
      return false;
  }
  return true;
}

// Device -> host copy of rows on stream s (after whatever s already waits for).  A direct
// copy is only enqueued; a staged one has landed in `dst` when this returns.
bool d2h_rows(char* dst, size_t dpitch, const char* src, size_t spitch, size_t width,
              size_t rows, cudaStream_t s, bool direct, const char* who) {
  if (!rows || !width) return true;
  if (direct || !staging_enabled() || width * rows < kStageMin || width > kStageSlot ||
      !stage_ring())
    return rt_check(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows,
                                      cudaMemcpyDeviceToHost, s), who);
  const size_t per = kStageSlot / width;
  struct Piece { int slot; size_t r0, n; };
  Piece q[kStageOut];
  int head = 0, count = 0;
  auto scatter_oldest = [&]() {
    const Piece& p = q[head];
    if (!rt_check(cudaEventSynchronize(g_rt.ev_slot[kStageIn + p.slot]), who)) return false;
    copy_rows(dst + p.r0 * dpitch, dpitch, g_rt.ring + (kStageIn + p.slot) * kStageSlot,
              width, width, p.n);
    head = (head + 1) % kStageOut;
    --count;
    return true;
  };
  // Up to kStageOut - 1 pieces in flight: the slot a new piece takes was scattered.
  for (size_t r0 = 0; r0 < rows; r0 += per) {
    if (count == kStageOut - 1 && !scatter_oldest()) return false;
    const size_t n = std::min(per, rows - r0);
    const int slot = (int)(g_rt.next_out++ % kStageOut);
    if (!rt_check(cudaMemcpy2DAsync(g_rt.ring + (kStageIn + slot) * kStageSlot, width,
                                    src + r0 * spitch, spitch, width, n,
                                    cudaMemcpyDeviceToHost, s), who) ||
        !rt_check(cudaEventRecord(g_rt.ev_slot[kStageIn + slot], s), who))
      return false;
    q[(head + count) % kStageOut] = Piece{slot, r0, n};
    ++count;
  }
  while (count > 0)
    if (!scatter_oldest()) return false;
  return true;
}

// A contiguous buffer as rows of 256 KiB (and a direct tail).
constexpr size_t kStageRow = size_t(256) << 10;
bool h2d_bytes(void* dst, const void* src, size_t n, cudaStream_t s, const char* who) {
  const bool direct = n < kStageMin || direct_copyable(src);
  const size_t rows = direct ? 0 : n / kStageRow, body = rows * kStageRow;
  if (!h2d_rows(static_cast<char*>(dst), kStageRow, static_cast<const char*>(src), kStageRow,
                kStageRow, rows, s, false, who))
    return false;
  return n == body || rt_check(cudaMemcpyAsync(static_cast<char*>(dst) + body,
                                               static_cast<const char*>(src) + body, n - body,
                                               cudaMemcpyHostToDevice, s), who);
}
bool d2h_bytes(void* dst, const void* src, size_t n, cudaStream_t s, const char* who) {
  const bool direct = n < kStageMin || direct_copyable(dst);
  const size_t rows = direct ? 0 : n / kStageRow, body = rows * kStageRow;
  if (!d2h_rows(static_cast<char*>(dst), kStageRow, static_cast<const char*>(src), kStageRow,
                kStageRow, rows, s, false, who))
    return false;
  return n == body || rt_check(cudaMemcpyAsync(static_cast<char*>(dst) + body,
                                               static_cast<const char*>(src) + body, n - body,
                                               cudaMemcpyDeviceToHost, s), who);
}

// One host buffer of a compatibility call (nullptr host: an absent optional input).
struct RtBuf {
  const void* host;
  size_t bytes;
};

// Body of the single-kernel host entries: copies each input into the library workspace,
// runs `launch(device inputs, device output, sm_count, stream)` and copies `out_bytes` of
// its output back to `out`, all on the library stream, then checks the status word.  On a
// failure after the first enqueue the stream is drained before false is returned, so no
// copy still touches the caller's arrays.
template <class F>
bool rt_call(const char* who, std::initializer_list<RtBuf> ins, void* out, size_t out_bytes,
             F launch) {
  constexpr int kMaxIns = 4;
  if (ins.size() > (size_t)kMaxIns) return rt_fail(std::string(who) + ": too many inputs");
  std::lock_guard<std::recursive_mutex> lk(g_rt_mu);
  size_t offs[kMaxIns] = {}, off = 0;
  int n = 0;
  for (const RtBuf& b : ins) {
    offs[n++] = off;
    off = align_up(off + b.bytes);
  }
  const size_t o_out = off;
  if (!rt_prepare(align_up(o_out + out_bytes))) return false;
  char* ws = static_cast<char*>(g_rt.ws);
  cudaStream_t st = g_rt.stream;
  auto bail = [&]() {
    cudaStreamSynchronize(st);
    cudaGetLastError();
    return false;
  };
  const void* dev_in[kMaxIns] = {};
  n = 0;
  for (const RtBuf& b : ins) {
    if (b.host) {
      dev_in[n] = ws + offs[n];
      if (b.bytes && !h2d_bytes(ws + offs[n], b.host, b.bytes, st, who)) return bail();
    }
    ++n;
  }
  int rc = ANIMA_OK;
  DeviceState* dev = current_device(&rc);
  if (!dev) return bail();
  rc = launch(dev_in, ws + o_out, dev->sm_count, st);
  if (rc != ANIMA_OK) {
    rt_fail(std::string(who) + ": " + code_name(rc));
    return bail();
  }
  if (!d2h_bytes(out, ws + o_out, out_bytes, st, who)) return bail();
  return rt_finish(who);
}

// Shared body of anima_rt_run_sdpa_flash / anima_rt_run_sdpa / anima_rt_run_attention.
bool rt_attention(const float* q, const float* k, const float* v, const float* q_w,
                  const float* k_w, const float* freqs, const int* kv_valid, float* out,
                  int B, int S_q, int S_kv, int H, int D, float eps, float scale,
                  unsigned flags, const char* who) {
  if (!q || !k || !v || !out) return rt_fail(std::string(who) + ": null pointer");
  if (D != 128)
    return rt_fail(std::string(who) + ": head size " + std::to_string(D) +
                   " unsupported (the B200 kernels take D = 128)");
  if (B <= 0 || H <= 0 || S_q <= 0 || S_kv <= 0)
    return rt_fail(std::string(who) + ": empty or negative shape");
  if ((flags & ANIMA_FLAG_ROPE) && (!freqs || S_q != S_kv))
    return rt_fail(std::string(who) + ": RoPE needs freqs and S_q == S_kv");
  std::lock_guard<std::recursive_mutex> lk(g_rt_mu);
  // Chunks of Bc batch rows x G heads, pipelined over three streams: host->device copies
  // of chunk c+1 run while chunk c's prologue and attention run and chunk c-1's output
  // goes back, so a call costs about its H2D time.  The caller's [B, S, H, D] arrays are
  // copied with 2D copies (rows of G*D floats, pitch H*D), straight into the same layout
  // on the device; each chunk then runs the prologue and attention on its own heads.
  // Two head groups measured best at B=2, H=16, L=4096 (4.40 ms; 4.51 with four groups,
  // 4.66 with one, 5.30 unpipelined): the copies then run at about 50 GB/s each way.
  constexpr int kGroups = 2;
  const int G = (H % kGroups == 0) ? H / kGroups : H;       // heads per chunk
  int Bc = (B * (H / G) <= 8) ? 1 : (B * (H / G) + 7) / 8;  // batch rows per chunk
  while ((B + Bc - 1) / Bc * (H / G) > kRtMaxChunks - 2) ++Bc;
  const int nb = (B + Bc - 1) / Bc, ng = H / G;
  // Pageable arrays go through the staging ring (h2d_rows / d2h_rows).  A staged output
  // chunk is collected one chunk late, after the next chunk's inputs are on their way,
  // so the scatter into `out` overlaps the copy engine's host->device work.
  const bool q_direct = direct_copyable(q), k_direct = direct_copyable(k),
             v_direct = direct_copyable(v), out_direct = direct_copyable(out);
  const bool out_staged = !out_direct && staging_enabled() &&
                          (size_t)G * D * 4 <= kStageSlot && stage_ring();
  // Chunks of bn batch rows from b0 x g heads from h0.  The last chunk's kernels and its
  // device->host copy run after every input has arrived, so with a page-locked `out` it is
  // made small: the last uniform chunk is split into g/2, g/4 and g/4 heads (B=2, H=16,
  // L=4096: the tail falls from 8 heads' 16.8 MB copy back to 2 heads'; 4.50-4.55 -> 4.37-4.45 ms
  // per call, same box, interleaved).  A staged output keeps uniform chunks: there the host threads' scatter is the
  // bound, and the extra chunk boundaries measured slower (5.18 -> 5.4-5.7 ms).
  struct Chunk { int b0, bn, h0, g; };
  std::vector<Chunk> chunks;
  for (int c = 0; c < nb * ng; ++c) {
    const int b0 = (c / ng) * Bc;
    chunks.push_back({b0, min(Bc, B - b0), (c % ng) * G, G});
  }
  if (G % 4 == 0 && out_direct) {
    const Chunk t = chunks.back();
    chunks.back().g = G / 2;
    chunks.push_back({t.b0, t.bn, t.h0 + G / 2, G / 4});
    chunks.push_back({t.b0, t.bn, t.h0 + 3 * G / 4, G / 4});
  }
  const int nchunks = (int)chunks.size();
  const size_t nq = (size_t)B * S_q * H * D, nk = (size_t)B * S_kv * H * D;
  size_t off = 0;
  auto carve = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes); return o; };
  const size_t o_q = carve(nq * 4), o_k = carve(nk * 4), o_v = carve(nk * 4);
  // 16-bit operands: one head-major block of Bc*G heads per chunk (the last may be short)
  const size_t cq = (size_t)Bc * G * S_q * D, ck = (size_t)Bc * G * S_kv * D;
  const size_t o_qb = carve(nchunks * cq * 2), o_kb = carve(nchunks * ck * 2),
               o_vb = carve(nchunks * ck * 2);
  const size_t o_out = carve(nq * 4);
  const size_t o_w = carve(2 * D * 4);
  const size_t o_f = carve(freqs ? (size_t)S_q * D * 2 * 4 : 0);
  const size_t o_valid = carve(kv_valid ? (size_t)B * 4 : 0);
  const unsigned aflags = (flags & ANIMA_FLAG_CAUSAL) | (kv_valid ? ANIMA_FLAG_MASK : 0u);
  int drc = ANIMA_OK;
  DeviceState* dev = current_device(&drc);
  if (!dev) return false;
  size_t ws_split = 0;  // the largest any chunk's schedule needs; the chunks run in turn
  for (const Chunk& ch : chunks)
    ws_split = std::max(ws_split, attn_workspace_bytes(ch.bn, ch.g, S_q, S_kv, aflags,
                                                       dev->sm_count));
  const size_t o_split = carve(ws_split);
  if (!rt_prepare(off)) return false;
  char* ws = static_cast<char*>(g_rt.ws);
  cudaStream_t st = g_rt.stream, sin = g_rt.in, sout = g_rt.out;
  // On a failure after the first enqueue, copies of earlier chunks may still read q/k/v
  // or write `out`: every stream finishes before the caller sees false and reuses them.
  auto bail = [&]() {
    cudaStreamSynchronize(sin);
    cudaStreamSynchronize(st);
    cudaStreamSynchronize(sout);
    cudaGetLastError();
    return false;
  };
  // The split schedule's arrival counters (first 4 KiB of its workspace) must start at
  // zero; this workspace is shared with other data, so clear them on every call.
  if (ws_split && !rt_check(cudaMemsetAsync(ws + o_split, 0, 4096, st), who)) return bail();
  float *dq = (float*)(ws + o_q), *dk = (float*)(ws + o_k), *dv = (float*)(ws + o_v);
  float* dout = (float*)(ws + o_out);
  float* dw = (float*)(ws + o_w);
  if (q_w && !rt_check(cudaMemcpyAsync(dw, q_w, D * 4, cudaMemcpyHostToDevice, sin), who))
    return bail();
  if (k_w && !rt_check(cudaMemcpyAsync(dw + D, k_w, D * 4, cudaMemcpyHostToDevice, sin), who))
    return bail();
  if (freqs && !h2d_bytes(ws + o_f, freqs, (size_t)S_q * D * 2 * 4, sin, who)) return bail();
  if (kv_valid && !rt_check(cudaMemcpyAsync(ws + o_valid, kv_valid, (size_t)B * 4,
                                            cudaMemcpyHostToDevice, sin), who))
    return bail();
  const size_t row = (size_t)H * D * 4;  // bytes: pitch of a token row
  auto chunk_geom = [&](int c, int& bn, size_t& qo, size_t& ko, size_t& crow) {
    const Chunk& ch = chunks[c];
    bn = ch.bn;
    qo = ((size_t)ch.b0 * S_q * H + ch.h0) * D;
    ko = ((size_t)ch.b0 * S_kv * H + ch.h0) * D;
    crow = (size_t)ch.g * D * 4;  // bytes of one token row of the chunk's heads
  };
  auto copy_out = [&](int c) {  // after chunk c's kernels
    int bn;
    size_t qo, ko, crow;
    chunk_geom(c, bn, qo, ko, crow);
    if (!rt_check(cudaStreamWaitEvent(sout, g_rt.ev_done[c], 0), who)) return false;
    return d2h_rows(reinterpret_cast<char*>(out + qo), row,
                    reinterpret_cast<const char*>(dout + qo), row, crow, (size_t)bn * S_q, sout,
                    out_direct, who);
  };
  for (int c = 0; c < nchunks; ++c) {
    const int b0 = chunks[c].b0, g = chunks[c].g;
    int bn;
    size_t qo, ko, crow;
    chunk_geom(c, bn, qo, ko, crow);
    // ---- copy in
    auto in = [&](float* d, const float* h, size_t off, int S, bool direct) {
      return h2d_rows(reinterpret_cast<char*>(d + off), row,
                      reinterpret_cast<const char*>(h + off), row, crow, (size_t)bn * S, sin,
                      direct, who);
    };
    if (!in(dq, q, qo, S_q, q_direct) || !in(dk, k, ko, S_kv, k_direct) ||
        !in(dv, v, ko, S_kv, v_direct) ||
        !rt_check(cudaEventRecord(g_rt.ev_in[c], sin), who) ||
        !rt_check(cudaStreamWaitEvent(st, g_rt.ev_in[c], 0), who))
      return bail();
    // ---- prologue + attention on this chunk's heads (its own head-major operand block)
    uint16_t* qb = (uint16_t*)(ws + o_qb) + c * cq;
    uint16_t* kb = (uint16_t*)(ws + o_kb) + c * ck;
    uint16_t* vb = (uint16_t*)(ws + o_vb) + c * ck;
    AnimaPrologueArgs pa = {};
    pa.q = dq + qo;
    pa.k = dk + ko;
    pa.v = dv + ko;
    pa.in_dtype = ANIMA_DTYPE_F32;
    const int64_t sq3[3] = {(int64_t)S_q * H * D, (int64_t)H * D, D};
    const int64_t sk3[3] = {(int64_t)S_kv * H * D, (int64_t)H * D, D};
    for (int i = 0; i < 3; ++i) {
      pa.q_stride[i] = sq3[i];
      pa.k_stride[i] = sk3[i];
      pa.v_stride[i] = sk3[i];
    }
    pa.B = bn;
    pa.H = g;
    pa.S_q = S_q;
    pa.S_kv = S_kv;
    pa.D = D;
    pa.q_norm_w = q_w ? dw : nullptr;
    pa.k_norm_w = k_w ? dw + D : nullptr;
    pa.eps = eps;
    pa.rope_freqs = freqs ? (const float*)(ws + o_f) : nullptr;
    pa.flags = flags & (ANIMA_FLAG_QNORM | ANIMA_FLAG_KNORM | ANIMA_FLAG_ROPE);
    pa.q_out = qb;
    pa.k_out = kb;
    pa.v_out = vb;
    pa.op_dtype = ANIMA_DTYPE_BF16;
    int rc = anima_attn_prologue(&pa, st);
    if (rc != ANIMA_OK) {
      rt_fail(std::string(who) + ": prologue: " + code_name(rc));
      return bail();
    }
    AnimaAttnArgs aa = {};
    aa.q = qb;
    aa.k = kb;
    aa.v = vb;
    aa.op_dtype = ANIMA_DTYPE_BF16;
    aa.out = dout + qo;
    aa.out_dtype = ANIMA_DTYPE_F32;
    aa.out_stride[0] = (int64_t)S_q * H * D;  // [B, S_q, H, D]
    aa.out_stride[1] = D;
    aa.out_stride[2] = (int64_t)H * D;
    aa.B = bn;
    aa.H = g;
    aa.S_q = S_q;
    aa.S_kv = S_kv;
    aa.D = D;
    aa.scale = scale;
    aa.flags = aflags;
    aa.kv_valid_len = kv_valid ? (const int*)(ws + o_valid) + b0 : nullptr;
    aa.workspace = ws_split ? ws + o_split : nullptr;
    aa.workspace_bytes = ws_split;
    rc = anima_attn_fwd(&aa, st);
    if (rc != ANIMA_OK) {
      rt_fail(std::string(who) + ": attention: " + code_name(rc));
      return bail();
    }
    // ---- copy out (a staged chunk one chunk late)
    if (!rt_check(cudaEventRecord(g_rt.ev_done[c], st), who)) return bail();
    if (!out_staged) {
      if (!copy_out(c)) return bail();
    } else if (c > 0 && !copy_out(c - 1)) {
      return bail();
    }
  }
  if (out_staged && !copy_out(nchunks - 1)) return bail();
  if (!rt_check(cudaStreamSynchronize(sout), who)) return bail();
  return rt_finish(who);
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- device-pointer ABI
int anima_attn_prologue(const AnimaPrologueArgs* a, void* stream) {
  if (!a) return ANIMA_ERR_ARG;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  rc = prologue_launch(a, d->sm_count, static_cast<cudaStream_t>(stream));
  if (rc != ANIMA_OK) set_error(std::string("anima_attn_prologue: ") + code_name(rc));
  return rc;
}

int anima_attn_fwd(const AnimaAttnArgs* a, void* stream) {
  if (!a || !a->q || !a->k || !a->v || !a->out) return ANIMA_ERR_ARG;
  if ((a->flags & ANIMA_FLAG_MASK) && !a->kv_valid_len) return ANIMA_ERR_ARG;
  const int oe = a->out_dtype == ANIMA_DTYPE_F32 ? 4 : 8;  // elements per 16 bytes
  for (int i = 0; i < 3; ++i)
    if (a->out_stride[i] < 0 || a->out_stride[i] % oe) return ANIMA_ERR_ARG;
  const uintptr_t al = reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k) |
                       reinterpret_cast<uintptr_t>(a->v) | reinterpret_cast<uintptr_t>(a->out);
  if (al & 15u) return ANIMA_ERR_ARG;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  if (a->flags & ANIMA_FLAG_PAIR)
    rc = attn_fwd_pair_launch(a, d->status, static_cast<cudaStream_t>(stream));
  else
    rc = attn_fwd_launch(a, d->status, d->sm_count, static_cast<cudaStream_t>(stream));
  if (rc != ANIMA_OK) set_error(std::string("anima_attn_fwd: ") + code_name(rc));
  return rc;
}

int anima_attn_fwd_noalloc(const AnimaAttnArgs* a, void* stream) {
  if (!a || !a->q || !a->k || !a->v || !a->out) return ANIMA_ERR_ARG;
  if ((a->flags & ANIMA_FLAG_MASK) && !a->kv_valid_len) return ANIMA_ERR_ARG;
  const int oe = a->out_dtype == ANIMA_DTYPE_F32 ? 4 : 8;
  for (int i = 0; i < 3; ++i)
    if (a->out_stride[i] < 0 || a->out_stride[i] % oe) return ANIMA_ERR_ARG;
  const uintptr_t al = reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k) |
                       reinterpret_cast<uintptr_t>(a->v) | reinterpret_cast<uintptr_t>(a->out);
  if (al & 15u) return ANIMA_ERR_ARG;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  if (a->flags & ANIMA_FLAG_PAIR) {  // the CTA-pair kernel uses no scratch
    rc = attn_fwd_pair_launch(a, d->status, static_cast<cudaStream_t>(stream));
    if (rc != ANIMA_OK) set_error(std::string("anima_attn_fwd_noalloc: ") + code_name(rc));
    return rc;
  }
  void* scratch = noalloc_scratch(d);
  if (!scratch) {
    set_error("anima_attn_fwd_noalloc: cudaGetSymbolAddress of the no-allocation scratch failed");
    return ANIMA_ERR_CUDA;
  }
  const char* why = nullptr;
  rc = attn_fwd_launch_noalloc(a, d->status, d->sm_count, scratch,
                               static_cast<cudaStream_t>(stream), &why);
  if (rc != ANIMA_OK)
    set_error(std::string("anima_attn_fwd_noalloc: ") + (why ? why : code_name(rc)));
  return rc;
}

int anima_gemm_gelu(const void* x, const void* w, void* y, int M, int N, int K, int dtype,
                    void* stream) {
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  rc = gemm_gelu_launch(x, w, y, M, N, K, dtype, d->status, d->sm_count,
                        static_cast<cudaStream_t>(stream));
  if (rc != ANIMA_OK) set_error(std::string("anima_gemm_gelu: ") + code_name(rc));
  return rc;
}

int anima_qkv_projection_scatter(const AnimaQkvProjArgs* a, int rows, int row0,
                                 void* const* dest, int n_dest, void* stream) {
  if (!a) return ANIMA_ERR_ARG;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  rc = qkv_projection_scatter_launch(a, rows, row0, dest, n_dest, d->status, d->sm_count,
                                     static_cast<cudaStream_t>(stream));
  if (rc != ANIMA_OK) set_error(std::string("anima_qkv_projection_scatter: ") + code_name(rc));
  return rc;
}

int anima_attn_fwd_scatter_rows(const AnimaAttnArgs* a, void* const* dest, int n_dest,
                                int rows_per_dest, int64_t dest_row_stride, int head0,
                                void* stream) {
  if (!a || !dest || n_dest < 1 || n_dest > 8 || rows_per_dest <= 0 || head0 < 0)
    return ANIMA_ERR_ARG;
  if (a->flags & ANIMA_FLAG_PAIR) return ANIMA_ERR_ARG;
  if (a->S_q <= 0 || a->S_q % 32 != 0 || rows_per_dest % 32 != 0) return ANIMA_ERR_SHAPE;
  if ((long long)a->B * a->S_q > (long long)n_dest * rows_per_dest) return ANIMA_ERR_SHAPE;
  const int esz = a->out_dtype == ANIMA_DTYPE_F32 ? 4 : 2;
  if (dest_row_stride <= 0 || (dest_row_stride * esz) % 16 ||
      ((long long)head0 + a->H) * 128 > dest_row_stride)
    return ANIMA_ERR_ARG;
  for (int i = 0; i < n_dest; ++i)
    if (!dest[i] || (reinterpret_cast<uintptr_t>(dest[i]) & 15u)) return ANIMA_ERR_ARG;
  AnimaAttnArgs b = *a;
  b.out = dest[0];
  b.out_stride[0] = b.out_stride[1] = b.out_stride[2] = dest_row_stride;  // unused by the kernel
  if (!b.q || !b.k || !b.v) return ANIMA_ERR_ARG;
  if ((b.flags & ANIMA_FLAG_MASK) && !b.kv_valid_len) return ANIMA_ERR_ARG;
  const uintptr_t al = reinterpret_cast<uintptr_t>(b.q) | reinterpret_cast<uintptr_t>(b.k) |
                       reinterpret_cast<uintptr_t>(b.v);
  if (al & 15u) return ANIMA_ERR_ARG;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  rc = attn_fwd_launch(&b, d->status, d->sm_count, static_cast<cudaStream_t>(stream), dest,
                       n_dest, rows_per_dest, dest_row_stride, head0);
  if (rc != ANIMA_OK) set_error(std::string("anima_attn_fwd_scatter_rows: ") + code_name(rc));
  return rc;
}

int anima_attn_fwd_gather(const AnimaAttnArgs* a, void* const* peer_out, int n_peers,
                          void* stream) {
  if (!a || !peer_out || n_peers < 1 || n_peers > 8) return ANIMA_ERR_ARG;
  if (a->flags & ANIMA_FLAG_PAIR) return ANIMA_ERR_ARG;  // the CTA-pair kernel stores locally
  for (int i = 0; i < n_peers; ++i)
    if (!peer_out[i] || (reinterpret_cast<uintptr_t>(peer_out[i]) & 15u)) return ANIMA_ERR_ARG;
  AnimaAttnArgs b = *a;
  b.out = peer_out[0];  // strides and dtype of every destination; the launch stores to all
  if (!b.q || !b.k || !b.v) return ANIMA_ERR_ARG;
  if ((b.flags & ANIMA_FLAG_MASK) && !b.kv_valid_len) return ANIMA_ERR_ARG;
  const int oe = b.out_dtype == ANIMA_DTYPE_F32 ? 4 : 8;
  for (int i = 0; i < 3; ++i)
    if (b.out_stride[i] < 0 || b.out_stride[i] % oe) return ANIMA_ERR_ARG;
  const uintptr_t al = reinterpret_cast<uintptr_t>(b.q) | reinterpret_cast<uintptr_t>(b.k) |
                       reinterpret_cast<uintptr_t>(b.v);
  if (al & 15u) return ANIMA_ERR_ARG;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  rc = attn_fwd_launch(&b, d->status, d->sm_count, static_cast<cudaStream_t>(stream), peer_out,
                       n_peers, 0, 0, 0);
  if (rc != ANIMA_OK) set_error(std::string("anima_attn_fwd_gather: ") + code_name(rc));
  return rc;
}

// ---------------------------------------------------------------- peer buffers (CUDA IPC)
typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(ptr);
  }
  return fn;
}

int anima_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  if (!ptr || !handle || !offset) return ANIMA_ERR_ARG;
  AddressRangeFn range = address_range_fn();
  if (!range) {
    set_error("anima_ipc_export: cuMemGetAddressRange unavailable");
    return ANIMA_ERR_CUDA;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_error("anima_ipc_export: pointer is not device memory of this process");
    return ANIMA_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) {
    set_error(std::string("anima_ipc_export: ") + cudaGetErrorString(cudaGetLastError()));
    return ANIMA_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == ANIMA_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  return ANIMA_OK;
}

int anima_ipc_open(const void* handle, uint64_t offset, void** ptr) {
  if (!handle || !ptr) return ANIMA_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    set_error(std::string("anima_ipc_open: ") + cudaGetErrorString(cudaGetLastError()));
    return ANIMA_ERR_CUDA;
  }
  *ptr = static_cast<char*>(base) + offset;
  return ANIMA_OK;
}

int anima_ipc_close(void* ptr, uint64_t offset) {
  if (!ptr) return ANIMA_ERR_ARG;
  if (cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset) != cudaSuccess) {
    set_error(std::string("anima_ipc_close: ") + cudaGetErrorString(cudaGetLastError()));
    return ANIMA_ERR_CUDA;
  }
  return ANIMA_OK;
}

uint64_t anima_attn_workspace_size(int B, int H, int S_q, int S_kv, unsigned flags) {
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d || B <= 0 || H <= 0 || S_q <= 0 || S_kv <= 0) return 0;
  return attn_workspace_bytes(B, H, S_q, S_kv, flags, d->sm_count);
}

int anima_attn_schedule(int B, int H, int S_q, int S_kv, unsigned flags, int sm_count) {
  if (B <= 0 || H <= 0 || S_q <= 0 || S_kv <= 0 || (long long)B * H > 0x7fffffffLL)
    return ANIMA_ERR_SHAPE;
  if (sm_count <= 0) {
    int rc = ANIMA_OK;
    DeviceState* d = current_device(&rc);
    if (!d) return rc;
    sm_count = d->sm_count;
  }
  if (flags & ANIMA_FLAG_PAIR) return ANIMA_SCHED_UNIT;
  return attn_schedule_mode(B, H, S_q, S_kv, flags, sm_count);
}

int anima_attn_status(void* stream, int reset) {
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) {
    cudaGetLastError();
    return ANIMA_ERR_CUDA;
  }
  int code = 0;
  if (cudaMemcpy(&code, d->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return ANIMA_ERR_CUDA;
  }
  if (reset && code) cudaMemset(d->status, 0, sizeof(int));
  return code;
}

int anima_qkv_projection(const AnimaQkvProjArgs* a, void* stream) {
  if (!a) return ANIMA_ERR_ARG;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  rc = qkv_projection_launch(a, d->status, d->sm_count, static_cast<cudaStream_t>(stream));
  if (rc != ANIMA_OK) set_error(std::string("anima_qkv_projection: ") + code_name(rc));
  return rc;
}

int anima_attn_rope(const float* t, const int64_t t_stride[3], const float* freqs, float* out,
                    const int64_t out_stride[3], int O, int S, int Hn, int D, void* stream) {
  if (!t || !t_stride || !freqs || !out || !out_stride || O < 0 || S < 0 || Hn < 0 || D <= 0 ||
      (D & 1))
    return ANIMA_ERR_ARG;
  for (int i = 0; i < 3; ++i)
    if (t_stride[i] < 0 || out_stride[i] < 0) return ANIMA_ERR_ARG;
  if ((long long)O * S * Hn == 0) return ANIMA_OK;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  const long long ts[3] = {t_stride[0], t_stride[1], t_stride[2]};
  const long long os[3] = {out_stride[0], out_stride[1], out_stride[2]};
  return rope_strided_launch(t, ts, freqs, out, os, O, S, Hn, D, d->sm_count,
                             static_cast<cudaStream_t>(stream));
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int anima_dit_ln_modulate(const float* x, const float* scale, const float* shift,
                          int64_t mod_stride_b, void* y, int out_dtype, int64_t rows,
                          int rows_per_b, int D, float eps, void* stream) {
  if (!x || !scale || !shift || !y || rows < 0 || rows_per_b <= 0 || mod_stride_b % 4) return ANIMA_ERR_ARG;
  if (!al16(x) || !al16(scale) || !al16(shift) || !al16(y)) return ANIMA_ERR_ARG;
  if (rows == 0) return ANIMA_OK;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  return ln_modulate_launch(x, scale, shift, mod_stride_b, y, out_dtype, rows, rows_per_b, D, eps,
                            d->sm_count, static_cast<cudaStream_t>(stream));
}

int anima_dit_gate_residual(float* x, const float* gate, int64_t gate_stride_b, const float* y,
                            int64_t rows, int rows_per_b, int D, void* stream) {
  if (!x || !gate || !y || rows < 0 || rows_per_b <= 0 || gate_stride_b % 4) return ANIMA_ERR_ARG;
  if (!al16(x) || !al16(gate) || !al16(y)) return ANIMA_ERR_ARG;
  if (rows == 0) return ANIMA_OK;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  return gate_residual_launch(x, gate, gate_stride_b, y, rows, rows_per_b, D, d->sm_count,
                              static_cast<cudaStream_t>(stream));
}

int anima_dit_gate_residual_ln_modulate(float* x, const float* gate, int64_t gate_stride_b,
                                        const void* y, int y_dtype, const float* scale,
                                        const float* shift, int64_t mod_stride_b, void* h,
                                        int out_dtype, int64_t rows, int rows_per_b, int D,
                                        float eps, void* stream) {
  if (!x || !gate || !y || !scale || !shift || !h || rows < 0 || rows_per_b <= 0 ||
      gate_stride_b % 4 || mod_stride_b % 4)
    return ANIMA_ERR_ARG;
  if (!al16(x) || !al16(gate) || !al16(y) || !al16(scale) || !al16(shift) || !al16(h))
    return ANIMA_ERR_ARG;
  if (rows == 0) return ANIMA_OK;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  return gate_residual_ln_modulate_launch(x, gate, gate_stride_b, y, y_dtype, scale, shift,
                                          mod_stride_b, h, out_dtype, rows, rows_per_b, D, eps,
                                          d->sm_count, static_cast<cudaStream_t>(stream));
}

int anima_dit_gelu(const void* x, void* y, int dtype, int64_t n, void* stream) {
  if (!x || !y || n < 0 || !al16(x) || !al16(y)) return ANIMA_ERR_ARG;
  if (n == 0) return ANIMA_OK;
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  return gelu16_launch(x, y, dtype, n, d->sm_count, static_cast<cudaStream_t>(stream));
}

int anima_attn_selftest_timeout(unsigned timeout_us, void* stream) {
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  return selftest_wait_launch(d->status, timeout_us, static_cast<cudaStream_t>(stream));
}

int anima_attn_device_info(int* sm_count, int* cc) {
  int rc = ANIMA_OK;
  DeviceState* d = current_device(&rc);
  if (!d) return rc;
  if (sm_count) *sm_count = d->sm_count;
  if (cc) *cc = d->cc;
  return ANIMA_OK;
}

const char* anima_attn_version(void) {
  return "anima_attn sm_100a: tcgen05 flash fwd (2x128-row Q tiles per unit, 128-key tiles, "
         "4-slot K/V ring, TMEM S/P/O, persistent split schedule for the last round), fused "
         "RMSNorm+RoPE "
         "prologue";
}

// ---------------------------------------------------------------- anima_rt drop-ins
bool anima_rt_init(void) {
  std::lock_guard<std::recursive_mutex> lk(g_rt_mu);
  if (g_rt.inited) return true;
  if (!rt_prepare(0)) return false;
  g_rt.inited = true;
  return true;
}

void anima_rt_destroy(void) {
  std::lock_guard<std::recursive_mutex> lk(g_rt_mu);
  if (g_rt.ws) cudaFree(g_rt.ws);
  if (g_rt.stream) cudaStreamDestroy(g_rt.stream);
  g_rt = RtState();
}

bool anima_rt_run_sdpa_flash(const float* Q, const float* K, const float* V, float* output,
                             int BH, int S_q, int S_kv, int D, float scale, bool is_causal) {
  // [BH, S, D] is [B, S, H, D] with B = BH and H = 1.
  return rt_attention(Q, K, V, nullptr, nullptr, nullptr, nullptr, output, BH, S_q, S_kv, 1, D,
                      0.f, scale, is_causal ? ANIMA_FLAG_CAUSAL : 0u, "anima_rt_run_sdpa_flash");
}

bool anima_rt_run_sdpa(const float* Q, const float* K, const float* V, float* output, int BH,
                       int S_q, int S_kv, int D, float scale, bool is_causal) {
  if (!g_rt.inited) return rt_fail("anima_rt_run_sdpa: anima_rt_init has not been called");
  return rt_attention(Q, K, V, nullptr, nullptr, nullptr, nullptr, output, BH, S_q, S_kv, 1, D,
                      0.f, scale, is_causal ? ANIMA_FLAG_CAUSAL : 0u, "anima_rt_run_sdpa");
}

bool anima_rt_run_attention(const float* q, const float* k, const float* v, const float* q_w,
                            const float* k_w, const float* freqs, const int* kv_valid,
                            float* out, int B, int S_q, int S_kv, int H, int D, float eps,
                            float scale, unsigned flags) {
  return rt_attention(q, k, v, q_w, k_w, freqs, kv_valid, out, B, S_q, S_kv, H, D, eps, scale,
                      flags, "anima_rt_run_attention");
}

bool anima_rt_run_rmsnorm(const float* x, const float* w, float* out, int m, int d, float eps) {
  if (!g_rt.inited) return rt_fail("anima_rt_run_rmsnorm: anima_rt_init has not been called");
  if (!x || !out || m < 0 || d <= 0) return rt_fail("anima_rt_run_rmsnorm: bad arguments");
  if (m == 0) return true;
  const size_t n = (size_t)m * d;
  return rt_call("anima_rt_run_rmsnorm", {{x, n * 4}, {w, (size_t)d * 4}}, out, n * 4,
                 [&](const void* const* in, void* y, int sms, cudaStream_t st) {
                   return rmsnorm_launch((const float*)in[0], (const float*)in[1], (float*)y, m,
                                         d, eps, sms, st);
                 });
}

bool anima_rt_run_rope(const float* t, const float* freqs, float* out, int N, int S, int D) {
  if (!t || !freqs || !out || N < 0 || S < 0 || D <= 0 || (D & 1))
    return rt_fail("anima_rt_run_rope: bad arguments");
  if (N == 0 || S == 0) return true;
  const size_t n = (size_t)N * S * D, nf = (size_t)S * D * 2;
  return rt_call("anima_rt_run_rope", {{t, n * 4}, {freqs, nf * 4}}, out, n * 4,
                 [&](const void* const* in, void* y, int sms, cudaStream_t st) {
                   return rope_launch((const float*)in[0], (const float*)in[1], (float*)y, N, S,
                                      D, sms, st);
                 });
}

// The reference's activation, normalisation and softmax entries fail before
// anima_rt_init (anima_rt.cpp:24-57); its GEMM entries (gemm_backend.cpp:140-171) do not
// need it.  Same here.
static bool rt_act(int which, const float* x, float* out, int n, const char* who) {
  if (!g_rt.inited) return rt_fail(std::string(who) + ": anima_rt_init has not been called");
  if (!x || !out || n < 0) return rt_fail(std::string(who) + ": bad arguments");
  if (n == 0) return true;
  return rt_call(who, {{x, (size_t)n * 4}}, out, (size_t)n * 4,
                 [&](const void* const* in, void* y, int sms, cudaStream_t st) {
                   return act_launch(which, (const float*)in[0], (float*)y, n, sms, st);
                 });
}

bool anima_rt_run_gelu(const float* x, float* out, int n) {
  return rt_act(0, x, out, n, "anima_rt_run_gelu");
}

bool anima_rt_run_silu(const float* x, float* out, int n) {
  return rt_act(1, x, out, n, "anima_rt_run_silu");
}

bool anima_rt_run_layernorm(const float* x, float* out, int m, int d, float eps) {
  if (!g_rt.inited) return rt_fail("anima_rt_run_layernorm: anima_rt_init has not been called");
  if (!x || !out || m < 0 || d <= 0) return rt_fail("anima_rt_run_layernorm: bad arguments");
  if (m == 0) return true;
  const size_t n = (size_t)m * d;
  return rt_call("anima_rt_run_layernorm", {{x, n * 4}}, out, n * 4,
                 [&](const void* const* in, void* y, int sms, cudaStream_t st) {
                   return layernorm_launch((const float*)in[0], (float*)y, m, d, eps, sms, st);
                 });
}

bool anima_rt_run_softmax(const float* x, float* out, int outer, int dim) {
  if (!g_rt.inited) return rt_fail("anima_rt_run_softmax: anima_rt_init has not been called");
  if (!x || !out || outer < 0 || dim <= 0) return rt_fail("anima_rt_run_softmax: bad arguments");
  if (outer == 0) return true;
  const size_t n = (size_t)outer * dim;
  return rt_call("anima_rt_run_softmax", {{x, n * 4}}, out, n * 4,
                 [&](const void* const* in, void* y, int sms, cudaStream_t st) {
                   return softmax_launch((const float*)in[0], (float*)y, outer, dim, sms, st);
                 });
}

static bool rt_gemm(const float* A, const void* Bm, bool bf16, float* C, int M, int N, int K,
                    const char* who) {
  if (!A || !Bm || !C || M < 0 || N < 0 || K < 0) return rt_fail(std::string(who) + ": bad arguments");
  if (M == 0 || N == 0) return true;
  return rt_call(who, {{A, (size_t)M * K * 4}, {Bm, (size_t)N * K * (bf16 ? 2 : 4)}}, C,
                 (size_t)M * N * 4, [&](const void* const* in, void* y, int, cudaStream_t st) {
                   return gemm_nt_launch((const float*)in[0], in[1], bf16, (float*)y, M, N, K, st);
                 });
}

bool anima_rt_run_gemm_fp32(const float* A, const float* B, float* C, int M, int N, int K) {
  return rt_gemm(A, B, false, C, M, N, K, "anima_rt_run_gemm_fp32");
}

bool anima_rt_run_gemm_bf16(const float* A, const uint16_t* W, float* C, int M, int N, int K) {
  return rt_gemm(A, W, true, C, M, N, K, "anima_rt_run_gemm_bf16");
}

const char* anima_rt_last_error(void) { return g_last_error.c_str(); }

}  // extern "C"
