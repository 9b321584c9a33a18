// ctx.cu -- the wp_* C ABI of the reference's GEMM library (csrc/wtlgpu.h) on top of the
// tcgen05 GEMM of gemm.cuh.
//
// The ABI fixes the behaviour that the Rust shell (src/gpu.rs) relies on, and this file keeps
// it: null arguments -> -1, empty shapes -> 0 with nothing enqueued, weight ranges outside the
// blob -> -2; every op is enqueued on the context's call stream, which is the legacy default
// stream until the first capture and the context's own capturable stream from then on; capture
// is thread-local; whatever goes wrong while a capture is open, wp_capture_end leaves the stream
// out of capture mode and returns one of -13 / -14 / -15; replay and graph release report -17 /
// -18.  What is new: no cuBLASLt handle, algorithm search or disk cache (the GEMM handles any n
// with compile-time tiles), and a device error word that wp_sync reports as -21.
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <type_traits>

#include "../../include/wtlgpu.h"
#include "gemm.cuh"
#include "kern.cuh"

using namespace wasr;

namespace {

// A failed runtime call leaves a sticky last-error value behind, which a later
// cudaGetLastError() in the caller's own code would wrongly pick up.  Every failure path in
// this file consumes it before it returns its ABI code.
bool cuda_ok(cudaError_t e) {
  if (e == cudaSuccess) return true;
  cudaGetLastError();
  return false;
}

struct GraphRelease {
  void operator()(cudaGraph_t g) const { cudaGraphDestroy(g); }
};
using OwnedGraph = std::unique_ptr<std::remove_pointer_t<cudaGraph_t>, GraphRelease>;

bool is_capturing(cudaStream_t s) {
  if (s == nullptr) return false;  // the legacy stream is never put into capture mode here
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  return cuda_ok(cudaStreamIsCapturing(s, &st)) && st != cudaStreamCaptureStatusNone;
}

// Makes device `d` current for one call and restores the caller's device afterwards.
class DeviceScope {
 public:
  explicit DeviceScope(int d) {
    if (cudaGetDevice(&saved_) != cudaSuccess) {
      cudaGetLastError();
      saved_ = -1;
    }
    ok_ = saved_ == d || cuda_ok(cudaSetDevice(d));
  }
  ~DeviceScope() {
    int cur = -1;
    if (saved_ >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != saved_) cudaSetDevice(saved_);
  }
  bool ok() const { return ok_; }

 private:
  int saved_ = -1;
  bool ok_ = false;
};

// sized at create for t <= 512 rows of n <= 4096, so engine shapes never grow it in capture
constexpr size_t kScratchInit = 512ull * 4096 * 4;
constexpr size_t kRowmaxInit = 4096;

}  // namespace

struct WpCtx {
  int dev = 0;
  cudaStream_t call_stream = nullptr;  // nullptr: the legacy default stream
  cudaStream_t own_stream = nullptr;   // non-blocking, capturable; the call stream after a capture
  bool capturing = false;
  size_t last_graph_nodes = 0;
  uint8_t* w = nullptr;
  size_t w_bytes = 0;
  float* scratch = nullptr;  // fp32 [t][n] staging of wp_gemm_q / wp_gemm_qg
  size_t scratch_bytes = 0;
  unsigned* rowmax = nullptr;
  size_t rowmax_n = 0;
  int* err_host = nullptr;  // mapped pinned error word
  int* err_dev = nullptr;
  std::mutex mu;

  // Everything wp_create sets up; false leaves a partly built context for release().
  bool init(const void* w_host, size_t bytes) {
    if (!cuda_ok(cudaGetDevice(&dev))) return false;
    gemm_prepare();
    kern_prepare();
    if (!cuda_ok(cudaStreamCreateWithFlags(&own_stream, cudaStreamNonBlocking))) return false;
    if (!cuda_ok(cudaHostAlloc(reinterpret_cast<void**>(&err_host), sizeof(int), cudaHostAllocMapped)) ||
        !cuda_ok(cudaHostGetDevicePointer(reinterpret_cast<void**>(&err_dev), err_host, 0)))
      return false;
    *err_host = 0;
    if (!cuda_ok(cudaMalloc(&scratch, kScratchInit))) return false;
    scratch_bytes = kScratchInit;
    if (!cuda_ok(cudaMalloc(&rowmax, kRowmaxInit * sizeof(unsigned)))) return false;
    rowmax_n = kRowmaxInit;
    w_bytes = bytes;
    if (bytes == 0) return true;
    if (!cuda_ok(cudaMalloc(&w, bytes))) return false;
    return cuda_ok(w_host ? cudaMemcpy(w, w_host, bytes, cudaMemcpyHostToDevice) : cudaMemset(w, 0, bytes));
  }

  void release() {
    cudaDeviceSynchronize();
    for (void* p : {static_cast<void*>(w), static_cast<void*>(scratch), static_cast<void*>(rowmax)})
      if (p) cudaFree(p);
    if (err_host) cudaFreeHost(err_host);
    if (own_stream) cudaStreamDestroy(own_stream);
    cudaGetLastError();
  }

  // Capture needs a stream other than the legacy one.  The first capture drains the legacy
  // stream and moves the context to its own stream, which then stays the call stream (callers
  // re-query wp_stream, so their own kernels land in the same graphs).
  int open_capture() {
    if (capturing || own_stream == nullptr) return -10;
    if (call_stream == nullptr) {
      if (!cuda_ok(cudaStreamSynchronize(nullptr))) return -10;
      call_stream = own_stream;
    }
    if (!cuda_ok(cudaStreamBeginCapture(call_stream, cudaStreamCaptureModeThreadLocal))) return -10;
    capturing = true;
    return 0;
  }

  // Ends the open capture.  On every path the stream leaves capture mode; only a graph with at
  // least one node that instantiates becomes an exec.
  int close_capture(cudaGraphExec_t* exec) {
    if (!capturing) return -12;
    capturing = false;
    cudaGraph_t raw = nullptr;
    const bool ended = cuda_ok(cudaStreamEndCapture(call_stream, &raw));
    OwnedGraph graph(raw);
    if (!ended) {
      // an error inside the region invalidated the capture; make sure it is really closed
      while (is_capturing(call_stream)) {
        cudaGraph_t rest = nullptr;
        const bool closed = cuda_ok(cudaStreamEndCapture(call_stream, &rest));
        OwnedGraph drop(rest);
        if (!closed) break;
      }
      return -13;
    }
    if (!graph) return -14;
    size_t nodes = 0;
    if (!cuda_ok(cudaGraphGetNodes(graph.get(), nullptr, &nodes))) nodes = 0;
    last_graph_nodes = nodes;
    if (nodes == 0) return -14;  // nothing was enqueued: no use handing back an empty graph
    return cuda_ok(cudaGraphInstantiateWithFlags(exec, graph.get(), 0)) ? 0 : -15;
  }
};

extern "C" {

const char* wp_version(void) {
  return "wasr-b200 wtlgpu 2.0 (tcgen05 kind::i8 sm_100a, TMA + TMEM; wp_gemm/2/q/qg; cuda-graph)";
}

WpCtx* wp_create(const void* w_host, size_t bytes) {
  std::unique_ptr<WpCtx> c(new WpCtx());
  if (!c->init(w_host, bytes)) {
    c->release();
    return nullptr;
  }
  return c.release();
}

void wp_destroy(WpCtx* c) {
  if (c == nullptr) return;
  c->release();
  delete c;
}

void* wp_alloc(size_t bytes) {
  void* p = nullptr;
  if (bytes > 0 && !cuda_ok(cudaMalloc(&p, bytes))) p = nullptr;
  return p;
}

void wp_free(void* p) {
  if (p != nullptr) cuda_ok(cudaFree(p));
}

}  // extern "C"

// The synchronous copies of the ABI: -1 for a null pointer, -2 if the copy fails.
static int blocking_copy(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind) {
  if (dst == nullptr || src == nullptr) return -1;
  if (bytes == 0) return 0;
  return cuda_ok(cudaMemcpy(dst, src, bytes, kind)) ? 0 : -2;
}

extern "C" {

int wp_h2d(void* dev, const void* host, size_t bytes) {
  return blocking_copy(dev, host, bytes, cudaMemcpyHostToDevice);
}

int wp_d2h(void* host, const void* dev, size_t bytes) {
  return blocking_copy(host, dev, bytes, cudaMemcpyDeviceToHost);
}

void* wp_devptr(WpCtx* c, size_t off) {
  return (c != nullptr && off <= c->w_bytes) ? static_cast<void*>(c->w + off) : nullptr;
}

int wp_sync(WpCtx* c) {
  if (c == nullptr) return -1;
  if (!cuda_ok(cudaStreamSynchronize(c->call_stream))) return -2;
  // a kernel of this context gave up a bounded wait since the last sync
  volatile int* word = c->err_host;
  if (*word != 0) {
    *word = 0;
    return -21;
  }
  return 0;
}

int wp_set_stream(WpCtx* c, void* stream) {
  if (c == nullptr) return -1;
  if (c->capturing) return -16;
  c->call_stream = static_cast<cudaStream_t>(stream);
  return 0;
}

void* wp_stream(WpCtx* c) { return c == nullptr ? nullptr : static_cast<void*>(c->call_stream); }
size_t wp_scratch_bytes(WpCtx* c) { return c == nullptr ? 0 : c->scratch_bytes; }

}  // extern "C"

// One GEMM call of the wp_gemm family.  mode 0: fp32 out; 1: re-quant; 2: GELU + re-quant;
// 3: raw int32.  ws_vec (nullable) gives per-output-channel scales.
static int gemm_impl(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
                     const float* ws_vec, const float* bias, cudaStream_t stream, float* out, int8_t* out_q,
                     float* out_s, int32_t* out_i32, int mode) {
  if (!c || !xq || (mode != 3 && !xs)) return -1;
  if (mode == 3 ? !out_i32 : (out_q ? !out_s : !out)) return -1;
  if (t <= 0 || k <= 0 || n <= 0) return 0;
  if (static_cast<size_t>(n) * static_cast<size_t>(k) > c->w_bytes ||
      w_off > c->w_bytes - static_cast<size_t>(n) * static_cast<size_t>(k))
    return -2;
  std::lock_guard<std::mutex> lock(c->mu);
  GemmArgs g{};
  g.a = xq;
  g.b = reinterpret_cast<const int8_t*>(c->w + w_off);
  g.M = t;
  g.N = n;
  g.K = k;
  g.n_store = n;
  g.xs = xs;
  g.ws = ws;
  g.ws_vec = ws_vec;
  g.bias = bias;
  g.ldo = n;
  g.err = c->err_dev;
  if (mode == 0) {
    g.out = out;
    g.epi = EPI_F32;
    return gemm_run(g, stream);
  }
  if (mode == 3) {
    g.out_i32 = out_i32;
    g.epi = EPI_I32;
    return gemm_run(g, stream);
  }
  // re-quant modes: fp32 staging + per-row |max|, then quantise with that max
  const size_t need = static_cast<size_t>(t) * n * sizeof(float);
  if (need > c->scratch_bytes || static_cast<size_t>(t) > c->rowmax_n) {
    if (is_capturing(stream)) return -5;
    cudaStreamSynchronize(stream);
    if (need > c->scratch_bytes) {
      float* ns = nullptr;
      if (cudaMalloc(&ns, need + need / 2) != cudaSuccess) return -5;
      cudaFree(c->scratch);
      c->scratch = ns;
      c->scratch_bytes = need + need / 2;
    }
    if (static_cast<size_t>(t) > c->rowmax_n) {
      unsigned* nr = nullptr;
      if (cudaMalloc(&nr, static_cast<size_t>(t) * 2 * sizeof(unsigned)) != cudaSuccess) return -5;
      cudaFree(c->rowmax);
      c->rowmax = nr;
      c->rowmax_n = static_cast<size_t>(t) * 2;
    }
  }
  if (cudaMemsetAsync(c->rowmax, 0, static_cast<size_t>(t) * sizeof(unsigned), stream) != cudaSuccess) return -4;
  g.out = c->scratch;
  g.rowmax = c->rowmax;
  g.epi = mode == 2 ? EPI_GELU_ROWMAX : EPI_F32_ROWMAX;
  int rc = gemm_run(g, stream);
  if (rc) return rc;
  return launch_quant_rows_max(c->scratch, t, n, c->rowmax, out_q, out_s, stream);
}

extern "C" {

int wp_gemm(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
            size_t bias_off, float* out) {
  const float* bias = nullptr;
  if (c && bias_off != static_cast<size_t>(-1)) {
    if (bias_off + static_cast<size_t>(n) * 4 > c->w_bytes) return -2;
    bias = reinterpret_cast<const float*>(c->w + bias_off);
  }
  return gemm_impl(c, xq, xs, t, k, w_off, n, ws, nullptr, bias, c ? c->call_stream : nullptr, out, nullptr, nullptr,
                   nullptr, 0);
}

int wp_gemm2(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
             const float* bias_dev, void* stream, float* out) {
  return gemm_impl(c, xq, xs, t, k, w_off, n, ws, nullptr, bias_dev, static_cast<cudaStream_t>(stream), out, nullptr,
                   nullptr, nullptr, 0);
}

int wp_gemm_q(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
              const float* bias_dev, void* stream, int8_t* out_q, float* out_s) {
  if (!out_q) return -1;
  return gemm_impl(c, xq, xs, t, k, w_off, n, ws, nullptr, bias_dev, static_cast<cudaStream_t>(stream), nullptr,
                   out_q, out_s, nullptr, 1);
}

int wp_gemm_qg(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
               const float* bias_dev, void* stream, int8_t* out_q, float* out_s) {
  if (!out_q) return -1;
  return gemm_impl(c, xq, xs, t, k, w_off, n, ws, nullptr, bias_dev, static_cast<cudaStream_t>(stream), nullptr,
                   out_q, out_s, nullptr, 2);
}

int wp_gemm2_pc(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, const float* ws_dev,
                const float* bias_dev, void* stream, float* out) {
  if (!ws_dev) return -1;
  return gemm_impl(c, xq, xs, t, k, w_off, n, 0.0f, ws_dev, bias_dev, static_cast<cudaStream_t>(stream), out,
                   nullptr, nullptr, nullptr, 0);
}

int wp_gemm_i32(WpCtx* c, const int8_t* xq, int t, int k, size_t w_off, int n, void* stream, int32_t* acc) {
  return gemm_impl(c, xq, nullptr, t, k, w_off, n, 0.0f, nullptr, nullptr, static_cast<cudaStream_t>(stream),
                   nullptr, nullptr, nullptr, acc, 3);
}

}  // extern "C"

// ------------------------------------------------------------------------ no-allocation GEMM+quant
// Some callers cannot allocate device memory at the time they run a GEMM.  An embedding process
// may have handed the whole GPU to its own caching allocator up front, so that a cudaMalloc
// outside that pool fails; a latency-bound caller (the audio thread of a streaming recogniser)
// must not block, and cudaMalloc / cudaFree may synchronise the device and wait on the driver.
// wp_gemm_q grows its fp32 staging buffer on demand; wp_gemm_q_noalloc instead stages through
// this fixed array, which every GPU that loads the library holds until the process exits:
// WP_NOALLOC_MAX_ELEMS fp32 values of GEMM output (t*n <= 1,048,576, 4 MiB) followed by
// WP_NOALLOC_MAX_ROWS per-row maxima (t <= 4096).
static __device__ __align__(256) float g_noalloc_scratch[WP_NOALLOC_MAX_ELEMS + WP_NOALLOC_MAX_ROWS];

// Device address of g_noalloc_scratch on each device.  In host code the array's name is only a
// host-side stand-in, so the address is looked up with cudaGetSymbolAddress once per device,
// with that device current (the caller holds a DeviceScope for it).
static std::mutex g_noalloc_mu;
static float* g_noalloc_addr[64] = {};

static int noalloc_scratch(int dev, float** out) {
  if (dev < 0 || dev >= 64) return -23;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      fprintf(stderr, "[wasr] wp_gemm_q_noalloc: cudaGetSymbolAddress failed: %s\n", cudaGetErrorString(e));
      cudaGetLastError();
      return -23;
    }
    g_noalloc_addr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_addr[dev];
  return 0;
}

extern "C" {

int wp_gemm_q_noalloc(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
                      const float* bias_dev, void* stream, int8_t* out_q, float* out_s) {
  if (!c || !xq || !xs || !out_q || !out_s) return -1;
  if (t <= 0 || k <= 0 || n <= 0) return 0;
  if (static_cast<size_t>(n) * static_cast<size_t>(k) > c->w_bytes ||
      w_off > c->w_bytes - static_cast<size_t>(n) * static_cast<size_t>(k))
    return -2;
  if (t > WP_NOALLOC_MAX_ROWS || static_cast<size_t>(t) * static_cast<size_t>(n) > WP_NOALLOC_MAX_ELEMS) {
    fprintf(stderr,
            "[wasr] wp_gemm_q_noalloc: t=%d, n=%d exceeds the static scratch (t <= %d, t*n <= %d); "
            "use wp_gemm_q\n",
            t, n, WP_NOALLOC_MAX_ROWS, WP_NOALLOC_MAX_ELEMS);
    return -22;
  }
  // the weights, the error word and the scratch all live on the context's device
  DeviceScope on(c->dev);
  if (!on.ok()) return -23;
  float* scratch = nullptr;
  if (const int rc = noalloc_scratch(c->dev, &scratch)) return rc;
  unsigned* rowmax = reinterpret_cast<unsigned*>(scratch + WP_NOALLOC_MAX_ELEMS);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(c->mu);
  // the array keeps the previous call's values: the row maxima must start from zero
  if (cudaMemsetAsync(rowmax, 0, static_cast<size_t>(t) * sizeof(unsigned), st) != cudaSuccess) return -4;
  GemmArgs g{};
  g.a = xq;
  g.b = reinterpret_cast<const int8_t*>(c->w + w_off);
  g.M = t;
  g.N = n;
  g.K = k;
  g.n_store = n;
  g.xs = xs;
  g.ws = ws;
  g.bias = bias_dev;
  g.ldo = n;
  g.err = c->err_dev;
  g.out = scratch;
  g.rowmax = rowmax;
  g.epi = EPI_F32_ROWMAX;
  const int rc = gemm_run(g, st);
  if (rc) return rc;
  return launch_quant_rows_max(scratch, t, n, rowmax, out_q, out_s, st);
}

// Failure-handling test hook: one int32 GEMM whose producer warp issues no loads, so the MMA
// and epilogue warps' mbarrier waits run out after wait_ns with no copy or MMA in flight; the
// kernel records ERR_WAIT_* in the context's error word, releases its TMEM and returns, and
// the next wp_sync reports -21.
int wp_gemm_i32_wait_probe(WpCtx* c, const int8_t* xq, int t, int k, size_t w_off, int n, void* stream,
                           int32_t* acc, unsigned long long wait_ns) {
  if (!c || !xq || !acc) return -1;
  if (t <= 0 || k <= 0 || n <= 0) return 0;
  if (wait_ns == 0 || wait_ns > 1000000000ull || k % 16 != 0) return -2;  // the tcgen05 path only
  if (static_cast<size_t>(n) * static_cast<size_t>(k) > c->w_bytes ||
      w_off > c->w_bytes - static_cast<size_t>(n) * static_cast<size_t>(k))
    return -2;
  std::lock_guard<std::mutex> lock(c->mu);
  GemmArgs g{};
  g.a = xq;
  g.b = reinterpret_cast<const int8_t*>(c->w + w_off);
  g.M = t;
  g.N = n;
  g.K = k;
  g.n_store = n;
  g.ldo = n;
  g.err = c->err_dev;
  g.out_i32 = acc;
  g.epi = EPI_I32;
  g.wait_ns = wait_ns;
  g.idle_producer = 1;
  return gemm_run(g, static_cast<cudaStream_t>(stream));
}

int wp_quant_rows(const float* y, int t, int n, void* stream, int8_t* out_q, float* out_s) {
  if (!y || !out_q || !out_s) return -1;
  if (t <= 0 || n <= 0) return 0;
  if (n > 65536) return -7;
  return launch_quant_rows(y, t, n, n, out_q, out_s, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------------ CUDA graphs
int wp_capture_begin(WpCtx* c) {
  if (c == nullptr) return -1;
  const int rc = c->open_capture();
  if (rc != 0 && c->capturing) fprintf(stderr, "[wasr] wp_capture_begin: a capture is already open\n");
  return rc;
}

int wp_capture_end(WpCtx* c, void** out_exec) {
  if (c == nullptr || out_exec == nullptr) return -1;
  cudaGraphExec_t exec = nullptr;
  const int rc = c->close_capture(&exec);
  *out_exec = rc == 0 ? static_cast<void*>(exec) : nullptr;
  return rc;
}

int wp_replay(WpCtx* c, void* exec) {
  if (c == nullptr || exec == nullptr) return -1;
  return cuda_ok(cudaGraphLaunch(static_cast<cudaGraphExec_t>(exec), c->call_stream)) ? 0 : -17;
}

int wp_graph_free(WpCtx*, void* exec) {
  if (exec == nullptr) return 0;
  return cuda_ok(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(exec))) ? 0 : -18;
}

size_t wp_graph_count(WpCtx* c) { return c == nullptr ? 0 : c->last_graph_nodes; }
int wp_is_capturing(WpCtx* c) { return (c != nullptr && c->capturing) ? 1 : 0; }

}  // extern "C"
