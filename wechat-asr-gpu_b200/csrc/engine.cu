// engine.cu -- the batched transcription engine behind include/wasr.h.
//
// The reference runs one window per forward (Model::run_gpu, src/model.rs:546-619: upload
// feats, conv frontend, quant, linear, 40 x window_ops, output GEMM, argmax, download ids)
// and one utterance at a time (src/bin/wasr.rs:147-169).  Here many windows -- the k-th
// window of every utterance in flight -- are stacked along the row axis of every GEMM, so
// the int8 GEMMs see M = sum of t1 instead of t1 <= 400, while the conv frontend and
// attention stay inside each window (segment tables).  The op sequence per layer follows
// window_ops (src/model.rs:522-541) / run_post (src/model.rs:488-502), with these fusions:
//   q/k/v         : one GEMM over the contiguous [1536][512] weight block (per-column scale)
//   o, f2         : residual add fused into the GEMM epilogue (h += ...)
//   f1            : bias in the GEMM epilogue; GELU + row |max| + quant in one row kernel that
//                   never writes the GELU values back
//   output layer  : GEMM fused with the argmax (logits never written unless asked for)
// A whole chunk of windows is captured once in a CUDA graph and replayed when the same
// window layout comes back (the reference graphs one window per t1, src/model.rs:576-604).
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/wasr.h"
#include "gemm.cuh"
#include "kern.cuh"

using namespace wasr;

namespace {

constexpr size_t kMaxGraphs = 64;

struct Chunk {
  int w0, w1;        // windows [w0, w1) of the call
  int frames, rows;  // totals over the chunk
  int max_t1;
  int tiles;         // attention query tiles
};

struct Rec {
  int cat;
  cudaEvent_t a, b;
};

struct GraphEntry {
  cudaGraphExec_t exec = nullptr;
  int* seg = nullptr;  // device copy of this layout's segment tables
  uint64_t use = 0;
  int64_t kernels = 0;  // kernel nodes in the graph
  std::vector<Rec> recs;
};

}  // namespace

struct WasrModel {
  int dev = 0;
  cudaStream_t own = nullptr, stream = nullptr;
  uint8_t* w = nullptr;
  size_t w_bytes = 0;
  WasrPlan plan{};
  int max_rows = 0, max_frames = 0;
  // q/k/v fused: per-column scale (and bias) vectors over the [1536] output
  float* qkv_scale[WASR_MAX_LAYERS] = {};
  float* qkv_bias[WASR_MAX_LAYERS] = {};
  bool qkv_fused[WASR_MAX_LAYERS] = {};
  // activations
  float *feats = nullptr, *y1 = nullptr, *y2 = nullptr;
  Conv1W c1w{};             // conv1 weights on the host: conv1w_k takes them by value
  float* c2pre = nullptr;   // conv2 weights transposed to [tap][out] (the position-pair kernel)
  float* c3cert = nullptr;  // conv3 weights transposed for conv3_cert_k, and their row norms
  int8_t* xq = nullptr;
  float* xs = nullptr;
  float *h = nullptr, *qkv = nullptr, *att = nullptr, *f = nullptr;
  unsigned* rowmax = nullptr;
  unsigned long long* keys = nullptr;
  uint32_t* ids = nullptr;
  int* seg = nullptr;  // segment tables of eager runs: foff | roff | toff | tord
  int seg_cap = 0;
  int* err_host = nullptr;
  int* err_dev = nullptr;
  // second branch of a chunk's forward (small chunks run as two halves that overlap)
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  bool graphs = true;
  bool prof = false;
  int64_t launches = 0;
  std::vector<Rec> eager_recs;
  uint64_t tick = 0;
  std::unordered_map<std::string, GraphEntry> graph_cache;
  // pinned host staging
  float* h_feats = nullptr;
  size_t h_feats_cap = 0;
  // device staging of wasr_transcribe_device: one round's gathered windows and their table
  float* d_win = nullptr;
  size_t d_win_cap = 0;
  long long* d_wtab = nullptr;
  size_t d_wtab_cap = 0;
  uint32_t* h_ids = nullptr;
  size_t h_ids_cap = 0;
  int* h_seg = nullptr;
  size_t h_seg_cap = 0;
  std::mutex mu;
};

namespace {

template <typename T>
bool dmalloc(T** p, size_t n) {
  return cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(n, 1) * sizeof(T)) == cudaSuccess;
}

template <typename T>
bool hgrow(T** p, size_t* cap, size_t n) {
  if (n <= *cap) return true;
  if (*p) cudaFreeHost(*p);
  *p = nullptr;
  *cap = 0;
  if (cudaHostAlloc(reinterpret_cast<void**>(p), n * sizeof(T), cudaHostAllocDefault) != cudaSuccess) return false;
  *cap = n;
  return true;
}

// device buffer of at least n elements (contents not kept); callers grow it only while the
// model's stream is idle
template <typename T>
bool dgrow(T** p, size_t* cap, size_t n) {
  if (n <= *cap) return true;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  if (cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T)) != cudaSuccess) {
    *p = nullptr;
    return false;
  }
  *cap = n;
  return true;
}

// engine-internal forward flag: feats on the device, ids / logits on the host
constexpr int F_FEATS_DEV = 1 << 16;

struct DevGuard {
  int prev = -1;
  explicit DevGuard(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
  }
  ~DevGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

inline int t1_of(int t) { return t >= 5 ? (t - 5) / 5 + 1 : 0; }

const float* fptr(const WasrModel* m, uint64_t off) {
  return off == WASR_NONE ? nullptr : reinterpret_cast<const float*>(m->w + off);
}

// Chunks of at least this many rows run f1 + GELU + quant as one fused kernel (100 row blocks
// of 128: two thirds of a wave of 148 SMs and more).
constexpr int kFusedGeluRows = 12800;

GemmArgs gemm_args(WasrModel* m, const int8_t* a, const float* xs, int M, int K, const WasrMat& q, int N,
                   uint64_t bias, int epi, float* out, int ldo) {
  GemmArgs g{};
  g.a = a;
  g.b = reinterpret_cast<const int8_t*>(m->w + q.off);
  g.M = M;
  g.N = N;
  g.K = K;
  g.n_store = N;
  g.xs = xs;
  g.ws = q.s;
  g.ws_vec = fptr(m, q.scale_off);
  g.bias = fptr(m, bias);
  g.out = out;
  g.ldo = ldo;
  g.err = m->err_dev;
  g.epi = epi;
  return g;
}

#define TRY(x)           \
  do {                   \
    int rc_ = (x);       \
    if (rc_) return rc_; \
  } while (0)

void free_recs(std::vector<Rec>* r) {
  for (Rec& x : *r) {
    cudaEventDestroy(x.a);
    cudaEventDestroy(x.b);
  }
  r->clear();
}

// Counts every kernel enqueued and, when recs != nullptr, brackets it with an event pair.
struct Launcher {
  WasrModel* m;
  std::vector<Rec>* recs;
  int64_t kernels = 0;
  template <typename F>
  int operator()(int cat, F&& f) {
    Rec r{cat, nullptr, nullptr};
    // during stream capture a plain record only becomes a dependency edge; the External flag
    // makes it a real event-record node that is timed at every replay (profiling runs every
    // chunk on the model's stream alone)
    if (recs) {
      if (cudaEventCreate(&r.a) != cudaSuccess || cudaEventCreate(&r.b) != cudaSuccess) return -4;
      cudaEventRecordWithFlags(r.a, m->stream, cudaEventRecordExternal);
    }
    const int rc = f();
    if (recs) {
      cudaEventRecordWithFlags(r.b, m->stream, cudaEventRecordExternal);
      recs->push_back(r);
    }
    kernels++;
    return rc;
  }
};

// Enqueue the whole forward of windows c on stream st.  Their frames are at m->feats + fo
// frames; every per-row buffer is used from row ro on (so two halves of a chunk can run at once
// on their own rows); seg points at their device segment tables [foff n+1 | roff n+1 | toff
// n+1 | tord tiles].
int enqueue_chunk(WasrModel* m, const Chunk& c, const int* seg, float* logits, Launcher& K, cudaStream_t st,
                  int64_t fo, int64_t ro) {
  const int n = c.w1 - c.w0;
  float* const feats = m->feats + fo * DIM;
  float* const y1 = m->y1 + fo * C1 * DIM;
  float* const y2 = m->y2 + ro * C2 * W2;
  int8_t* const xq = m->xq + ro * FLAT;
  float* const xs = m->xs + ro;
  float* const hh = m->h + ro * D;
  float* const qkv = m->qkv + ro * 3 * D;
  float* const att = m->att + ro * D;
  float* const ff = m->f + ro * FF;
  unsigned long long* const keys = m->keys + ro;
  uint32_t* const ids = m->ids + ro;
  Segs s{};
  s.foff = seg;
  s.roff = seg + (n + 1);
  s.n = n;
  const int* toff = seg + 2 * (n + 1);
  const int* tord = seg + 3 * (n + 1);
  const int M = c.rows;
  const WasrPlan& P = m->plan;
  // conv frontend -> int8 rows of y3 -> linear (src/model.rs:389-478,489)
  TRY(K(WASR_K_CONV1, [&] { return launch_conv1_w(feats, m->c1w, s, c.frames, y1, st); }));
  TRY(K(WASR_K_CONV2, [&] { return launch_conv2(y1, fptr(m, P.c2), m->c2pre, s, M, y2, st); }));
  // conv3 with its row quantisation fused and certified (int8 rows identical to quant(conv3))
  TRY(K(WASR_K_CONV3, [&] { return launch_conv3_cert(y2, fptr(m, P.c3), m->c3cert, s, M, xq, xs, st); }));
  TRY(K(WASR_K_GEMM_LIN, [&] { return gemm_run(gemm_args(m, xq, xs, M, FLAT, P.lin, D, P.lin_b, EPI_F32, hh, D), st); }));
  for (int l = 0; l < P.n_layers; l++) {
    const WasrLayer& L = P.layers[l];
    // prior norm -> q, k, v
    TRY(K(WASR_K_LN, [&] { return launch_ln_quant(hh, nullptr, fptr(m, L.pn_g), fptr(m, L.pn_b), M, xq, xs, st); }));
    if (m->qkv_fused[l]) {
      GemmArgs g = gemm_args(m, xq, xs, M, D, L.q, 3 * D, WASR_NONE, EPI_F32, qkv, 3 * D);
      g.ws_vec = m->qkv_scale[l];
      g.bias = m->qkv_bias[l];
      TRY(K(WASR_K_GEMM_QKV, [&] { return gemm_run(g, st); }));
    } else {
      const WasrMat* pm[3] = {&L.q, &L.k, &L.v};
      const uint64_t pb[3] = {L.qb, L.kb, L.vb};
      for (int p = 0; p < 3; p++)
        TRY(K(WASR_K_GEMM_QKV, [&] {
          return gemm_run(gemm_args(m, xq, xs, M, D, *pm[p], D, pb[p], EPI_F32, qkv + p * D, 3 * D), st);
        }));
    }
    // attention -> quant -> o projection, residual fused (src/model.rs:493)
    TRY(K(WASR_K_ATTN, [&] { return launch_attention(qkv, qkv + D, qkv + 2 * D, 3 * D, s, toff, tord, c.tiles, c.max_t1, att, D, st); }));
    TRY(K(WASR_K_QUANT, [&] { return launch_quant_rows(att, M, D, D, xq, xs, st); }));
    TRY(K(WASR_K_GEMM_O, [&] { return gemm_run(gemm_args(m, xq, xs, M, D, L.o, D, L.ob, EPI_F32_ADD, hh, D), st); }));
    // middle norm -> f1 + bias + GELU (+ row max) -> quant -> f2 + bias, residual fused
    TRY(K(WASR_K_LN, [&] { return launch_ln_quant(hh, nullptr, fptr(m, L.mn_g), fptr(m, L.mn_b), M, xq, xs, st); }));
    // f1, GELU and the row quantisation in one kernel (gemm_gq.cuh) for chunks of at least
    // kFusedGeluRows rows: its int8 rows, scales and exact-row list take the place of the fp32 f1
    // output in the ff region.  It runs one CTA per 128-row block, so a small chunk leaves SMs
    // idle and the two-kernel path is faster (measured: 8,802 rows 15.69 against 16.72 ms per
    // step, 17,329 rows 29.13 against 28.84)
    int8_t* const q2 = reinterpret_cast<int8_t*>(ff);
    float* const s2 = reinterpret_cast<float*>(q2 + static_cast<size_t>(M) * FF);
    GemmArgs g1 = gemm_args(m, xq, xs, M, D, L.f1, FF, L.f1b, EPI_GELU_Q, nullptr, FF);
    g1.q_out = q2;
    g1.q_scale = s2;
    g1.fix = reinterpret_cast<int*>(s2 + M);
    if (M >= kFusedGeluRows && gemm_gq_supported(g1)) {
      TRY(K(WASR_K_GEMM_F1, [&] { return gemm_run(g1, st); }));
      TRY(K(WASR_K_GEMM_F2, [&] { return gemm_run(gemm_args(m, q2, s2, M, FF, L.f2, D, L.f2b, EPI_F32_ADD, hh, D), st); }));
    } else {  // f1's fp32 output, then the certified GELU + quant kernel
      TRY(K(WASR_K_GEMM_F1, [&] {
        return gemm_run(gemm_args(m, xq, xs, M, D, L.f1, FF, L.f1b, EPI_F32, ff, FF), st);
      }));
      TRY(K(WASR_K_GELU, [&] { return launch_gelu_quant_ro(ff, M, FF, xq, xs, st); }));
      TRY(K(WASR_K_GEMM_F2, [&] { return gemm_run(gemm_args(m, xq, xs, M, FF, L.f2, D, L.f2b, EPI_F32_ADD, hh, D), st); }));
    }
  }
  // output layer + argmax (src/model.rs:498-501)
  TRY(K(WASR_K_QUANT, [&] { return launch_quant_rows(hh, M, D, D, xq, xs, st); }));
  if (logits) {
    TRY(K(WASR_K_GEMM_OUT, [&] { return gemm_run(gemm_args(m, xq, xs, M, D, P.out, P.out_n, P.out_b, EPI_F32, logits, P.out_n), st); }));
    TRY(K(WASR_K_IDS, [&] { return launch_argmax_rows(logits, M, P.out_n, ids, st); }));
  } else {
    if (cudaMemsetAsync(keys, 0, static_cast<size_t>(M) * sizeof(unsigned long long), st) != cudaSuccess)
      return -4;
    GemmArgs g = gemm_args(m, xq, xs, M, D, P.out, P.out_n, P.out_b, EPI_ARGMAX, nullptr, P.out_n);
    g.keys = keys;
    TRY(K(WASR_K_GEMM_OUT, [&] { return gemm_run(g, st); }));
    TRY(K(WASR_K_IDS, [&] { return launch_keys_to_ids(keys, M, ids, st); }));
  }
  return 0;
}

// segment tables of windows [w0, w1): foff | roff | toff (each n+1 ints) | tord (one int per
// attention tile: the tiles in launch order, longest segment first, so the longest blocks
// start in the first wave)
void build_seg(const int32_t* t, int w0, int w1, int* out) {
  const int n = w1 - w0;
  int* fo = out;
  int* ro = out + n + 1;
  int* to = out + 2 * (n + 1);
  int* tord = out + 3 * (n + 1);
  fo[0] = ro[0] = to[0] = 0;
  for (int i = 0; i < n; i++) {
    const int tt = std::max(0, t[w0 + i]);
    const int t1 = t1_of(tt);
    fo[i + 1] = fo[i] + tt;
    ro[i + 1] = ro[i] + t1;
    to[i + 1] = to[i] + (t1 + ATT_QT - 1) / ATT_QT;
  }
  std::vector<int> order(n);
  for (int i = 0; i < n; i++) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return ro[a + 1] - ro[a] > ro[b + 1] - ro[b]; });
  int k = 0;
  for (int i : order)
    for (int tl = to[i]; tl < to[i + 1]; tl++) tord[k++] = tl;
}

// split windows into chunks that fit the activation buffers
bool plan_chunks(const WasrModel* m, const int32_t* t, int n, std::vector<Chunk>* out) {
  out->clear();
  int i = 0;
  while (i < n) {
    Chunk c{i, i, 0, 0, 0, 0};
    while (c.w1 < n) {
      const int tt = std::max(0, t[c.w1]);
      const int t1 = t1_of(tt);
      if (tt > m->max_frames || t1 > m->max_rows) return false;  // one window alone too big
      if (c.frames + tt > m->max_frames || c.rows + t1 > m->max_rows) break;
      c.frames += tt;
      c.rows += t1;
      c.max_t1 = std::max(c.max_t1, t1);
      c.tiles += (t1 + ATT_QT - 1) / ATT_QT;
      c.w1++;
    }
    out->push_back(c);
    i = c.w1;
  }
  return true;
}

std::string layout_key(const int32_t* t, const Chunk& c, bool logits) {
  std::string k;
  k.reserve((c.w1 - c.w0) * 4 + 2);
  k.push_back(logits ? 'L' : 'I');
  k.append(reinterpret_cast<const char*>(t + c.w0), (c.w1 - c.w0) * sizeof(int32_t));
  return k;
}

void free_graphs(WasrModel* m) {
  for (auto& kv : m->graph_cache) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.seg) cudaFree(kv.second.seg);
    free_recs(&kv.second.recs);
  }
  m->graph_cache.clear();
}

// A chunk of at least this many rows runs as two halves of its windows on two streams (one graph
// with two branches), so that each kernel's last partial wave overlaps the other half's work
// (measured: 71,599 rows 115.2 -> 114.7 ms per forward; below this size the halves' smaller
// kernels lose more than the overlap gains: 8,802 rows 16.2 -> 17.3 ms).
constexpr int kSplitRows = 40000;

// windows [w0, w1) as one chunk's totals
Chunk chunk_of(const int32_t* t, int w0, int w1) {
  Chunk c{w0, w1, 0, 0, 0, 0};
  for (int i = w0; i < w1; i++) {
    const int tt = std::max(0, t[i]), t1 = t1_of(tt);
    c.frames += tt;
    c.rows += t1;
    c.max_t1 = std::max(c.max_t1, t1);
    c.tiles += (t1 + ATT_QT - 1) / ATT_QT;
  }
  return c;
}
size_t seg_ints_of(const Chunk& c) { return 3 * static_cast<size_t>(c.w1 - c.w0 + 1) + static_cast<size_t>(c.tiles); }

// the halves of a chunk split by rows (false: no split)
bool split_halves(const WasrModel* m, const int32_t* t, const Chunk& c, bool logits, Chunk* a, Chunk* b) {
  if (logits || m->prof || c.rows < kSplitRows || c.w1 - c.w0 < 2) return false;
  int rows = 0, w = c.w0;
  while (w < c.w1 - 1 && 2 * (rows + t1_of(std::max(0, t[w]))) <= c.rows) rows += t1_of(std::max(0, t[w++]));
  if (w == c.w0) w = c.w0 + 1;
  *a = chunk_of(t, c.w0, w);
  *b = chunk_of(t, w, c.w1);
  return a->rows > 0 && b->rows > 0;
}

// Enqueue chunk c (seg: its device tables; for a split chunk the two halves' tables back to
// back) on m->stream, the second half on m->side between a fork and a join event.
int enqueue_forward(WasrModel* m, const int32_t* t, const Chunk& c, const int* seg, float* logits, Launcher& K) {
  Chunk a, b;
  cudaStream_t st = m->stream;
  if (!split_halves(m, t, c, logits != nullptr, &a, &b)) return enqueue_chunk(m, c, seg, logits, K, st, 0, 0);
  if (cudaEventRecord(m->ev_fork, st) != cudaSuccess || cudaStreamWaitEvent(m->side, m->ev_fork, 0) != cudaSuccess)
    return -4;
  const int ra = enqueue_chunk(m, a, seg, nullptr, K, st, 0, 0);
  const int rb = ra ? 0 : enqueue_chunk(m, b, seg + seg_ints_of(a), nullptr, K, m->side, a.frames, a.rows);
  // always join, so that a capture in progress ends with both branches merged
  const bool joined = cudaEventRecord(m->ev_join, m->side) == cudaSuccess &&
                      cudaStreamWaitEvent(st, m->ev_join, 0) == cudaSuccess;
  return ra ? ra : rb ? rb : joined ? 0 : -4;
}
// host segment tables of chunk c, split like enqueue_forward
size_t build_tables(const WasrModel* m, const int32_t* t, const Chunk& c, bool logits, int* out) {
  Chunk a, b;
  if (!split_halves(m, t, c, logits, &a, &b)) {
    build_seg(t, c.w0, c.w1, out);
    return seg_ints_of(c);
  }
  build_seg(t, a.w0, a.w1, out);
  build_seg(t, b.w0, b.w1, out + seg_ints_of(a));
  return seg_ints_of(a) + seg_ints_of(b);
}

// Run one chunk (frames already in m->feats): replay its graph if this layout was seen,
// else capture it (graphs on) or run it eagerly.
int run_chunk(WasrModel* m, const int32_t* t, const Chunk& c, float* logits) {
  const int n = c.w1 - c.w0;
  // (a split chunk's two tables hold one more entry per table than the whole chunk's)
  const size_t seg_ints = 3 * static_cast<size_t>(n + 1) + static_cast<size_t>(c.tiles) + 3;
  if (!hgrow(&m->h_seg, &m->h_seg_cap, seg_ints)) return -5;
  cudaStream_t st = m->stream;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  const bool use_graph = m->graphs && logits == nullptr && cs == cudaStreamCaptureStatusNone;
  if (use_graph) {
    const std::string key = layout_key(t, c, false);
    auto it = m->graph_cache.find(key);
    if (it == m->graph_cache.end()) {
      if (m->graph_cache.size() >= kMaxGraphs) {
        auto lru = m->graph_cache.begin();
        for (auto i2 = m->graph_cache.begin(); i2 != m->graph_cache.end(); ++i2)
          if (i2->second.use < lru->second.use) lru = i2;
        cudaStreamSynchronize(st);
        if (lru->second.exec) cudaGraphExecDestroy(lru->second.exec);
        if (lru->second.seg) cudaFree(lru->second.seg);
        free_recs(&lru->second.recs);
        m->graph_cache.erase(lru);
      }
      GraphEntry e;
      if (!dmalloc(&e.seg, seg_ints)) return -5;
      build_tables(m, t, c, false, m->h_seg);
      if (cudaMemcpy(e.seg, m->h_seg, seg_ints * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(e.seg);
        return -4;
      }
      if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaFree(e.seg);
        cudaGetLastError();
        return -10;
      }
      Launcher K{m, m->prof ? &e.recs : nullptr};
      const int rc = enqueue_forward(m, t, c, e.seg, nullptr, K);
      e.kernels = K.kernels;
      cudaGraph_t g = nullptr;
      const cudaError_t ee = cudaStreamEndCapture(st, &g);
      if (rc || ee != cudaSuccess || !g) {
        if (g) cudaGraphDestroy(g);
        cudaFree(e.seg);
        free_recs(&e.recs);
        cudaGetLastError();
        return rc ? rc : -13;
      }
      const cudaError_t ie = cudaGraphInstantiate(&e.exec, g, 0);
      cudaGraphDestroy(g);
      if (ie != cudaSuccess) {
        cudaFree(e.seg);
        free_recs(&e.recs);
        cudaGetLastError();
        return -15;
      }
      it = m->graph_cache.emplace(key, e).first;
    }
    it->second.use = ++m->tick;
    m->launches += it->second.kernels;
    return cudaGraphLaunch(it->second.exec, st) == cudaSuccess ? 0 : -17;
  }
  // eager: per-call segment tables
  if (static_cast<size_t>(m->seg_cap) < seg_ints) {
    cudaStreamSynchronize(st);
    if (m->seg) cudaFree(m->seg);
    m->seg = nullptr;
    m->seg_cap = 0;
    if (!dmalloc(&m->seg, seg_ints * 2)) return -5;
    m->seg_cap = static_cast<int>(seg_ints * 2);
  }
  build_tables(m, t, c, logits != nullptr, m->h_seg);
  if (cudaMemcpyAsync(m->seg, m->h_seg, seg_ints * sizeof(int), cudaMemcpyHostToDevice, st) != cudaSuccess)
    return -4;
  cudaStreamSynchronize(st);  // the previous eager chunk's events may still be pending
  free_recs(&m->eager_recs);
  Launcher K{m, m->prof ? &m->eager_recs : nullptr};
  const int rc = enqueue_forward(m, t, c, m->seg, logits, K);
  m->launches += K.kernels;
  // the pinned table is reused by the next chunk: make sure this copy has consumed it
  cudaStreamSynchronize(st);
  return rc;
}

int device_error(WasrModel* m) {
  const int e = *reinterpret_cast<volatile int*>(m->err_host);
  if (e) {
    *m->err_host = 0;
    return -21;
  }
  return 0;
}

// forward over windows whose frames are at feats (host or device per flags)
int forward_impl(WasrModel* m, const float* feats, const int32_t* t, int n, uint32_t* ids, float* logits, int flags) {
  if (!m || !t || n < 0 || (!feats && n > 0) || !ids) return -1;
  if (n == 0) return 0;
  std::vector<Chunk> chunks;
  if (!plan_chunks(m, t, n, &chunks)) return -2;
  const bool on_dev = flags & WASR_F_DEVICE;
  cudaStream_t st = m->stream;
  int64_t f_off = 0, r_off = 0;
  for (const Chunk& c : chunks) {
    const size_t fbytes = static_cast<size_t>(c.frames) * DIM * sizeof(float);
    if (fbytes) {
      const float* src = feats + f_off * DIM;
      if (on_dev || (flags & F_FEATS_DEV)) {
        if (cudaMemcpyAsync(m->feats, src, fbytes, cudaMemcpyDeviceToDevice, st) != cudaSuccess) return -4;
      } else {
        if (cudaMemcpyAsync(m->feats, src, fbytes, cudaMemcpyHostToDevice, st) != cudaSuccess) return -4;
      }
    }
    float* lo = nullptr;
    if (logits) lo = logits + r_off * m->plan.out_n;
    float* lo_dev = lo;
    if (logits && !on_dev) lo_dev = nullptr;  // host logits: computed into m->f-sized scratch below
    if (logits && !on_dev) {
      if (!dmalloc(&lo_dev, static_cast<size_t>(c.rows) * m->plan.out_n)) return -5;
    }
    TRY(run_chunk(m, t, c, lo_dev));
    const size_t ibytes = static_cast<size_t>(c.rows) * sizeof(uint32_t);
    if (ibytes) {
      const cudaMemcpyKind kind = on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
      if (cudaMemcpyAsync(ids + r_off, m->ids, ibytes, kind, st) != cudaSuccess) return -4;
    }
    if (logits && !on_dev) {
      const size_t lb = static_cast<size_t>(c.rows) * m->plan.out_n * sizeof(float);
      cudaMemcpyAsync(lo, lo_dev, lb, cudaMemcpyDeviceToHost, st);
      cudaStreamSynchronize(st);
      cudaFree(lo_dev);
    }
    // the next chunk overwrites m->feats / m->ids: host copies must have landed
    if (!on_dev || chunks.size() > 1) cudaStreamSynchronize(st);
    f_off += c.frames;
    r_off += c.rows;
  }
  if (!(flags & WASR_F_NOSYNC) || !on_dev) {
    if (cudaStreamSynchronize(st) != cudaSuccess) return -4;
    return device_error(m);
  }
  return 0;
}

}  // namespace

// ============================================================================ host fbank
// src/fbank.rs restated for the product (feature extraction feeding the window schedule):
#include "fbank.cuh"  // the host fbank (fb::frame) and its tables

// ============================================================================ C ABI
extern "C" {

const char* wasr_version(void) { return "wasr-b200 engine 1.0 (batched ragged windows; sm_100a)"; }

// Parity hook for the engine's fused f1 + GELU + row quantisation (see include/wasr.h).
int wasr_gemm_gelu_quant(const int8_t* a, const float* xs, const int8_t* w, float ws, const float* ws_vec,
                         const float* bias, int M, int K, int N, int8_t* q, float* qs, int* work, void* stream) {
  if (!a || !xs || !w || !q || !qs || !work || M < 0 || K <= 0 || N <= 0) return -1;
  if (M == 0) return 0;
  if (!gemm_init()) return -4;
  GemmArgs g{};
  g.a = a;
  g.b = w;
  g.M = M;
  g.N = N;
  g.K = K;
  g.n_store = N;
  g.xs = xs;
  g.ws = ws;
  g.ws_vec = ws_vec;
  g.bias = bias;
  g.err = work;
  g.epi = EPI_GELU_Q;
  g.q_out = q;
  g.q_scale = qs;
  g.fix = work + 1;
  return gemm_run(g, static_cast<cudaStream_t>(stream));
}

// Failure-handling probe of the fused kernel: its producer issues no loads, so the MMA warp's wait
// for the first k-block runs out after wait_ns with nothing in flight; the kernel records the
// error code in work[0], releases its tensor memory and returns.
int wasr_gemm_gelu_quant_wait_probe(const int8_t* a, const float* xs, const int8_t* w, float ws, const float* ws_vec,
                                    const float* bias, int M, int K, int N, int8_t* q, float* qs, int* work,
                                    unsigned long long wait_ns, void* stream) {
  if (!a || !xs || !w || !q || !qs || !work || M <= 0 || K <= 0 || N <= 0) return -1;
  if (wait_ns == 0 || wait_ns > 1000000000ull) return -2;
  if (!gemm_init()) return -4;
  GemmArgs g{};
  g.a = a;
  g.b = w;
  g.M = M;
  g.N = N;
  g.K = K;
  g.n_store = N;
  g.xs = xs;
  g.ws = ws;
  g.ws_vec = ws_vec;
  g.bias = bias;
  g.err = work;
  g.epi = EPI_GELU_Q;
  g.q_out = q;
  g.q_scale = qs;
  g.fix = work + 1;
  g.wait_ns = wait_ns;
  g.idle_producer = 1;
  return gemm_run(g, static_cast<cudaStream_t>(stream));
}

WasrModel* wasr_model_create(const void* blob, size_t bytes, const WasrPlan* plan, int device, int max_rows) {
  if (!blob || !bytes || !plan || max_rows <= 0) return nullptr;
  if (plan->n_layers < 0 || plan->n_layers > WASR_MAX_LAYERS || plan->out_n <= 0) return nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return nullptr;
  DevGuard dg(device);
  gemm_prepare();
  kern_prepare();
  WasrModel* m = new WasrModel();
  m->dev = device;
  m->plan = *plan;
  m->max_rows = max_rows;
  m->max_frames = 5 * max_rows + 4 * std::max(1, max_rows / 20);  // t = 5*t1 + 0..4 per window
  bool ok = cudaStreamCreateWithFlags(&m->own, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&m->side, cudaStreamNonBlocking) == cudaSuccess &&
            cudaEventCreateWithFlags(&m->ev_fork, cudaEventDisableTiming) == cudaSuccess &&
            cudaEventCreateWithFlags(&m->ev_join, cudaEventDisableTiming) == cudaSuccess;
  m->stream = m->own;
  ok = ok && cudaHostAlloc(reinterpret_cast<void**>(&m->err_host), sizeof(int), cudaHostAllocMapped) == cudaSuccess;
  ok = ok && cudaHostGetDevicePointer(reinterpret_cast<void**>(&m->err_dev), m->err_host, 0) == cudaSuccess;
  if (ok) *m->err_host = 0;
  m->w_bytes = bytes;
  ok = ok && dmalloc(&m->w, bytes) && cudaMemcpy(m->w, blob, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
  ok = ok && plan->c1 <= bytes && bytes - plan->c1 >= sizeof(m->c1w.w);
  if (ok) std::memcpy(m->c1w.w, static_cast<const uint8_t*>(blob) + plan->c1, sizeof(m->c1w.w));
  const size_t R = static_cast<size_t>(max_rows), Fr = static_cast<size_t>(m->max_frames);
  ok = ok && dmalloc(&m->feats, Fr * DIM) && dmalloc(&m->y1, Fr * C1 * DIM) && dmalloc(&m->y2, R * C2 * W2) &&
       dmalloc(&m->xq, R * FLAT) && dmalloc(&m->xs, R) && dmalloc(&m->h, R * D) &&
       dmalloc(&m->qkv, R * 3 * D) && dmalloc(&m->att, R * D) && dmalloc(&m->f, R * FF) &&
       dmalloc(&m->rowmax, R) && dmalloc(&m->keys, R) && dmalloc(&m->ids, R);
  // q/k/v fusion: the three [512][512] matrices must sit back to back in the blob
  for (int l = 0; ok && l < plan->n_layers; l++) {
    const WasrLayer& L = plan->layers[l];
    const uint64_t mat = static_cast<uint64_t>(D) * D;
    if (L.k.off != L.q.off + mat || L.v.off != L.k.off + mat) continue;
    std::vector<float> sc(3 * D), bs(3 * D, 0.0f);
    const WasrMat* qs[3] = {&L.q, &L.k, &L.v};
    const uint64_t bo[3] = {L.qb, L.kb, L.vb};
    bool any_bias = false;
    for (int p = 0; p < 3; p++) {
      if (qs[p]->scale_off != WASR_NONE)
        std::memcpy(&sc[p * D], static_cast<const uint8_t*>(blob) + qs[p]->scale_off, D * sizeof(float));
      else
        std::fill(sc.begin() + p * D, sc.begin() + (p + 1) * D, qs[p]->s);
      if (bo[p] != WASR_NONE) {
        std::memcpy(&bs[p * D], static_cast<const uint8_t*>(blob) + bo[p], D * sizeof(float));
        any_bias = true;
      }
    }
    ok = ok && dmalloc(&m->qkv_scale[l], 3 * D) &&
         cudaMemcpy(m->qkv_scale[l], sc.data(), 3 * D * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess;
    if (ok && any_bias)
      ok = dmalloc(&m->qkv_bias[l], 3 * D) &&
           cudaMemcpy(m->qkv_bias[l], bs.data(), 3 * D * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess;
    m->qkv_fused[l] = ok;
  }
  // conv2 / conv3 weights in the per-stage layout their kernels stage from (once per model)
  ok = ok && dmalloc(&m->c2pre, conv2_prepare_floats()) && dmalloc(&m->c3cert, conv3_cert_prep_floats()) &&
       conv2_prepare(fptr(m, plan->c2), m->c2pre, m->stream) == 0 &&
       conv3_cert_prepare(fptr(m, plan->c3), m->c3cert, m->stream) == 0 &&
       cudaStreamSynchronize(m->stream) == cudaSuccess;
  if (!ok) {
    wasr_model_destroy(m);
    return nullptr;
  }
  return m;
}

void wasr_model_destroy(WasrModel* m) {
  if (!m) return;
  DevGuard dg(m->dev);
  cudaDeviceSynchronize();
  free_graphs(m);
  free_recs(&m->eager_recs);
  void* dptrs[] = {m->w, m->feats, m->y1, m->y2, m->xq, m->xs, m->h, m->qkv, m->att, m->f, m->rowmax,
                   m->keys, m->ids, m->seg, m->c2pre, m->c3cert, m->d_win, m->d_wtab};
  for (void* p : dptrs)
    if (p) cudaFree(p);
  for (int l = 0; l < WASR_MAX_LAYERS; l++) {
    if (m->qkv_scale[l]) cudaFree(m->qkv_scale[l]);
    if (m->qkv_bias[l]) cudaFree(m->qkv_bias[l]);
  }
  if (m->h_feats) cudaFreeHost(m->h_feats);
  if (m->h_ids) cudaFreeHost(m->h_ids);
  if (m->h_seg) cudaFreeHost(m->h_seg);
  if (m->err_host) cudaFreeHost(m->err_host);
  if (m->own) cudaStreamDestroy(m->own);
  if (m->side) cudaStreamDestroy(m->side);
  if (m->ev_fork) cudaEventDestroy(m->ev_fork);
  if (m->ev_join) cudaEventDestroy(m->ev_join);
  delete m;
}

int wasr_model_set_stream(WasrModel* m, void* stream) {
  if (!m) return -1;
  std::lock_guard<std::mutex> lk(m->mu);
  DevGuard dg(m->dev);
  cudaStreamSynchronize(m->stream);
  m->stream = stream ? static_cast<cudaStream_t>(stream) : m->own;
  return 0;
}

void* wasr_model_stream(WasrModel* m) { return m ? static_cast<void*>(m->stream) : nullptr; }

int wasr_model_set_graphs(WasrModel* m, int on) {
  if (!m) return -1;
  std::lock_guard<std::mutex> lk(m->mu);
  DevGuard dg(m->dev);
  m->graphs = on != 0;
  if (!m->graphs) {
    cudaStreamSynchronize(m->stream);
    free_graphs(m);
  }
  return 0;
}

int wasr_model_set_profile(WasrModel* m, int on) {
  if (!m) return -1;
  std::lock_guard<std::mutex> lk(m->mu);
  DevGuard dg(m->dev);
  cudaStreamSynchronize(m->stream);
  if (m->prof != (on != 0)) free_graphs(m);
  m->prof = on != 0;
  return 0;
}

int wasr_model_profile(WasrModel* m, double* ms, int64_t* launches, int ncat) {
  if (!m || !ms || !launches || ncat <= 0) return -1;
  std::lock_guard<std::mutex> lk(m->mu);
  DevGuard dg(m->dev);
  if (cudaStreamSynchronize(m->stream) != cudaSuccess) return -4;
  for (int i = 0; i < ncat; i++) {
    ms[i] = 0.0;
    launches[i] = 0;
  }
  int failed = 0;
  cudaError_t first_err = cudaSuccess;
  auto add = [&](const std::vector<Rec>& recs) {
    for (const Rec& r : recs) {
      float t = 0.0f;
      const cudaError_t e = r.cat < ncat ? cudaEventElapsedTime(&t, r.a, r.b) : cudaErrorInvalidValue;
      if (e == cudaSuccess) {
        ms[r.cat] += t;
        launches[r.cat]++;
      } else if (!failed++) {
        first_err = e;
      }
    }
  };
  for (auto& kv : m->graph_cache) add(kv.second.recs);
  add(m->eager_recs);
  cudaGetLastError();  // events of graphs not yet replayed report "not ready"
  if (failed && getenv("WASR_DEBUG"))
    fprintf(stderr, "[wasr] profile: %d event pairs not timed (%s)\n", failed, cudaGetErrorString(first_err));
  return 0;
}

int64_t wasr_model_kernel_launches(WasrModel* m) { return m ? m->launches : -1; }

int wasr_model_error(WasrModel* m) {
  if (!m) return -1;
  const int e = *reinterpret_cast<volatile int*>(m->err_host);
  *m->err_host = 0;
  return e;
}

int wasr_forward(WasrModel* m, const float* feats, const int32_t* t, int n_win, uint32_t* ids, float* logits,
                 int flags) {
  if (!m) return -1;
  std::lock_guard<std::mutex> lk(m->mu);
  DevGuard dg(m->dev);
  return forward_impl(m, feats, t, n_win, ids, logits, flags & (WASR_F_DEVICE | WASR_F_NOSYNC));
}

int64_t wasr_fbank(const int16_t* pcm, int64_t n, float* feats, int64_t cap, float* sil) {
  using namespace fb;
  if (!pcm && n > 0) return -1;
  const int64_t nfr = n >= WIN ? (n - WIN) / HOP + 1 : 0;
  if (!feats) return nfr;
  if (nfr > cap) return -1;
  std::vector<double> raw(static_cast<size_t>(std::max<int64_t>(nfr, 1)) * DIM);
  (void)tables();
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < nfr; k++) frame(pcm + k * HOP, raw.data() + k * DIM);
  double sum[DIM] = {0};
  int64_t hn = 0;
  for (int64_t k = 0; k < nfr; k++) {
    const double* f = raw.data() + k * DIM;
    if (hn == CMS_WIN) {
      const double* o = raw.data() + (k - CMS_WIN) * DIM;
      for (int i = 0; i < DIM; i++) sum[i] -= o[i];
      hn--;
    }
    hn++;
    for (int i = 0; i < DIM; i++) sum[i] += f[i];
    const double nn = static_cast<double>(hn > 0 ? hn : 1);
    for (int i = 0; i < DIM; i++) feats[k * DIM + i] = static_cast<float>(f[i] - sum[i] / nn);
  }
  if (sil) {
    double s[DIM] = {0};
    s[NCH] = std::log(1e-10);
    const double nn = static_cast<double>(hn > 0 ? hn : 1);
    for (int i = 0; i < DIM; i++) sil[i] = static_cast<float>(s[i] - sum[i] / nn);
  }
  return nfr;
}

// Streaming fbank (src/fbank.rs:122-161 Fbank): PCM arrives in pieces; a push emits the frames
// its samples complete, each normalised by the rolling mean as it stands after that frame, and
// the silence frame uses the rolling mean as it stands now.  The same frame() and CMS order as
// wasr_fbank, so the frames of any split of a signal equal wasr_fbank's frames of the whole.
struct WasrFbank {
  std::vector<int16_t> buf;                  // samples not yet consumed by a frame hop
  std::deque<std::vector<double>> hist;      // raw frames in the rolling window (<= CMS_WIN)
  double sum[fb::FDIM] = {0};
};

WasrFbank* wasr_fbank_stream_create() { return new (std::nothrow) WasrFbank(); }
void wasr_fbank_stream_destroy(WasrFbank* st) { delete st; }

int64_t wasr_fbank_stream_pending(const WasrFbank* st, int64_t n) {
  if (!st || n < 0) return -1;
  const int64_t have = static_cast<int64_t>(st->buf.size()) + n;
  return have >= fb::WIN ? (have - fb::WIN) / fb::HOP + 1 : 0;
}

int64_t wasr_fbank_stream_push(WasrFbank* st, const int16_t* pcm, int64_t n, float* feats, int64_t cap) {
  using namespace fb;
  if (!st || n < 0 || (!pcm && n > 0)) return -1;
  const int64_t nfr = wasr_fbank_stream_pending(st, n);
  if (nfr > 0 && (!feats || nfr > cap)) return -1;  // nothing is consumed
  st->buf.insert(st->buf.end(), pcm, pcm + n);
  if (nfr == 0) return 0;
  std::vector<double> raw(static_cast<size_t>(nfr) * FDIM);
  (void)tables();
  if (nfr >= 16) {  // frames are independent: parallel like the reference's rayon path
#pragma omp parallel for schedule(static)
    for (int64_t k = 0; k < nfr; k++) frame(st->buf.data() + k * HOP, raw.data() + k * FDIM);
  } else {
    for (int64_t k = 0; k < nfr; k++) frame(st->buf.data() + k * HOP, raw.data() + k * FDIM);
  }
  for (int64_t k = 0; k < nfr; k++) {  // the rolling mean, in frame order
    const double* f = raw.data() + k * FDIM;
    if (static_cast<int>(st->hist.size()) == CMS_WIN) {
      const std::vector<double>& o = st->hist.front();
      for (int i = 0; i < FDIM; i++) st->sum[i] -= o[i];
      st->hist.pop_front();
    }
    st->hist.emplace_back(f, f + FDIM);
    for (int i = 0; i < FDIM; i++) st->sum[i] += f[i];
    const double nn = static_cast<double>(st->hist.size());
    for (int i = 0; i < FDIM; i++) feats[k * FDIM + i] = static_cast<float>(f[i] - st->sum[i] / nn);
  }
  st->buf.erase(st->buf.begin(), st->buf.begin() + nfr * HOP);
  return nfr;
}

int wasr_fbank_stream_silence(const WasrFbank* st, float* sil) {
  using namespace fb;
  if (!st || !sil) return -1;
  double s[FDIM] = {0};
  s[NCH] = std::log(1e-10);
  const double nn = static_cast<double>(st->hist.empty() ? 1 : st->hist.size());
  for (int i = 0; i < FDIM; i++) sil[i] = static_cast<float>(s[i] - st->sum[i] / nn);
  return 0;
}

int64_t wasr_ctc_collapse(const uint32_t* ids, int64_t n, uint32_t* out) {
  if ((!ids || !out) && n > 0) return -1;
  int64_t k = 0;
  uint32_t prev = 0xFFFFFFFFu;
  for (int64_t i = 0; i < n; i++) {
    if (ids[i] != prev && ids[i] != 0) out[k++] = ids[i];
    prev = ids[i];
  }
  return k;
}

}  // extern "C"

namespace {

// One block per window of a device transcription round (tab: 5 entries per window): frames
// [src, src + n) of the features, then `pad` copies of utterance u's silence frame, written to
// rows dst, dst + 1, ... of out.
__global__ void gather_windows_k(const float* __restrict__ feats, const float* __restrict__ sil,
                                 const long long* __restrict__ tab, float* __restrict__ out) {
  const long long* e = tab + 5 * static_cast<long long>(blockIdx.x);
  const long long src = e[0], n = e[1], pad = e[2], u = e[3], dst = e[4];
  const long long total = (n + pad) * DIM;
  for (long long i = threadIdx.x; i < total; i += blockDim.x) {
    const long long r = i / DIM, c = i - r * DIM;
    out[(dst + r) * DIM + c] = r < n ? feats[(src + r) * DIM + c] : sil[u * DIM + c];
  }
}

// Batch transcription (src/stream.rs:58-70 push, 128-134 decode, 136-147 commit, 159-168
// finish).  Every utterance keeps its own commit position; each round stacks one window per
// unfinished utterance into a single forward.  dev: feats and sil are device pointers, and a
// round's windows are gathered on the device instead of in pinned host staging.
int transcribe_impl(WasrModel* m, const float* feats, const int64_t* n_frames, const float* sil, int n_utt, int prev,
                    int blk, int post, uint32_t* ids, int64_t* ids_off, int64_t ids_cap, bool dev) {
  if (!m || !n_frames || !sil || !ids || !ids_off || n_utt < 0 || (!feats && n_utt > 0)) return -1;
  if (prev < 0 || blk <= 0 || post < 0) return -1;
  std::lock_guard<std::mutex> lk(m->mu);
  DevGuard dg(m->dev);
  std::vector<int64_t> start(n_utt + 1, 0);
  for (int u = 0; u < n_utt; u++) start[u + 1] = start[u] + std::max<int64_t>(0, n_frames[u]);
  struct U {
    int64_t s = 0;
    bool done = false;
    std::vector<uint32_t> out;
  };
  std::vector<U> st(n_utt);
  // windows of the current round
  struct Win {
    int u;
    int64_t a, end;  // frames [a, end) of utterance u, then `pad` silence frames
    int pad;
    int kind;        // 0 whole, 1 commit, 2 finish tail
  };
  for (;;) {
    std::vector<Win> wins;
    for (int u = 0; u < n_utt; u++) {
      U& x = st[u];
      if (x.done) continue;
      const int64_t n = std::max<int64_t>(0, n_frames[u]);
      if (n <= WASR_WHOLE_MAX) {  // finish(): whole utterance, no pad (commits are discarded)
        wins.push_back({u, 0, n, 0, 0});
      } else if (n >= x.s + blk + post) {
        wins.push_back({u, x.s > prev ? x.s - prev : 0, x.s + blk + post, WASR_PAD, 1});
      } else if (n > x.s) {
        wins.push_back({u, x.s > prev ? x.s - prev : 0, n, WASR_PAD, 2});
      } else {
        x.done = true;
      }
    }
    if (wins.empty()) break;
    // assemble frames into pinned staging; a round made only of whole utterances laid out
    // back to back in the caller's array is copied straight from it
    std::vector<int32_t> tv(wins.size());
    int64_t total = 0;
    for (size_t i = 0; i < wins.size(); i++) {
      tv[i] = static_cast<int32_t>(wins[i].end - wins[i].a + wins[i].pad);
      total += tv[i];
    }
    bool contiguous = true;
    for (size_t i = 0; i < wins.size() && contiguous; i++)
      contiguous = wins[i].kind == 0 && (i == 0 ? start[wins[i].u] == 0 : start[wins[i].u] == start[wins[i - 1].u] +
                                                                              (wins[i - 1].end - wins[i - 1].a));
    const float* src = feats;
    std::vector<long long> wtab;  // device rounds: src, n, pad, u, dst per window
    if (!contiguous && dev) {
      wtab.resize(5 * wins.size());
      int64_t d = 0;
      for (size_t i = 0; i < wins.size(); i++) {
        const Win& w = wins[i];
        long long* e = wtab.data() + 5 * i;
        e[0] = start[w.u] + w.a;
        e[1] = w.end - w.a;
        e[2] = w.pad;
        e[3] = w.u;
        e[4] = d;
        d += tv[i];
      }
      if (!dgrow(&m->d_win, &m->d_win_cap, static_cast<size_t>(std::max<int64_t>(total, 1)) * DIM) ||
          !dgrow(&m->d_wtab, &m->d_wtab_cap, wtab.size()))
        return -5;
      if (cudaMemcpyAsync(m->d_wtab, wtab.data(), wtab.size() * sizeof(long long), cudaMemcpyHostToDevice,
                          m->stream) != cudaSuccess)
        return -4;
      gather_windows_k<<<static_cast<unsigned>(wins.size()), 256, 0, m->stream>>>(feats, sil, m->d_wtab, m->d_win);
      if (cudaPeekAtLastError() != cudaSuccess) return -4;
      src = m->d_win;
    } else if (!contiguous) {
      if (!hgrow(&m->h_feats, &m->h_feats_cap, static_cast<size_t>(total) * DIM)) return -5;
      float* d = m->h_feats;
      for (const Win& w : wins) {
        const float* uf = feats + start[w.u] * DIM;
        std::memcpy(d, uf + w.a * DIM, static_cast<size_t>(w.end - w.a) * DIM * sizeof(float));
        d += (w.end - w.a) * DIM;
        for (int p = 0; p < w.pad; p++, d += DIM) std::memcpy(d, sil + static_cast<int64_t>(w.u) * DIM, DIM * 4);
      }
      src = m->h_feats;
    }
    int64_t rows = 0;
    for (int32_t tt : tv) rows += t1_of(tt);
    if (!hgrow(&m->h_ids, &m->h_ids_cap, static_cast<size_t>(std::max<int64_t>(rows, 1)))) return -5;
    TRY(forward_impl(m, src, tv.data(), static_cast<int>(wins.size()), m->h_ids, nullptr, dev ? F_FEATS_DEV : 0));
    int64_t r = 0;
    for (size_t i = 0; i < wins.size(); i++) {
      const Win& w = wins[i];
      U& x = st[w.u];
      const int64_t t1 = t1_of(tv[i]);
      const uint32_t* o = m->h_ids + r;
      r += t1;
      if (w.kind == 0) {
        x.out.assign(o, o + t1);
        x.done = true;
        continue;
      }
      const int64_t from = (x.s - w.a) / 5;
      int64_t len = t1 > from ? t1 - from : 0;
      if (w.kind == 2) {
        x.out.insert(x.out.end(), o + from, o + from + len);
        x.done = true;
        continue;
      }
      // commit: keep blk/5 frames, cut at the last blank pair of the second half
      len = std::min<int64_t>(len, blk / 5);
      for (int64_t cpos = len - 1; cpos >= len / 2 && cpos >= 1; cpos--)
        if (o[from + cpos] == 0 && o[from + cpos - 1] == 0) {
          len = cpos;
          break;
        }
      x.out.insert(x.out.end(), o + from, o + from + len);
      x.s += len * 5;
      if (len == 0) x.done = true;  // cannot advance (only reachable for blk < 10)
    }
  }
  int64_t k = 0;
  ids_off[0] = 0;
  for (int u = 0; u < n_utt; u++) {
    if (k + static_cast<int64_t>(st[u].out.size()) > ids_cap) return -20;
    std::memcpy(ids + k, st[u].out.data(), st[u].out.size() * sizeof(uint32_t));
    k += static_cast<int64_t>(st[u].out.size());
    ids_off[u + 1] = k;
  }
  return 0;
}

}  // namespace

extern "C" {

int wasr_transcribe(WasrModel* m, const float* feats, const int64_t* n_frames, const float* sil, int n_utt, int prev,
                    int blk, int post, uint32_t* ids, int64_t* ids_off, int64_t ids_cap) {
  return transcribe_impl(m, feats, n_frames, sil, n_utt, prev, blk, post, ids, ids_off, ids_cap, false);
}

int wasr_transcribe_device(WasrModel* m, const float* feats, const int64_t* n_frames, const float* sil, int n_utt,
                           int prev, int blk, int post, uint32_t* ids, int64_t* ids_off, int64_t ids_cap) {
  return transcribe_impl(m, feats, n_frames, sil, n_utt, prev, blk, post, ids, ids_off, ids_cap, true);
}

}  // extern "C"
