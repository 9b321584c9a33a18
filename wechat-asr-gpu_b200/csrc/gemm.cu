// gemm.cu -- host side of the tcgen05 int8 GEMM: tensor-map encoding (cached), tile-shape
// choice and launch.  Replaces the reference's cuBLASLt descriptor / heuristic / on-disk
// algorithm cache (csrc/wtlgpu.cu:48-200,397-504): tile shapes are compile-time here, so
// there is nothing to search and nothing to warm up.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <cstdio>
#include <mutex>
#include <unordered_map>

#include "gemm.cuh"
#include "gemm_gq.cuh"

namespace wasr {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

bool gemm_init() {
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}

namespace {

struct MapKey {
  uintptr_t p;
  int rows, cols, ld, box_rows, kind;  // kind 0: int8 operand, 1: fp32 / int32 output
  bool operator==(const MapKey& o) const {
    return p == o.p && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows && kind == o.kind;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uintptr_t>()(k.p) ^ (static_cast<size_t>(k.rows) * 0x9E3779B97F4A7C15ull) ^
           (static_cast<size_t>(k.cols) << 20) ^ (static_cast<size_t>(k.ld) << 40) ^
           static_cast<size_t>(k.box_rows * 2 + k.kind);
  }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// Tensor maps, cached by (pointer, shape, kind).  Both kinds use 128-byte boxes with 128-byte
// swizzle and zero fill out of bounds:
//   kind 0: int8 operand [rows][cols = K], box 128 (K) x box_rows -- the UMMA K-major SW128 layout;
//   kind 1: 32-bit output [rows][cols] with row stride ld elements, box 32 x 32 -- the epilogue's
//           staging layout (stores are clipped to rows x cols).
bool tensor_map(const void* p, int rows, int cols, int ld, int box_rows, int kind, CUtensorMap* out) {
  MapKey key{reinterpret_cast<uintptr_t>(p), rows, cols, ld, box_rows, kind};
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return true;
    }
  }
  const int esize = kind == 0 ? 1 : 4;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esize};
  cuuint32_t boxd[2] = {static_cast<cuuint32_t>(128 / esize), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUtensorMap m;
  CUresult r = g_encode(&m, kind == 0 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                        const_cast<void*>(p), dims, strides, boxd, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lk(g_map_mu);
  if (g_maps.size() > 8192) g_maps.clear();
  g_maps.emplace(key, m);
  *out = m;
  return true;
}

int num_sms() {
  static int sms[32] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& n = sms[dev & 31];
  if (!n) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Opt the kernel into its dynamic shared memory once per device (outside any capture: the
// host entry points call gemm_prepare() at context / model creation).
template <int BN, int EPI, int EW = 8>
bool ensure_attr() {
  static unsigned done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (done & (1u << (dev & 31))) return true;
  if (cudaFuncSetAttribute(gemm_i8_tc<BN, EPI, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           TcCfg<BN, EPI, EW>::SMEM) != cudaSuccess)
    return false;
  done |= 1u << (dev & 31);
  return true;
}

template <int EPI>
bool prepare_epi() {
  return ensure_attr<256, EPI>() && ensure_attr<128, EPI>() && ensure_attr<64, EPI>() &&
         (EPI != EPI_F32_ADD || ensure_attr<128, EPI, 4>());
}

template <int BN, int EPI, int EW = 8>
int launch_tc(const GemmArgs& g0, cudaStream_t s) {
  CUtensorMap ta, tb, to;
  if (!tensor_map(g0.a, g0.M, g0.K, g0.K, 128, 0, &ta) || !tensor_map(g0.b, g0.N, g0.K, g0.K, BN, 0, &tb)) return -4;
  GemmArgs g = g0;
  // output blocks move by TMA when the output rows are 16-byte aligned
  void* obase = EPI == EPI_I32 ? static_cast<void*>(g.out_i32) : static_cast<void*>(g.out);
  g.tma_out = EPI != EPI_ARGMAX && obase && (reinterpret_cast<uintptr_t>(obase) % 16 == 0) && (g.ldo % 4 == 0) &&
              tensor_map(obase, g.M, g.n_store, g.ldo, 32, 1, &to);
  if (!g.tma_out) memset(&to, 0, sizeof(to));
  constexpr int smem = TcCfg<BN, EPI, EW>::SMEM;
  if (!ensure_attr<BN, EPI, EW>()) return -4;
  const int tiles = ((g.n_store + BN - 1) / BN) * ((g.M + 127) / 128);
  gemm_i8_tc<BN, EPI, EW><<<std::min(tiles, num_sms()), TcCfg<BN, EPI, EW>::THREADS, smem, s>>>(ta, tb, to, g);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

template <int EPI>
int launch_epi(const GemmArgs& g, cudaStream_t s) {
  const bool tma_ok = g_encode && (g.K % 16 == 0) && (reinterpret_cast<uintptr_t>(g.a) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(g.b) % 16 == 0);
  if (!tma_ok) {
    dim3 grid((g.n_store + 31) / 32, (g.M + 7) / 8);
    gemm_i8_simt<EPI><<<grid, 256, 0, s>>>(g);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
  }
  // widest N tile that still fills every SM once; narrow tiles for small (per-window) M.  The
  // 256-wide tile takes four tiles per SM: a persistent CTA overlaps one tile's epilogue with
  // the next tile's loads and MMAs, and at few 256-wide tiles per CTA the fill and the last
  // epilogue stay exposed (measured on 8,802 rows at 128: qkv 1.03 -> 0.87, f1 1.14 -> 1.01 ms
  // per step)
  const int tm = (g.M + 127) / 128, sms = num_sms();
  auto ctas = [&](int bn) { return tm * ((g.n_store + bn - 1) / bn); };
  // (the residual epilogue keeps 3 staging blocks per warp: at BN=256 only 2 ring stages fit)
  if (EPI != EPI_F32_ADD && ctas(256) >= 4 * sms) return launch_tc<256, EPI>(g, s);
  // a long K keeps the tensor pipe busy longer than the residual epilogue: 4 epilogue warps
  // leave shared memory for 5 ring stages instead of 3
  if (EPI == EPI_F32_ADD && g.K >= 1024 && ctas(128) >= sms) return launch_tc<128, EPI, 4>(g, s);
  if (ctas(128) >= sms) return launch_tc<128, EPI>(g, s);
  return launch_tc<64, EPI>(g, s);
}

bool ensure_gq_attr() {
  static unsigned done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (done & (1u << (dev & 31))) return true;
  if (cudaFuncSetAttribute(gemm_i8_gelu_q, cudaFuncAttributeMaxDynamicSharedMemorySize, GqCfg::SMEM) != cudaSuccess)
    return false;
  done |= 1u << (dev & 31);
  return true;
}

}  // namespace

bool gemm_gq_supported(const GemmArgs& g) {
  const uintptr_t al = reinterpret_cast<uintptr_t>(g.a) | reinterpret_cast<uintptr_t>(g.b) |
                       reinterpret_cast<uintptr_t>(g.q_out);
  return gemm_init() && g.K % GqCfg::BK == 0 && g.K <= 2048 && g.n_store == g.N && g.N % GqCfg::BN == 0 &&
         g.N <= GqCfg::NMAX && g.q_out && g.q_scale && g.fix && (al & 15) == 0;
}

namespace {

// f1 + GELU + row quantisation (gemm_gq.cuh): the fused kernel, then the exact kernel for the
// rows it listed.  Shapes it does not take return -1 (gemm_gq_supported says which).
int launch_gq(const GemmArgs& g, cudaStream_t s) {
  if (!gemm_gq_supported(g)) return -1;
  CUtensorMap ta, tb;
  if (!tensor_map(g.a, g.M, g.K, g.K, 128, 0, &ta) || !tensor_map(g.b, g.N, g.K, g.K, GqCfg::BN, 0, &tb)) return -4;
  if (!ensure_gq_attr()) return -4;
  if (cudaMemsetAsync(g.fix, 0, sizeof(int), s) != cudaSuccess) return -4;
  const int blocks = (g.M + GqCfg::BM - 1) / GqCfg::BM;
  gemm_i8_gelu_q<<<std::min(blocks, num_sms()), GqCfg::THREADS, GqCfg::SMEM, s>>>(ta, tb, g);
  gelu_q_rows_exact_k<<<std::min(g.M, 2 * num_sms()), 256, 0, s>>>(g);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace

bool gemm_prepare() {
  gemm_init();
  return prepare_epi<EPI_F32>() && prepare_epi<EPI_F32_ADD>() && prepare_epi<EPI_I32>() &&
         prepare_epi<EPI_F32_ROWMAX>() && prepare_epi<EPI_GELU_ROWMAX>() && prepare_epi<EPI_ARGMAX>() &&
         ensure_gq_attr();
}

int gemm_run(const GemmArgs& g, cudaStream_t s) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0 || g.n_store <= 0) return 0;
  gemm_init();
  switch (g.epi) {
    case EPI_F32: return launch_epi<EPI_F32>(g, s);
    case EPI_F32_ADD: return launch_epi<EPI_F32_ADD>(g, s);
    case EPI_I32: return launch_epi<EPI_I32>(g, s);
    case EPI_F32_ROWMAX: return launch_epi<EPI_F32_ROWMAX>(g, s);
    case EPI_GELU_ROWMAX: return launch_epi<EPI_GELU_ROWMAX>(g, s);
    case EPI_ARGMAX: return launch_epi<EPI_ARGMAX>(g, s);
    case EPI_GELU_Q: return launch_gq(g, s);
  }
  return -1;
}

// Dense int8 tensor-core throughput probe: one CTA per SM, one elected thread issues `iters`
// rounds of 4 back-to-back tcgen05.mma kind::i8 (M = 128, N = 256, K = 32; 2 * 128 * 256 * 128
// ops a round) from fixed 128B-swizzled shared-memory tiles into two alternating TMEM
// accumulators, with no loads at all, then waits (bounded) for their completion.  Operand values
// do not affect the rate.  The denominator for the int8 GEMMs' tensor-core fractions.
constexpr int I8_PEAK_SMEM = 120 * 1024;  // more than the tiles need: keeps one CTA per SM
__global__ void __launch_bounds__(128, 1) i8_mma_peak_k(int iters, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;           // [128 rows][128 B]
  uint8_t* sB = smem + 16384;   // [256 rows][128 B]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sB + 32768);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  for (int i = tid; i < 49152 / 4; i += 128) reinterpret_cast<uint32_t*>(smem)[i] = 0x01010101u * (i & 7);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();  // the operand stores before the tensor core reads them
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (tid == 0) {
    constexpr uint32_t idesc = idesc_i8(256);
    const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
    for (int it = 0; it < iters; it++) {
      const uint32_t d = tmem + static_cast<uint32_t>((it & 1) * 256);
#pragma unroll
      for (int kk = 0; kk < 4; kk++)
        mma_i8(d, desc_sw128(a0 + kk * 32), desc_sw128(b0 + kk * 32), idesc, (it >= 2 || kk > 0) ? 1u : 0u);
    }
    mma_commit(bar);
    if (!mbar_wait(bar, 0)) atomicExch(err, ERR_WAIT_ACC);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace wasr

extern "C" int wasr_i8_mma_peak(int iters, int ctas, int* err, void* stream) {
  using namespace wasr;
  if (iters <= 0 || ctas <= 0 || err == nullptr) return -1;
  static unsigned done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(done & (1u << (dev & 31)))) {
    if (cudaFuncSetAttribute(i8_mma_peak_k, cudaFuncAttributeMaxDynamicSharedMemorySize, I8_PEAK_SMEM) != cudaSuccess)
      return -4;
    done |= 1u << (dev & 31);
  }
  i8_mma_peak_k<<<ctas, 128, I8_PEAK_SMEM, static_cast<cudaStream_t>(stream)>>>(iters, err);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}
