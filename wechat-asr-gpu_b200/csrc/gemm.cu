// gemm.cu -- host side of the tcgen05 int8 GEMM: tensor-map encoding (cached), tile-shape
// choice and launch.  Replaces the reference's cuBLASLt descriptor / heuristic / on-disk
// algorithm cache (csrc/wtlgpu.cu:48-200,397-504): tile shapes are compile-time here, so
// there is nothing to search and nothing to warm up.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <unordered_map>

#include "gemm.cuh"

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
  int rows, k, box;
  bool operator==(const MapKey& o) const { return p == o.p && rows == o.rows && k == o.k && box == o.box; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uintptr_t>()(k.p) ^ (static_cast<size_t>(k.rows) * 0x9E3779B97F4A7C15ull) ^
           (static_cast<size_t>(k.k) << 20) ^ static_cast<size_t>(k.box);
  }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// Tensor map of an int8 [rows][k] row-major matrix, box = 128 bytes of K x `box` rows,
// 128-byte swizzle (the UMMA K-major SW128 canonical layout), zero fill out of bounds.
bool tensor_map(const void* p, int rows, int k, int box, CUtensorMap* out) {
  MapKey key{reinterpret_cast<uintptr_t>(p), rows, k, box};
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return true;
    }
  }
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k)};
  cuuint32_t boxd[2] = {128u, static_cast<cuuint32_t>(box)};
  cuuint32_t estr[2] = {1u, 1u};
  CUtensorMap m;
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(p), dims, strides, boxd, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
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
template <int BN, int EPI>
bool ensure_attr() {
  static unsigned done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (done & (1u << (dev & 31))) return true;
  if (cudaFuncSetAttribute(gemm_i8_tc<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<BN>::SMEM) !=
      cudaSuccess)
    return false;
  done |= 1u << (dev & 31);
  return true;
}

template <int EPI>
bool prepare_epi() {
  return ensure_attr<256, EPI>() && ensure_attr<128, EPI>() && ensure_attr<64, EPI>();
}

template <int BN, int EPI>
int launch_tc(const GemmArgs& g, cudaStream_t s) {
  CUtensorMap ta, tb;
  if (!tensor_map(g.a, g.M, g.K, 128, &ta) || !tensor_map(g.b, g.N, g.K, BN, &tb)) return -4;
  constexpr int smem = TcCfg<BN>::SMEM;
  if (!ensure_attr<BN, EPI>()) return -4;
  const int tiles = ((g.n_store + BN - 1) / BN) * ((g.M + 127) / 128);
  gemm_i8_tc<BN, EPI><<<std::min(tiles, num_sms()), TcCfg<BN>::THREADS, smem, s>>>(ta, tb, g);
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
  // widest N tile that still fills every SM once; narrow tiles for small (per-window) M
  const int tm = (g.M + 127) / 128, sms = num_sms();
  auto ctas = [&](int bn) { return tm * ((g.n_store + bn - 1) / bn); };
  if (ctas(256) >= sms) return launch_tc<256, EPI>(g, s);
  if (ctas(128) >= sms) return launch_tc<128, EPI>(g, s);
  return launch_tc<64, EPI>(g, s);
}

}  // namespace

bool gemm_prepare() {
  gemm_init();
  return prepare_epi<EPI_F32>() && prepare_epi<EPI_F32_ADD>() && prepare_epi<EPI_I32>() &&
         prepare_epi<EPI_F32_ROWMAX>() && prepare_epi<EPI_GELU_ROWMAX>() && prepare_epi<EPI_ARGMAX>();
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
  }
  return -1;
}

}  // namespace wasr
